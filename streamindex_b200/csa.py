"""CSA layer forward on B200: ``flash_csa_forward`` and ``build_csa_topk_idxs``.

Mirrors ``flash_sparse/csa.py:30-207`` of the reference:

1. indexer + top-k over the compressed keys with the causal mask
   ``(i+1)*m - 1 <= s``  (== ``i < (s+1)//m``), -1 for empty slots,
2. index list ``[window(n_win) | compressed + S]``, built inside the
   attention kernel's index ring from the top-k output (never materialised),
3. sparse attention over ``cat[kv; kv_compressed]`` with the attention sink.

The reference picks between a materialised ``[B,S,T]`` score path and the
chunked path by a memory threshold; here step 1 always runs the fused
streaming indexer (same result, O(S*k) memory), and the concatenated kv is
never built: the attention kernel reads the window rows from ``kv`` and the
compressed rows from ``kv_compressed`` directly.  Forward only.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .attention import _csa_attn_call
from .indexer import chunked_indexer_topk, indexer_topk_slice


def sliding_window_idxs(B: int, S: int, n_win: int, device) -> torch.Tensor:
    """``[B,S,n_win]`` int32 window indices (``flash_sparse/reference.py:460-475``), built on the GPU."""
    empty = torch.empty((B, S, 0), dtype=torch.int64, device=device)
    return csa_index_list(empty, n_win)


def csa_index_list(comp_idx: torch.Tensor, n_win: int) -> torch.Tensor:
    """``[B,S,n_win+k]`` int32 from compressed top-k indices ``[B,S,k]`` (int64, -1 = empty)."""
    assert comp_idx.is_cuda and comp_idx.dim() == 3
    B, S, k = comp_idx.shape
    comp_idx = comp_idx.to(torch.int64).contiguous()
    out = torch.empty((B, S, n_win + k), dtype=torch.int32, device=comp_idx.device)
    lib = _lib.load()
    with torch.cuda.device(comp_idx.device):
        _lib.check(lib.si_csa_build_idx(comp_idx.data_ptr() if k > 0 else None, B, S, k, int(n_win), out.data_ptr(),
                                        _lib.stream_handle(comp_idx.device)))
    return out


def scores_topk(scores: torch.Tensor, top_k: int, causal_ratio: Optional[int] = None,
                causal_mask: Optional[torch.Tensor] = None):
    """Top-k (score desc, index asc) of materialised scores ``[B,S,T]`` under
    ``t < (s+1)//causal_ratio`` and/or an explicit bool mask (True = legal)."""
    assert scores.is_cuda and scores.dim() == 3
    B, S, T = scores.shape
    sc = scores.float().contiguous()
    dev = sc.device
    m = None
    if causal_mask is not None:
        m = causal_mask.to(device=dev, dtype=torch.bool).expand(B, S, T).contiguous().view(torch.uint8)
    out_i = torch.empty((B, S, top_k), dtype=torch.int64, device=dev)
    out_v = torch.empty((B, S, top_k), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        wsb = lib.si_scores_topk_ws_bytes(B, S, top_k)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        _lib.check(lib.si_scores_topk_mask(sc.data_ptr(), B, S, T, int(top_k), int(causal_ratio or 0), _lib.ptr(m),
                                           out_i.data_ptr(), out_v.data_ptr(), ws.data_ptr(), wsb,
                                           _lib.stream_handle(dev)))
    return out_i, out_v


def token_compressor(c_a, z_a, b_a, m: int, *, c_b=None, z_b=None, b_b=None, overlap: bool = False):
    """Softmax-gated compressor ``[B,S,c] -> [B,S//m,c]`` (``reference_token_compressor``,
    ``flash_sparse/reference.py:176-272``); bf16 or fp32 tensors, fp32 math."""
    assert c_a.is_cuda and c_a.dim() == 3 and z_a.shape == c_a.shape
    B, S, c = c_a.shape
    if b_a.shape != (m, c):
        raise ValueError(f"b_a must be [m={m}, c={c}], got {tuple(b_a.shape)}")
    if overlap:
        if c_b is None or z_b is None or b_b is None:
            raise ValueError("overlap=True requires c_b, z_b, b_b")
        if b_b.shape != (m, c):
            raise ValueError(f"b_b must be [m={m}, c={c}], got {tuple(b_b.shape)}")
    dt = c_a.dtype
    if dt not in (torch.bfloat16, torch.float32):
        raise ValueError(f"compressor supports bf16 and fp32 tensors, got {dt}")
    cv = lambda t: None if t is None else t.to(device=c_a.device, dtype=dt).contiguous()  # noqa: E731
    ca, za, ba, cb, zb, bb = cv(c_a), cv(z_a), cv(b_a), cv(c_b), cv(z_b), cv(b_b)
    out = torch.empty((B, S // m, c), dtype=dt, device=c_a.device)
    lib = _lib.load()
    with torch.cuda.device(c_a.device):
        _lib.check(lib.si_token_compressor(ca.data_ptr(), za.data_ptr(), ba.data_ptr(), _lib.ptr(cb), _lib.ptr(zb),
                                           _lib.ptr(bb), B, S, c, int(m), int(bool(overlap)),
                                           int(dt == torch.bfloat16), out.data_ptr(),
                                           _lib.stream_handle(c_a.device)))
    return out


def build_csa_topk_idxs(
    indexer_scores: torch.Tensor,
    n_win: int,
    top_k: int,
    *,
    seq_len: int,
    n_compressed: int,
    m: int,
    device=None,
) -> torch.Tensor:
    """``[B,S,n_win+top_k]`` int32 from materialised indexer scores (``flash_sparse/csa.py:30-83``)."""
    B, S, T = indexer_scores.shape
    assert T == n_compressed
    assert S == seq_len
    comp, _ = scores_topk(indexer_scores, top_k, causal_ratio=m)
    return csa_index_list(comp, n_win)


def mean_pool_compress(x: torch.Tensor, m: int) -> torch.Tensor:
    """``[B,S,C]`` bf16 -> ``[B,S//m,C]``: mean over blocks of m tokens (non-overlapping compressor)."""
    assert x.is_cuda and x.dim() == 3 and x.dtype == torch.bfloat16
    B, S, C = x.shape
    x = x.contiguous()
    out = torch.empty((B, S // m, C), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    with torch.cuda.device(x.device):
        _lib.check(lib.si_mean_pool(x.data_ptr(), B, S, C, int(m), out.data_ptr(), _lib.stream_handle(x.device)))
    return out


def flash_csa_forward(
    q: torch.Tensor,
    kv: torch.Tensor,
    kv_compressed: torch.Tensor,
    q_idx: torch.Tensor,
    k_idx_compressed: torch.Tensor,
    indexer_weights: torch.Tensor,
    attn_sink: torch.Tensor,
    *,
    n_win: int,
    top_k: int,
    m: int = 4,
    softmax_scale: Optional[float] = None,
    use_triton: bool = True,
    use_chunked_indexer: Optional[bool] = None,
    chunk_s: int = 1024,
    chunk_t: int = 4096,
    auto_chunk_threshold_bytes: int = 1 << 30,
    d_v: Optional[int] = None,
) -> torch.Tensor:
    """End-to-end CSA forward (prefill, one layer).  Returns ``o [B,S,n_h,d_v or d]`` bf16.

    ``use_triton`` / ``use_chunked_indexer`` / ``chunk_*`` /
    ``auto_chunk_threshold_bytes`` select among the reference's backends and
    are accepted for compatibility; every combination runs the same CUDA path.
    """
    del use_triton, use_chunked_indexer, chunk_s, chunk_t, auto_chunk_threshold_bytes
    B, S, n_h, d = q.shape
    assert kv.shape == (B, S, d)
    n_compressed = kv_compressed.shape[1]
    assert kv_compressed.shape == (B, n_compressed, d)
    assert k_idx_compressed.shape[1] == n_compressed
    if softmax_scale is None:
        softmax_scale = d ** -0.5
    comp, _ = chunked_indexer_topk(q_idx, k_idx_compressed, indexer_weights, top_k, causal_ratio=m)
    dv = d if d_v is None else int(d_v)
    o, _ = _csa_attn_call(q, kv, kv_compressed, attn_sink, comp, n_win, 0, softmax_scale, dv)
    return o


def csa_forward_slice(
    q: torch.Tensor,
    kv: torch.Tensor,
    kv_compressed: torch.Tensor,
    q_idx: torch.Tensor,
    k_idx_compressed: torch.Tensor,
    indexer_weights: torch.Tensor,
    attn_sink: torch.Tensor,
    *,
    s_offset: int,
    n_win: int,
    top_k: int,
    m: int = 4,
    softmax_scale: Optional[float] = None,
    d_v: Optional[int] = None,
    return_indices: bool = False,
):
    """CSA forward for the query slice ``[s_offset, s_offset + q.shape[1])`` of a sequence.

    ``q`` / ``q_idx`` / ``indexer_weights`` hold only the slice; ``kv`` (all
    ``S_total`` tokens), ``kv_compressed`` and ``k_idx_compressed`` are full.
    Causality, the window and the compressed offset use global positions, so
    concatenating the slices' outputs equals :func:`flash_csa_forward` on the
    whole sequence.  This is what each rank runs in the S-sharded CSA forward.
    With ``return_indices`` it also returns the slice's compressed top-k
    indices ``[B,S_loc,top_k]`` int64 (the per-rank result an index gather
    collects).
    """
    B, S_loc, n_h, d = q.shape
    if softmax_scale is None:
        softmax_scale = d ** -0.5
    comp, _ = indexer_topk_slice(q_idx, k_idx_compressed, indexer_weights, top_k, m, s_offset)
    dv = d if d_v is None else int(d_v)
    o, _ = _csa_attn_call(q, kv, kv_compressed, attn_sink, comp, n_win, s_offset, softmax_scale, dv)
    if return_indices:
        return o, comp
    return o
