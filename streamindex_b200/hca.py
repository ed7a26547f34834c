"""HCA layer forward on B200: ``flash_hca_forward`` and ``build_hca_topk_idxs``.

Mirrors ``flash_sparse/hca.py:24-95`` of the reference: no indexer; every
causally legal compressed block (``(i+1)*m' - 1 <= s``) plus the sliding window
goes through the sparse-attention kernel.  As in the CSA layer, the
concatenated kv is never built (split-kv attention).  Forward only.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .attention import _attn_call


def build_hca_topk_idxs(*, B: int, seq_len: int, n_win: int, n_compressed: int, m_prime: int,
                        device) -> torch.Tensor:
    """``[B, S, n_win + n_compressed]`` int32 on ``device`` (a CUDA device)."""
    dev = torch.device(device)
    assert dev.type == "cuda", "no CPU fallback"
    out = torch.empty((B, seq_len, n_win + n_compressed), dtype=torch.int32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        _lib.check(lib.si_hca_build_idx(B, seq_len, int(n_win), int(n_compressed), int(m_prime), out.data_ptr(),
                                        _lib.stream_handle(dev)))
    return out


def flash_hca_forward(
    q: torch.Tensor,
    kv: torch.Tensor,
    kv_compressed: torch.Tensor,
    attn_sink: torch.Tensor,
    *,
    n_win: int,
    m_prime: int = 128,
    softmax_scale: Optional[float] = None,
    use_triton: bool = True,
    d_v: Optional[int] = None,
) -> torch.Tensor:
    """End-to-end HCA forward (prefill, one layer).  Returns ``o [B,S,n_h,d_v or d]`` bf16."""
    del use_triton
    B, S, n_h, d = q.shape
    n_compressed = kv_compressed.shape[1]
    if softmax_scale is None:
        softmax_scale = d ** -0.5
    idx = build_hca_topk_idxs(B=B, seq_len=S, n_win=n_win, n_compressed=n_compressed, m_prime=m_prime,
                              device=q.device)
    dv = d if d_v is None else int(d_v)
    o, _ = _attn_call(q, kv, kv_compressed, attn_sink, idx, softmax_scale, dv)
    return o
