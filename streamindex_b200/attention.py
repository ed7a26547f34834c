"""Sparse MQA attention forward with attention sink, over the C ABI.

* :func:`sparse_attn_fwd` — ``flash_sparse/triton/sparse_attn_fwd.py:180-292``
* :func:`sparse_attn_bwd` — ``flash_sparse/triton/sparse_attn_bwd.py:286-416``
* :func:`sparse_attn`     — ``flash_sparse/triton/__init__.py:50-61`` (autograd
  wrapper over the two)

q / kv / o are bf16 or fp16 (one type for all three, as the reference's
Triton kernel accepts, ``sparse_attn_fwd.py:207``).

Semantics follow ``reference_sparse_attn`` (``flash_sparse/reference.py:44-130``):
``-1`` indices are masked, the sink enters the denominator only, the default
scale is ``D**-0.5``, an all-masked query returns 0.  ``d_v`` (new keyword)
selects the value width: ``None`` returns the reference's full-``D`` output;
``d_v=512`` on the 576-wide MLA layout equals ``reference_sparse_attn(...)[..., :512]``.
``block_h`` / ``block_n`` are the reference's Triton tiling knobs, accepted and
ignored.  Returns ``(o bf16 [B,S,H,d_v], lse fp32 [B,S,H])``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from . import _lib


def _attn_call(q, kv, kv2, attn_sink, idx, softmax_scale, dv):
    """One C-ABI call; kv2 (optional) holds rows Nkv.. of the logical kv."""
    B, S, H, D = q.shape
    dev = q.device
    K = idx.shape[-1]
    dv_k = ((dv + 63) // 64) * 64
    Dp = ((max(D, dv_k) + 7) // 8) * 8
    qs = _lib.strides_arg(q, (0, 1, 2)) if Dp == D else None
    qk = q if qs is not None else q.contiguous()  # q is read in place when its last dim is contiguous
    kvk = kv.contiguous()
    kv2k = None if kv2 is None else kv2.contiguous()
    if Dp != D:
        qk = F.pad(qk, (0, Dp - D))
        kvk = F.pad(kvk, (0, Dp - D))
        if kv2k is not None:
            kv2k = F.pad(kv2k, (0, Dp - D))
    idx = idx.to(device=dev, dtype=torch.int32).contiguous()
    sink = attn_sink.to(device=dev, dtype=torch.float32).contiguous()
    o = torch.empty((B, S, H, dv_k), dtype=q.dtype, device=dev)
    lse = torch.empty((B, S, H), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(256, dtype=torch.uint8, device=dev)
        _lib.check(lib.si_sparse_attn_fwd_strided(
            qk.data_ptr(), qs, kvk.data_ptr(), kvk.shape[1], _lib.ptr(kv2k), 0 if kv2k is None else kv2k.shape[1],
            sink.data_ptr(), idx.data_ptr() if K > 0 else None, B, S, H, Dp, K, dv_k, float(softmax_scale),
            int(q.dtype == torch.float16), o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256,
            _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "sparse_attn_fwd")
    if dv_k != dv:
        o = o[..., :dv].contiguous()
    return o, lse


def _csa_attn_call(q, kv, kv_comp, attn_sink, comp_idx, n_win, s_offset, softmax_scale, dv):
    """CSA attention with the window + compressed index list built in the kernel
    (``si_csa_sparse_attn_fwd``).  ``q`` is the query slice starting at global
    position ``s_offset`` of the ``kv.shape[1]``-token sequence; ``comp_idx``
    ``[B,S,top_k]`` int64 holds the compressed picks (-1 = empty)."""
    B, S, H, D = q.shape
    dev = q.device
    top_k = comp_idx.shape[-1]
    dv_k = ((dv + 63) // 64) * 64
    Dp = ((max(D, dv_k) + 7) // 8) * 8
    qk, kvk, kck = q.contiguous(), kv.contiguous(), kv_comp.contiguous()
    if Dp != D:
        qk, kvk, kck = F.pad(qk, (0, Dp - D)), F.pad(kvk, (0, Dp - D)), F.pad(kck, (0, Dp - D))
    comp = comp_idx.to(device=dev, dtype=torch.int64).contiguous()
    sink = attn_sink.to(device=dev, dtype=torch.float32).contiguous()
    o = torch.empty((B, S, H, dv_k), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, S, H), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(256, dtype=torch.uint8, device=dev)
        _lib.check(lib.si_csa_sparse_attn_fwd(
            qk.data_ptr(), kvk.data_ptr(), kvk.shape[1], kck.data_ptr(), kck.shape[1], sink.data_ptr(),
            comp.data_ptr() if top_k > 0 else None, top_k, int(n_win), int(s_offset), B, S, H, Dp, dv_k,
            float(softmax_scale), o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256, _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "csa_sparse_attn_fwd")
    if dv_k != dv:
        o = o[..., :dv].contiguous()
    return o, lse


def sparse_attn_fwd(
    q: torch.Tensor,
    kv: torch.Tensor,
    attn_sink: torch.Tensor,
    topk_idxs: torch.Tensor,
    softmax_scale: Optional[float] = None,
    *,
    block_h: Optional[int] = None,
    block_n: int = 64,
    d_v: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    del block_h, block_n  # Triton tiling knobs of the reference
    assert q.is_cuda and kv.is_cuda, "inputs must be CUDA tensors (no CPU fallback)"
    assert q.dim() == 4 and kv.dim() == 3
    assert q.dtype in (torch.bfloat16, torch.float16), f"q must be bf16 or fp16, got {q.dtype}"
    assert kv.dtype == q.dtype, "q and kv must share one dtype"
    assert attn_sink.dtype == torch.float32
    B, S, H, D = q.shape
    B2, N_kv, D2 = kv.shape
    assert B2 == B and D2 == D, "q and kv shape mismatch"
    assert attn_sink.shape == (H,)
    assert topk_idxs.shape[:2] == (B, S)
    K = topk_idxs.shape[-1]
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dv = D if d_v is None else int(d_v)
    if not (0 < dv <= D):
        raise ValueError(f"d_v ({dv}) must be in (0, D={D}]")
    return _attn_call(q, kv, None, attn_sink, topk_idxs, softmax_scale, dv)


def fp8_kv_row_bytes(D: int, n_nope: int) -> int:
    """Bytes per FP8 KV row (``[n_nope e4m3 | fp32 block scales | bf16 rope]``, 16-byte padded)."""
    n = _lib.load().si_fp8_kv_row_bytes(int(D), int(n_nope))
    if n < 0:
        raise ValueError(f"unsupported FP8 row split D={D}, n_nope={n_nope}")
    return n


def quantize_kv_fp8(kv: torch.Tensor, n_nope: int = 512) -> torch.Tensor:
    """bf16 kv ``[..., D]`` -> FP8 rows ``[..., row_bytes]`` uint8 (e4m3 NoPE dims with one
    fp32 scale per 64 dims, bf16 RoPE dims).  Dequantised values equal the
    reference's ``act_quant_simulate(kv[..., :n_nope], 64)`` (``flash_sparse/utils/quantization.py:19-36``)."""
    assert kv.is_cuda and kv.dtype == torch.bfloat16, "kv must be a bf16 CUDA tensor"
    D = kv.shape[-1]
    if not (n_nope % 64 == 0 and 64 <= n_nope <= 512 and 0 < D - n_nope <= 64 and D % 8 == 0):
        raise ValueError(f"unsupported FP8 row split D={D}, n_nope={n_nope}")
    rb = fp8_kv_row_bytes(D, n_nope)
    x = kv.contiguous()
    rows = x.numel() // D
    out = torch.empty((*kv.shape[:-1], rb), dtype=torch.uint8, device=kv.device)
    with torch.cuda.device(kv.device):
        _lib.check(_lib.load().si_kv_quant_fp8(x.data_ptr(), rows, D, int(n_nope), out.data_ptr(),
                                               _lib.stream_handle(kv.device)))
    return out


def sparse_attn_fwd_fp8kv(q: torch.Tensor, kv_rows: torch.Tensor, n_nope: int, attn_sink: torch.Tensor,
                          topk_idxs: torch.Tensor, softmax_scale: Optional[float] = None, *,
                          d_v: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sparse attention over FP8 KV rows (from :func:`quantize_kv_fp8`).

    Same contract as :func:`sparse_attn_fwd` with ``kv`` replaced by its FP8
    rows: the result equals ``sparse_attn_fwd`` over the dequantised kv."""
    assert q.is_cuda and kv_rows.is_cuda and q.dtype == torch.bfloat16 and kv_rows.dtype == torch.uint8
    B, S, H, D = q.shape
    rb = fp8_kv_row_bytes(D, n_nope)
    assert kv_rows.dim() == 3 and kv_rows.shape[0] == B and kv_rows.shape[2] == rb, "kv_rows must be [B, N_kv, row_bytes]"
    assert attn_sink.shape == (H,) and topk_idxs.shape[:2] == (B, S)
    K = topk_idxs.shape[-1]
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dv = D if d_v is None else int(d_v)
    if dv % 64:
        raise ValueError(f"d_v ({dv}) must be a multiple of 64 for FP8 rows")
    dev = q.device
    qk, kvk = q.contiguous(), kv_rows.contiguous()
    idx = topk_idxs.to(device=dev, dtype=torch.int32).contiguous()
    sink = attn_sink.to(device=dev, dtype=torch.float32).contiguous()
    o = torch.empty((B, S, H, dv), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, S, H), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        ws = torch.empty(256, dtype=torch.uint8, device=dev)
        _lib.check(_lib.load().si_sparse_attn_fwd_fp8kv(
            qk.data_ptr(), kvk.data_ptr(), kvk.shape[1], None, 0, int(n_nope), sink.data_ptr(),
            idx.data_ptr() if K > 0 else None, B, S, H, D, K, dv, float(softmax_scale), o.data_ptr(), lse.data_ptr(),
            ws.data_ptr(), 256, _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "sparse_attn_fwd_fp8kv")
    return o, lse


def sparse_attn_bwd(q, kv, attn_sink, topk_idxs, o, lse, do, softmax_scale: Optional[float] = None, *,
                    block_h: Optional[int] = None):
    """Backward of :func:`sparse_attn_fwd` (``flash_sparse/triton/sparse_attn_bwd.py:286-416``).

    ``o`` / ``lse`` are the forward's outputs and ``do`` the gradient of ``o``
    (width ``d_v = o.shape[-1]``; the value is the first ``d_v`` dims of kv).
    Returns ``(dq, dkv, dattn_sink)`` in the dtypes of ``q``, ``kv`` and
    ``attn_sink``.  ``block_h`` is the reference's Triton tiling knob, ignored.
    """
    del block_h
    assert q.is_cuda and kv.is_cuda and do.is_cuda
    assert q.dtype == kv.dtype == do.dtype == torch.bfloat16, "backward supports bf16 tensors"
    assert attn_sink.dtype == torch.float32 and lse.dtype == torch.float32
    B, S, H, D = q.shape
    N_kv = kv.shape[1]
    K = topk_idxs.shape[-1]
    Dv = o.shape[-1]
    assert do.shape == o.shape == (B, S, H, Dv), "do must match o"
    if D not in (64, 128, 256, 512, 576):
        raise ValueError(f"backward supports D in (64, 128, 256, 512, 576), got {D}")
    if Dv % 32 or Dv > D:
        raise ValueError(f"backward needs d_v a multiple of 32 and <= D, got {Dv}")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dev = q.device
    qk, kvk, ok, dok = q.contiguous(), kv.contiguous(), o.contiguous(), do.contiguous()
    idx = topk_idxs.to(device=dev, dtype=torch.int32).contiguous()
    sink = attn_sink.contiguous()
    dq = torch.zeros_like(qk)
    dkv = torch.zeros((B, N_kv, D), dtype=torch.float32, device=dev)
    dsink = torch.zeros_like(sink)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().si_sparse_attn_bwd(
            qk.data_ptr(), kvk.data_ptr(), sink.data_ptr(), idx.data_ptr() if K > 0 else None, ok.data_ptr(),
            lse.contiguous().data_ptr(), dok.data_ptr(), B, S, H, D, N_kv, K, Dv, float(softmax_scale),
            dq.data_ptr(), dkv.data_ptr(), dsink.data_ptr(), _lib.stream_handle(dev)))
    return dq, dkv.to(kv.dtype), dsink


class _SparseAttnFunc(torch.autograd.Function):
    """Saves q, kv, attn_sink, topk_idxs, o and lse for the backward pass
    (``flash_sparse/triton/__init__.py:19-47``)."""

    @staticmethod
    def forward(ctx, q, kv, attn_sink, topk_idxs, softmax_scale, d_v):
        o, lse = sparse_attn_fwd(q, kv, attn_sink, topk_idxs, softmax_scale, d_v=d_v)
        ctx.save_for_backward(q, kv, attn_sink, topk_idxs, o, lse)
        ctx.softmax_scale = softmax_scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, kv, attn_sink, topk_idxs, o, lse = ctx.saved_tensors
        dq, dkv, dsink = sparse_attn_bwd(q, kv, attn_sink, topk_idxs, o, lse, do.contiguous(), ctx.softmax_scale)
        return dq, dkv, dsink, None, None, None


def sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale: Optional[float] = None, *, d_v: Optional[int] = None):
    """Differentiable sparse attention (``flash_sparse/triton/__init__.py:50-61``): forward
    :func:`sparse_attn_fwd`, backward :func:`sparse_attn_bwd`.  Returns ``o`` only."""
    return _SparseAttnFunc.apply(q, kv, attn_sink, topk_idxs, softmax_scale, d_v)
