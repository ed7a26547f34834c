"""Lightning indexer + top-k on B200: the reference's Python API over the C ABI.

* :func:`chunked_indexer_topk` — ``flash_sparse/triton/chunked_indexer.py:47-160``
* :func:`indexer_score`        — ``flash_sparse/triton/indexer_score.py:123-179``
* :func:`indexer_score_topk`   — ``flash_sparse/triton/indexer_score.py:182-205``

Same argument names, meanings and error types as the reference: shape and
device problems raise ``AssertionError`` (checked here, before the C call),
unsupported head counts raise ``ValueError``, and a non-zero status from the
library raises :class:`streamindex_b200._lib.SIError` (a ``RuntimeError``).
There is no CPU fallback: inputs must be CUDA tensors.

All three run one fused kernel (tcgen05 GEMM with the ReLU / head-weight /
mask epilogue and an exact streaming top-k) plus a row sort; the
``chunk_s`` / ``chunk_t`` hints of the reference are accepted and ignored,
because the selection here is exact and keeps memory at O(S·k) regardless of
chunking (the partition theorem of ``docs/streaming_topk.md:81-143`` is what
made the reference's results chunk-independent too).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib

_HEADS = (16, 32, 64, 128)


def _check(q: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor):
    """Shape / dtype / device checks shared by the wrappers (AssertionError / ValueError as the reference)."""
    assert q.is_cuda and k_idx.is_cuda and weights.is_cuda, "inputs must be CUDA tensors (no CPU fallback)"
    assert q.dim() == 4 and k_idx.dim() == 3 and weights.dim() == 3
    B, S, H, D = q.shape
    B2, T, D2 = k_idx.shape
    assert B2 == B and D2 == D, f"q/k shape mismatch: q={tuple(q.shape)}, k={tuple(k_idx.shape)}"
    assert weights.shape == (B, S, H)
    assert q.dtype in (torch.bfloat16, torch.float16), f"q must be bf16 or fp16, got {q.dtype}"
    assert k_idx.dtype == q.dtype, "k_idx must have q's dtype"
    if H not in _HEADS:
        raise ValueError(f"H_I ({H}) must be one of {_HEADS}")
    if D % 8 != 0 or D > 128:
        raise ValueError(f"D_I ({D}) must be a multiple of 8 and at most 128")
    return B, S, H, D, T


def _prep(q: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor):
    B, S, H, D, T = _check(q, k_idx, weights)
    q = q.contiguous()
    k_idx = k_idx.contiguous()
    if weights.dtype not in (torch.float32, torch.bfloat16):
        weights = weights.float()
    weights = weights.contiguous()
    return q, k_idx, weights, (B, S, H, D, T)


def _prep_strided(q: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor):
    """Like :func:`_prep`, but q / k_idx / weights whose last dim is contiguous
    are passed in place with their strides (the reference hands its kernels
    arbitrary strides); only other layouts are copied."""
    B, S, H, D, T = _check(q, k_idx, weights)
    qs = _lib.strides_arg(q, (0, 1, 2))
    ks = _lib.strides_arg(k_idx, (0, 1))
    if weights.dtype not in (torch.float32, torch.bfloat16):
        weights = weights.float()
    ws_ = _lib.strides_arg(weights, (0, 1, 2), align_elems=1) if weights.stride(-1) >= 0 else None
    if ws_ is None or weights.data_ptr() % weights.element_size():
        weights, ws_ = weights.contiguous(), None
    q2 = q if qs is not None else q.contiguous()
    k2 = k_idx if ks is not None else k_idx.contiguous()
    return q2, qs, k2, ks, weights, ws_, (B, S, H, D, T)


def _topk(q, k_idx, weights, top_k: int, width: int, ratio: Optional[int], mask: Optional[torch.Tensor]):
    q, qs, k_idx, ks, weights, ws_, (B, S, H, D, T) = _prep_strided(q, k_idx, weights)
    dev = q.device
    out_idx = torch.empty((B, S, width), dtype=torch.int64, device=dev)
    out_scores = torch.empty((B, S, width), dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws_bytes = lib.si_indexer_topk_ws_bytes(B, S, T, H, D, width)
    with torch.cuda.device(dev):
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        m = None
        if mask is not None:
            m = mask.to(device=dev, dtype=torch.bool).expand(B, S, T).contiguous().view(torch.uint8)
        _lib.check(lib.si_indexer_topk_strided(
            q.data_ptr(), qs, k_idx.data_ptr(), ks, weights.data_ptr(), ws_, int(weights.dtype == torch.bfloat16),
            int(q.dtype == torch.float16), B, S, T, H, D, width, int(ratio or 0), _lib.ptr(m), 0, 0,
            out_idx.data_ptr(), out_scores.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "indexer_topk")
    return out_idx, out_scores


def indexer_topk_slice(q, k_idx, weights, top_k: int, causal_ratio: int, s_offset: int):
    """Indexer + top-k for the query slice starting at global position ``s_offset``
    (causal limit ``t < (s_offset + s + 1)//causal_ratio``).  Returns ``(idx, scores)``."""
    q, k_idx, weights, (B, S, H, D, T) = _prep(q, k_idx, weights)
    dev = q.device
    out_idx = torch.empty((B, S, top_k), dtype=torch.int64, device=dev)
    out_scores = torch.empty((B, S, top_k), dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws_bytes = lib.si_indexer_topk_ws_bytes(B, S, T, H, D, top_k)
    with torch.cuda.device(dev):
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        _lib.check(lib.si_indexer_topk_ex(
            q.data_ptr(), k_idx.data_ptr(), weights.data_ptr(), int(weights.dtype == torch.bfloat16),
            int(q.dtype == torch.float16), B, S, T, H, D, int(top_k), int(causal_ratio), None, int(s_offset), 0,
            out_idx.data_ptr(), out_scores.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "indexer_topk")
    return out_idx, out_scores


def chunked_indexer_topk(
    q: torch.Tensor,
    k_idx: torch.Tensor,
    weights: torch.Tensor,
    top_k: int,
    *,
    causal_mask: Optional[torch.Tensor] = None,
    causal_ratio: Optional[int] = None,
    chunk_s: int = 4096,
    chunk_t: int = 4096,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Indexer + top-k.  Returns ``(idx int64 [B,S,top_k], scores fp32 [B,S,top_k])``.

    Sorted by score descending, ties toward the smaller key index; slots with
    no legal key are ``-1`` / ``-inf``.  ``causal_ratio=m`` applies
    ``t < (s+1)//m`` on the fly; ``causal_mask`` ([B,S,T] bool, True = legal)
    is the materialised alternative; they are mutually exclusive.
    """
    B, S = q.shape[0], q.shape[1]
    T = k_idx.shape[1]
    if causal_mask is not None:
        assert causal_mask.shape == (B, S, T)
        assert causal_ratio is None, "specify either causal_mask or causal_ratio, not both"
    if causal_ratio is not None:
        assert int(causal_ratio) >= 1, "causal_ratio must be a positive integer"
    assert int(top_k) >= 1
    del chunk_s, chunk_t  # tiling hints only; the result is chunk-independent
    return _topk(q, k_idx, weights, int(top_k), int(top_k), causal_ratio, causal_mask)


def indexer_score_topk(
    q: torch.Tensor,
    k_idx: torch.Tensor,
    weights: torch.Tensor,
    top_k: int,
    *,
    causal_mask: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Indexer + top-k of width ``min(top_k, T)``; ``-1`` / ``-inf`` where no legal key remains."""
    B, S = q.shape[0], q.shape[1]
    T = k_idx.shape[1]
    if causal_mask is not None:
        assert causal_mask.shape == (B, S, T)
    width = min(int(top_k), T)
    if width == 0:
        dev = q.device
        return (torch.empty((B, S, 0), dtype=torch.int64, device=dev),
                torch.empty((B, S, 0), dtype=torch.float32, device=dev))
    return _topk(q, k_idx, weights, width, width, None, causal_mask)


def indexer_score(q: torch.Tensor, k_idx: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """Materialised lightning-indexer scores ``[B,S,T]`` fp32 (eq. 16), no mask."""
    q, k_idx, weights, (B, S, H, D, T) = _prep(q, k_idx, weights)
    dev = q.device
    out = torch.empty((B, S, T), dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(256, dtype=torch.uint8, device=dev)
        _lib.check(lib.si_indexer_score(
            q.data_ptr(), k_idx.data_ptr(), weights.data_ptr(), int(weights.dtype == torch.bfloat16),
            int(q.dtype == torch.float16), B, S, T, H, D, out.data_ptr(), ws.data_ptr(), 256,
            _lib.stream_handle(dev)))
        _lib.maybe_check_status(ws, dev, "indexer_score")
    return out


class IndexerTopk:
    """Pre-planned indexer + top-k for repeated calls on fixed shapes.

    Holds the workspace and output buffers so a step enqueues exactly the
    fused kernel and the row sort (plus a 4-byte status reset).  ``s_offset``
    is the global position of local query 0, used when the query dimension is
    sharded across ranks.  ``run(..., sort=False)`` leaves the selection keys
    unsorted in ``out_idx`` so the two kernels can be timed separately;
    ``sort()`` then finishes the step.
    """

    def __init__(self, B, S, T, H, D, top_k, causal_ratio=None, s_offset=0, device="cuda",
                 q_dtype=torch.bfloat16, w_dtype=torch.float32):
        if H not in _HEADS:
            raise ValueError(f"H_I ({H}) must be one of {_HEADS}")
        self.B, self.S, self.T, self.H, self.D, self.k = B, S, T, H, D, int(top_k)
        self.ratio = int(causal_ratio or 0)
        self.s_offset = int(s_offset)
        self.device = torch.device(device)
        self.fp16 = int(q_dtype == torch.float16)
        self.w_bf16 = int(w_dtype == torch.bfloat16)
        self.lib = _lib.load()
        self.ws_bytes = self.lib.si_indexer_topk_ws_bytes(B, max(S, 1), T, H, D, self.k)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=self.device)
        self.out_idx = torch.empty((B, S, self.k), dtype=torch.int64, device=self.device)
        self.out_scores = torch.empty((B, S, self.k), dtype=torch.float32, device=self.device)

    def run(self, q, k_idx, weights, sort: bool = True):
        assert q.is_cuda and q.is_contiguous() and k_idx.is_contiguous() and weights.is_contiguous()
        assert q.shape == (self.B, self.S, self.H, self.D) and k_idx.shape == (self.B, self.T, self.D)
        _lib.check(self.lib.si_indexer_topk_ex(
            q.data_ptr(), k_idx.data_ptr(), weights.data_ptr(), self.w_bf16, self.fp16, self.B, self.S, self.T,
            self.H, self.D, self.k, self.ratio, None, self.s_offset, 0 if sort else 1, self.out_idx.data_ptr(),
            self.out_scores.data_ptr(), self.ws.data_ptr(), self.ws_bytes, _lib.stream_handle(self.device)))
        return self.out_idx, self.out_scores

    def sort(self):
        _lib.check(self.lib.si_topk_row_sort(self.out_idx.data_ptr(), self.out_scores.data_ptr(),
                                             self.B * self.S, self.k, _lib.stream_handle(self.device)))
        return self.out_idx, self.out_scores

    def status(self) -> int:
        return _lib.read_status(self.ws, self.device)

    def run_host(self, q_host, k_host, w_host, idx_host, scores_host, chunks: int = 8):
        """Indexer + top-k from pinned HOST buffers into pinned HOST outputs.

        The query range is cut into ``chunks`` slices.  Keys are copied once;
        then slice c+1's q / w host-to-device copies and slice c-1's results
        device-to-host copies run on two copy streams while slice c computes
        (each slice is one C-ABI call with its ``s_offset``), so the PCIe
        transfers hide behind the kernel.  Requires B == 1.  Returns once the
        outputs are in host memory.
        """
        assert self.B == 1
        for t in (q_host, k_host, w_host, idx_host, scores_host):
            assert not t.is_cuda and t.is_pinned() and t.is_contiguous(), "host buffers must be pinned and contiguous"
        dev = self.device
        S, H, D, T, k = self.S, self.H, self.D, self.T, self.k
        bounds = [S * c // chunks for c in range(chunks + 1)]
        bounds = [min(S, ((b + 127) // 128) * 128) for b in bounds[:-1]] + [S]
        nmax = max(b1 - b0 for b0, b1 in zip(bounds, bounds[1:]))
        if not hasattr(self, "_hbufs") or self._hbufs[0][0].shape[1] < nmax:
            self._hbufs = (
                [torch.empty((1, nmax, H, D), dtype=q_host.dtype, device=dev) for _ in range(2)],
                [torch.empty((1, nmax, H), dtype=w_host.dtype, device=dev) for _ in range(2)],
                [torch.empty((1, nmax, k), dtype=torch.int64, device=dev) for _ in range(2)],
                [torch.empty((1, nmax, k), dtype=torch.float32, device=dev) for _ in range(2)],
                torch.empty((1, T, D), dtype=k_host.dtype, device=dev),
                torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        qb, wb, ib, sb, kd, s_in, s_out = self._hbufs
        comp = torch.cuda.current_stream(dev)
        with torch.cuda.stream(s_in):
            kd.copy_(k_host, non_blocking=True)
        ev_in = [torch.cuda.Event() for _ in range(chunks)]
        ev_done = [torch.cuda.Event() for _ in range(chunks)]
        ev_out = [torch.cuda.Event() for _ in range(chunks)]

        def load(c):
            b0, b1 = bounds[c], bounds[c + 1]
            slot = c & 1
            with torch.cuda.stream(s_in):
                if c >= 2:
                    s_in.wait_event(ev_done[c - 2])  # slot's previous slice is no longer read
                qb[slot][:, : b1 - b0].copy_(q_host[:, b0:b1], non_blocking=True)
                wb[slot][:, : b1 - b0].copy_(w_host[:, b0:b1], non_blocking=True)
                ev_in[c].record(s_in)

        load(0)
        for c in range(chunks):
            if c + 1 < chunks:
                load(c + 1)
            b0, b1 = bounds[c], bounds[c + 1]
            n = b1 - b0
            slot = c & 1
            comp.wait_event(ev_in[c])
            if c >= 2:
                comp.wait_event(ev_out[c - 2])  # the output slot has been copied out
            if n > 0:
                _lib.check(self.lib.si_indexer_topk_ex(
                    qb[slot].data_ptr(), kd.data_ptr(), wb[slot].data_ptr(), self.w_bf16, self.fp16, 1, n, T, H, D,
                    k, self.ratio, None, self.s_offset + b0, 0, ib[slot].data_ptr(), sb[slot].data_ptr(), self.ws.data_ptr(),
                    self.ws_bytes, _lib.stream_handle(dev)))
            ev_done[c].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[c])
                idx_host[:, b0:b1].copy_(ib[slot][:, :n], non_blocking=True)
                scores_host[:, b0:b1].copy_(sb[slot][:, :n], non_blocking=True)
                ev_out[c].record(s_out)
        comp.wait_event(ev_out[chunks - 1])
        comp.synchronize()
        return idx_host, scores_host
