"""Query-dimension (S) sharding of the indexer + top-k across GPUs.

Each rank owns a contiguous query slice ``[s_lo, s_hi)`` of q / weights and a
full replica of the compressed keys; queries are independent
(``docs/streaming_topk.md:37-44`` of the reference), so the only exchanges
are a broadcast of the keys from rank 0 and a gather of the per-slice
results to rank 0 (NCCL over NVLink, via ``torch.distributed``).

Causal work grows linearly with s (query s has ``min(T, (s+1)//ratio)``
legal keys), so equal-length slices are unbalanced; ``balanced_bounds``
places the boundaries at equal shares of the cumulative legal-pair count.
"""

from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch
import torch.distributed as dist


# Fixed per-query cost of the fused indexer (selection, flushes, output write),
# in units of causally legal (s, t) pairs at the large-S pair rate.  Fitted on
# the single-GPU S sweep (H_I=64, D_I=128, k=512, T=S/4, S = 32K..1M): with
# pairs = S^2/8, 1/frac = a + b/S gives b ~ 1.9e4, i.e. ~2.4k pairs per query
# at the peak rate, ~1.8k at the large-S rate.  Balancing on pairs alone gives
# rank 0 (the most, and shortest, queries) ~5% more time at 8 GPUs.
INDEXER_QUERY_COST_PAIRS = 1800.0

# Sparse attention runs at a lower rate than the indexer's dense contraction
# (config 5 on one B200: indexer 852 TFLOP/s, attention 517 TFLOP/s), so one
# attention flop costs ~1.65 indexer flops of time.
ATTN_VS_INDEXER_FLOP_TIME = 1.65


def csa_query_cost_pairs(H: int, D: int, Dv: int, HI: int, DI: int, n_win: int, top_k: int) -> float:
    """Per-query work of a CSA layer that does not grow with s, in indexer
    key-pair units: the indexer's own per-query cost plus the query's sparse
    attention over n_win + top_k rows, weighted by the two kernels' measured
    relative speed."""
    attn = (n_win + top_k) * H * (D + Dv) / (HI * DI)
    return INDEXER_QUERY_COST_PAIRS * HI / 64 + ATTN_VS_INDEXER_FLOP_TIME * attn


def legal_pairs(S: int, T: int, ratio: Optional[int], lo: int = 0, hi: Optional[int] = None) -> int:
    """Sum over s in [lo, hi) of min(T, (s+1)//ratio) (T per query without a ratio)."""
    hi = S if hi is None else hi
    if hi <= lo:
        return 0
    if not ratio:
        return (hi - lo) * T
    s = np.arange(lo, hi, dtype=np.int64)
    return int(np.minimum(T, (s + 1) // int(ratio)).sum())


def balanced_bounds(S: int, N: int, T: int, ratio: Optional[int], align: int = 128,
                    extra_per_query: float = 0.0) -> List[int]:
    """N+1 boundaries, multiples of ``align`` (except S), splitting the work evenly.

    Work of query s = its legal key count ``min(T, (s+1)//ratio)`` plus
    ``extra_per_query`` (work that does not grow with s, e.g. the attention of a
    CSA layer, in the same units)."""
    if N <= 1:
        return [0, S]
    s = np.arange(S, dtype=np.int64)
    w = np.minimum(T, (s + 1) // int(ratio)) if ratio else np.full(S, T, dtype=np.int64)
    w = np.maximum(w.astype(np.float64) + float(extra_per_query), 1.0)  # every query costs at least its output
    cum = np.cumsum(w)
    total = int(cum[-1])
    bounds = [0]
    for r in range(1, N):
        b = int(np.searchsorted(cum, total * r / N))
        b = min(S, max(bounds[-1], (b // align) * align))
        bounds.append(b)
    bounds.append(S)
    return bounds


def broadcast_keys(k_idx: torch.Tensor, src: int = 0) -> torch.Tensor:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.broadcast(k_idx, src=src)
    return k_idx


def gather_to_rank0(local: torch.Tensor, bounds: List[int], full: Optional[torch.Tensor], dim: int = 1):
    """Point-to-point gather of each rank's S-slice into ``full`` on rank 0."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        if full is not None and full.data_ptr() != local.data_ptr():
            full.copy_(local)
        return full
    rank, world = dist.get_rank(), dist.get_world_size()
    ops = []
    if rank == 0:
        assert full is not None
        full.narrow(dim, bounds[0], bounds[1] - bounds[0]).copy_(local)
        staged = []
        for r in range(1, world):
            n = bounds[r + 1] - bounds[r]
            if n > 0:
                view = full.narrow(dim, bounds[r], n)
                buf = view if view.is_contiguous() else torch.empty(view.shape, dtype=view.dtype, device=view.device)
                if buf is not view:
                    staged.append((view, buf))
                ops.append(dist.P2POp(dist.irecv, buf, r))
    else:
        if local.numel() > 0:
            ops.append(dist.P2POp(dist.isend, local.contiguous(), 0))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if rank == 0:
        for view, buf in staged:
            view.copy_(buf)
    return full
