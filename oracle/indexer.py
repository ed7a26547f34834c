"""Oracle: lightning-indexer score and top-k (CPU, fp32).  Test infrastructure.

Restates, without the shipped defects (dropped call parentheses, shifted
block indentation):

* ``reference_lightning_indexer`` — ``flash_sparse/reference.py:138-168``
  (eq. 16: fp32 einsum ``bshd,btd->bsht``, ReLU, ``* w[..., None]``, sum
  over heads);
* the materialise-then-topk path with its post-mask —
  ``eval/test_v4_indexer_parity.py:111-137``;
* the chunked partition-merge top-k — ``flash_sparse/triton/chunked_indexer.py:47-160``
  (mask ``t < (s+1)//ratio`` at ``:123-141``, per-chunk top-k ``:144-146``,
  merge ``:149-153``, ``-1`` where the score is infinite ``:155``).

Tie order: the reference documents the total order
``(a, i) > (b, j)  <=>  a > b  or  (a == b and i < j)``
(``docs/streaming_topk.md:48-66,301-305``); ``torch.topk`` leaves ties
undefined, so this oracle realises the documented order with a stable
descending sort.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch


def causal_limit(S: int, T: int, ratio: Optional[int], device="cpu") -> torch.Tensor:
    """Number of legal keys per query: ``min(T, (s+1)//ratio)`` (``T`` if no ratio).

    Legal iff ``t < (s+1)//ratio`` (``chunked_indexer.py:137``), which equals
    the ``(i+1)*m - 1 <= s`` form of ``csa.py:61-63``.
    """
    s = torch.arange(S, device=device, dtype=torch.int64)
    if ratio is None:
        return torch.full((S,), T, dtype=torch.int64, device=device)
    return torch.clamp((s + 1) // int(ratio), max=T)


def lightning_indexer(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, s_chunk: int = 512) -> torch.Tensor:
    """``I[b,s,t] = sum_h w[b,s,h] * relu(q[b,s,h,:] . k[b,t,:])`` in fp32.

    ``flash_sparse/reference.py:163-168``.  Chunked over S only to bound host
    memory; each chunk evaluates the same fp32 einsum.
    """
    assert q.dim() == 4 and k.dim() == 3 and w.dim() == 3
    B, S, H, D = q.shape
    T = k.shape[1]
    out = torch.empty((B, S, T), dtype=torch.float32)
    kf = k.float()
    for s0 in range(0, S, s_chunk):
        s1 = min(S, s0 + s_chunk)
        qk = torch.einsum("bshd,btd->bsht", q[:, s0:s1].float(), kf)
        qk = qk.relu_()
        out[:, s0:s1] = (qk * w[:, s0:s1].float().unsqueeze(-1)).sum(dim=2)
    return out


def topk_desc_stable(scores: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k along the last dim in the order score desc, index asc (stable sort)."""
    vals, idx = torch.sort(scores, dim=-1, descending=True, stable=True)
    return idx[..., :k].to(torch.int64), vals[..., :k].contiguous()


def _post_mask(idx: torch.Tensor, vals: torch.Tensor, top_k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """-inf slots become idx -1 (``chunked_indexer.py:155``); pad the width to top_k."""
    idx = torch.where(torch.isinf(vals) & (vals < 0), torch.full_like(idx, -1), idx)
    k_eff = idx.shape[-1]
    if k_eff < top_k:
        pad_shape = idx.shape[:-1] + (top_k - k_eff,)
        idx = torch.cat([idx, torch.full(pad_shape, -1, dtype=idx.dtype)], dim=-1)
        vals = torch.cat([vals, torch.full(pad_shape, float("-inf"), dtype=vals.dtype)], dim=-1)
    return idx, vals


def materialize_topk(
    q: torch.Tensor,
    k: torch.Tensor,
    w: torch.Tensor,
    top_k: int,
    ratio: Optional[int] = None,
    causal_mask: Optional[torch.Tensor] = None,
    pad: bool = True,
    s_chunk: int = 512,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Materialise ``[B,S,T]`` scores, mask, top-k(min(k,T)), post-mask to -1/-inf.

    ``eval/test_v4_indexer_parity.py:121-137`` (mask ``t >= (s+1)//ratio`` is
    illegal; picks at illegal positions become -1).  Returns
    ``(idx int64 [B,S,top_k], scores fp32 [B,S,top_k])`` when ``pad`` (the
    ``chunked_indexer_topk`` width), else width ``min(top_k, T)``.
    """
    B, S, H, D = q.shape
    T = k.shape[1]
    k_eff = min(top_k, T)
    out_i, out_v = [], []
    for s0 in range(0, S, s_chunk):
        s1 = min(S, s0 + s_chunk)
        sc = lightning_indexer(q[:, s0:s1], k, w[:, s0:s1])
        if ratio is not None:
            lim = causal_limit(S, T, ratio)[s0:s1]
            illegal = torch.arange(T).unsqueeze(0) >= lim.unsqueeze(1)
            sc = sc.masked_fill(illegal.unsqueeze(0), float("-inf"))
        elif causal_mask is not None:
            sc = sc.masked_fill(~causal_mask[:, s0:s1].cpu(), float("-inf"))
        i, v = topk_desc_stable(sc, k_eff)
        i, v = _post_mask(i, v, top_k if pad else k_eff)
        out_i.append(i)
        out_v.append(v)
    return torch.cat(out_i, dim=1), torch.cat(out_v, dim=1)


def chunked_indexer_topk(
    q: torch.Tensor,
    k: torch.Tensor,
    w: torch.Tensor,
    top_k: int,
    ratio: Optional[int] = None,
    causal_mask: Optional[torch.Tensor] = None,
    chunk_s: int = 4096,
    chunk_t: int = 4096,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Partition-merge top-k (``flash_sparse/triton/chunked_indexer.py:88-160``).

    Per (chunk_s x chunk_t) tile: score, mask, tile top-k(min(k, chunk_T)),
    offset by ``t_start``, merge with the running ``[B, chunk_S, top_k]``
    state (seeded with -inf / -1), mark -inf slots -1.  Merges use the stable
    order so the result equals :func:`materialize_topk` exactly (the
    partition theorem, ``docs/streaming_topk.md:81-143``).
    """
    assert not (causal_mask is not None and ratio is not None)
    B, S, H, D = q.shape
    T = k.shape[1]
    out_idx = torch.empty((B, S, top_k), dtype=torch.int64)
    out_val = torch.empty((B, S, top_k), dtype=torch.float32)
    for s0 in range(0, S, chunk_s):
        s1 = min(S, s0 + chunk_s)
        run_v = torch.full((B, s1 - s0, top_k), float("-inf"))
        run_i = torch.full((B, s1 - s0, top_k), -1, dtype=torch.int64)
        for t0 in range(0, T, chunk_t):
            t1 = min(T, t0 + chunk_t)
            sc = lightning_indexer(q[:, s0:s1], k[:, t0:t1], w[:, s0:s1])
            if causal_mask is not None:
                sc = sc.masked_fill(~causal_mask[:, s0:s1, t0:t1].cpu(), float("-inf"))
            elif ratio is not None:
                s_idx = torch.arange(s0, s1).unsqueeze(1)
                t_idx = torch.arange(t0, t1).unsqueeze(0)
                legal = t_idx < (s_idx + 1) // ratio
                sc = sc.masked_fill(~legal.unsqueeze(0), float("-inf"))
            ci, cv = topk_desc_stable(sc, min(top_k, t1 - t0))
            ci = ci + t0
            # Running entries come from earlier chunks (smaller indices), so a
            # stable sort over [run, chunk] keeps the index-ascending tie order.
            comb_v = torch.cat([run_v, cv], dim=-1)
            comb_i = torch.cat([run_i, ci], dim=-1)
            pi, run_v = topk_desc_stable(comb_v, top_k)
            run_i = comb_i.gather(-1, pi)
            run_i = torch.where(torch.isinf(run_v), torch.full_like(run_i, -1), run_i)
        out_idx[:, s0:s1] = run_i
        out_val[:, s0:s1] = run_v
    return out_idx, out_val
