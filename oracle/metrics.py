"""Parity metrics used by the tests.  Test infrastructure.

* ``set_recall`` — valid-only set recall, ``eval/test_v4_indexer_parity.py:164-199``
  (per query ``|A ∩ B| / |A|`` over non-negative entries; both empty -> 1,
  A empty and B not -> 0).
* ``norm_corr`` — ``1 - 2<a,b>/(<a,a>+<b,b>)``,
  ``tests/test_triton_indexer_score.py:16-23``.
* ``score_close`` — north-star score tolerance
  ``|a-b| <= rtol * max(|b|, 1e-2 * rms(b))``.
"""

from __future__ import annotations

import torch


def set_recall(idx_a: torch.Tensor, idx_b: torch.Tensor) -> torch.Tensor:
    a = idx_a.long().cpu()
    b = idx_b.long().cpu()
    va, vb = a >= 0, b >= 0
    na, nb = va.sum(-1), vb.sum(-1)
    a = torch.where(va, a, torch.full_like(a, -2))
    b = torch.where(vb, b, torch.full_like(b, -3))
    sa, _ = a.sort(dim=-1)
    sb, _ = b.sort(dim=-1)
    # membership of each a in b via searchsorted on the sorted rows
    flat_a = sa.reshape(-1, sa.shape[-1])
    flat_b = sb.reshape(-1, sb.shape[-1]).contiguous()
    pos = torch.searchsorted(flat_b, flat_a.contiguous()).clamp(max=flat_b.shape[-1] - 1)
    hit = (flat_b.gather(-1, pos) == flat_a) & (flat_a >= 0)
    overlap = hit.sum(-1).reshape(na.shape).float()
    rec = overlap / na.clamp(min=1).float()
    rec = torch.where((na == 0) & (nb == 0), torch.ones_like(rec), rec)
    rec = torch.where((na == 0) & (nb > 0), torch.zeros_like(rec), rec)
    return rec


def norm_corr(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().flatten()
    b = b.double().flatten()
    fin = torch.isfinite(a) & torch.isfinite(b)
    a, b = a[fin], b[fin]
    return float(1 - 2 * (a * b).sum() / ((a * a).sum() + (b * b).sum()).clamp_min(1e-30))


def score_close(a: torch.Tensor, b: torch.Tensor, rtol: float = 1e-2) -> bool:
    a = a.double().cpu()
    b = b.double().cpu()
    fa, fb = torch.isfinite(a), torch.isfinite(b)
    if not torch.equal(fa, fb):
        return False
    if not torch.equal(a[~fa], b[~fb]):
        return False
    a, b = a[fa], b[fb]
    if b.numel() == 0:
        return True
    rms = b.pow(2).mean().sqrt()
    tol = rtol * torch.maximum(b.abs(), 1e-2 * rms)
    return bool(((a - b).abs() <= tol).all())
