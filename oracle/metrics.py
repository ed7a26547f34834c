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


def exact_pair_scores(q: torch.Tensor, k: torch.Tensor, w: torch.Tensor, b: torch.Tensor, s: torch.Tensor,
                      t: torch.Tensor):
    """Float64 indexer scores of the (b, s, t) pairs and an fp32 rounding bound.

    ``score = sum_h w[b,s,h] * relu(q[b,s,h,:] . k[b,t,:])`` (``flash_sparse/reference.py:163-168``)
    evaluated in float64 from the bf16/fp16 operands, which is exact to well
    below fp32 resolution.  The bound is the standard worst-case error of a
    recursive fp32 sum: ``gamma_n * sum|terms|`` with ``n = D + H + 1``
    (D products per dot, H weighted head terms) and ``gamma_n = n*u/(1-n*u)``,
    ``u = 2^-24``, so ``|fl32(score) - score| <= bound`` for ANY fp32
    evaluation order (tensor-core accumulation included).
    """
    qf = q[b, s].double()                       # [P,H,D]
    kf = k[b, t].double()                       # [P,D]
    wf = w[b, s].double()                       # [P,H]
    prod = qf * kf.unsqueeze(1)                 # [P,H,D]
    dot = prod.sum(-1)                          # [P,H]
    exact = (wf * dot.clamp_min(0)).sum(-1)
    absdot = prod.abs().sum(-1)
    mag = (wf.abs() * absdot).sum(-1)
    n = q.shape[-1] + q.shape[-2] + 1
    u = 2.0 ** -24
    gamma = n * u / (1 - n * u)
    return exact, gamma * mag


def measured_score_error(q, k, w, idx: torch.Tensor, scores: torch.Tensor, s_rows=None, chunk: int = 4096) -> float:
    """Largest ``|scores - exact|`` over the valid entries of ``idx``/``scores`` ``[B,S',k]``.

    ``exact`` is the float64 score of :func:`exact_pair_scores`.  This is the
    observed fp32 error of the scores under test, the scale that separates an
    fp32 tie from a real ranking difference.
    """
    gi = idx.long().cpu()
    gv = scores.double().cpu()
    B, S_, K = gi.shape
    if s_rows is None:
        s_rows = torch.arange(S_)
    s_rows = torch.as_tensor(s_rows).long().cpu()
    valid = gi >= 0
    bb = torch.arange(B).view(B, 1, 1).expand(B, S_, K)[valid]
    ss = s_rows.view(1, S_, 1).expand(B, S_, K)[valid]
    tt = gi[valid]
    vv = gv[valid]
    worst = 0.0
    for c in range(0, tt.numel(), chunk):
        ex, _ = exact_pair_scores(q, k, w, bb[c:c + chunk], ss[c:c + chunk], tt[c:c + chunk])
        worst = max(worst, float((vv[c:c + chunk] - ex).abs().max()))
    return worst


def topk_tie_violations(q, k, w, got_idx: torch.Tensor, ref_idx: torch.Tensor, s_rows=None, tie_tol=None):
    """Certify that every top-k set difference is an fp32 tie.

    ``got_idx`` / ``ref_idx`` are ``[B,S',k]`` index sets (``-1`` = empty) of the
    queries ``s_rows`` (default ``arange(S')``).  For each row whose sets
    differ, let ``X`` be the reference picks the candidate missed and ``Y`` the
    candidate's picks the reference did not make.  The candidate ranked every
    ``y`` at or above every ``x``, so the difference is an fp32 tie only if
    ``exact(x) - exact(y) <= allowance`` for every pair.  The allowance is
    ``tie_tol`` (an absolute score tolerance, normally a small multiple of
    :func:`measured_score_error`) or, when None, the worst-case fp32 bound
    ``bound(x) + bound(y)`` of :func:`exact_pair_scores`.  This is the
    north-star rule "exact except at score ties within fp32 epsilon"
    (``eval/test_v4_indexer_parity.py:164-226`` measures the same sets).

    Returns ``(n_rows_differing, worst_excess, n_rows_violating)`` where
    ``worst_excess`` is the largest ``gap - allowance`` seen (``<= 0`` = all ties).
    """
    gi = got_idx.long().cpu()
    ri = ref_idx.long().cpu()
    B, S_, K = gi.shape
    if s_rows is None:
        s_rows = torch.arange(S_)
    s_rows = torch.as_tensor(s_rows).long().cpu()
    n_diff = n_bad = 0
    worst = float("-inf")
    for b in range(B):
        for j in range(S_):
            g = set(int(x) for x in gi[b, j].tolist() if x >= 0)
            r = set(int(x) for x in ri[b, j].tolist() if x >= 0)
            if g == r:
                continue
            n_diff += 1
            if len(r - g) != len(g - r):
                n_bad += 1
                worst = float("inf")
                continue
            X = torch.tensor(sorted(r - g), dtype=torch.long)
            Y = torch.tensor(sorted(g - r), dtype=torch.long)
            s = int(s_rows[j])
            ex, bx = exact_pair_scores(q, k, w, torch.full_like(X, b), torch.full_like(X, s), X)
            ey, by = exact_pair_scores(q, k, w, torch.full_like(Y, b), torch.full_like(Y, s), Y)
            if tie_tol is None:
                excess = float((ex - bx).max() - (ey + by).min())
            else:
                excess = float(ex.max() - ey.min() - tie_tol)
            worst = max(worst, excess)
            if excess > 0:
                n_bad += 1
    return n_diff, (worst if n_diff else 0.0), n_bad
