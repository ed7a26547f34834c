"""Shared top-k parity check for the indexer tests (test infrastructure).

``assert_topk_exact_up_to_ties`` is the north-star rule for the indexer:
scores within 1e-2 relative, valid counts exact, pads (-1, -inf), rows sorted,
and index sets exact except at score ties within fp32 resolution.  A tie is
certified against float64 scores: for every row whose set differs from the
oracle's, each pick the candidate missed must score (exactly) no more than
``tie_tol`` above each pick it made instead.  ``tie_tol`` is derived from the
measured fp32 score error of both the candidate and the oracle on the same
rows (4x their sum, never below 8 fp32 ulps of the largest score), so a
kernel that drops a clear winner fails even in one row out of thousands.
"""

from __future__ import annotations

import torch

import oracle


def _sample_rows(n: int, max_rows: int = 96) -> torch.Tensor:
    if n <= max_rows:
        return torch.arange(n)
    return torch.linspace(0, n - 1, max_rows).round().long().unique()


def tie_tolerance(q, k, w, gi, gv, oi, ov, s_rows=None) -> float:
    """4 x (measured candidate error + measured oracle error), floored at 8 ulps of max |score|."""
    B, S_, _ = gi.shape
    if s_rows is None:
        s_rows = torch.arange(S_)
    s_rows = torch.as_tensor(s_rows).long()
    pick = _sample_rows(S_)
    e_gpu = oracle.measured_score_error(q, k, w, gi[:, pick], gv[:, pick], s_rows[pick])
    e_ref = oracle.measured_score_error(q, k, w, oi[:, pick], ov[:, pick], s_rows[pick])
    fin = ov[torch.isfinite(ov)]
    top = float(fin.abs().max()) if fin.numel() else 1.0
    ulp = top * 2.0 ** -23
    return max(4.0 * (e_gpu + e_ref), 8.0 * ulp)


def assert_topk_exact_up_to_ties(q, k, w, gi, gv, oi, ov, s_rows=None, check_mean_recall=True):
    """Candidate (gi, gv) against oracle (oi, ov) for queries ``s_rows`` of (q, k, w).

    ``check_mean_recall=False`` leaves the mean set recall (>= 0.999) to the
    caller, for callers that check a few rows one at a time."""
    gi, gv, oi, ov = gi.cpu(), gv.cpu(), oi.cpu(), ov.cpu()
    assert gi.shape == oi.shape and gv.shape == ov.shape
    assert torch.equal((gi >= 0).sum(-1), (oi >= 0).sum(-1)), "valid counts differ"
    assert torch.equal(gi < 0, torch.isinf(gv)), "pads must be (-1, -inf)"
    assert bool((gv[..., :-1] >= gv[..., 1:]).all()), "rows not sorted descending"
    assert oracle.score_close(gv, ov, 1e-2), "scores outside 1e-2 relative"
    rec = oracle.set_recall(oi, gi)
    if check_mean_recall:
        assert float(rec.mean()) >= 0.999, float(rec.mean())
    tol = tie_tolerance(q, k, w, gi, gv, oi, ov, s_rows)
    n_diff, worst, n_bad = oracle.topk_tie_violations(q, k, w, gi, oi, s_rows, tie_tol=tol)
    assert n_bad == 0, f"{n_bad} of {n_diff} differing rows are not fp32 ties (worst excess {worst:.3g}, tol {tol:.3g})"
    return n_diff, tol
