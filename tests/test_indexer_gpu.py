"""GPU parity: fused indexer + streaming top-k against the CPU oracle.

Tolerances (north star): scores within 1e-2 relative; top-k index sets exact
except at fp32-epsilon ties (every differing pick certified as a tie against
float64 scores, ``tests/topk_parity.py``), set recall >= 0.999; valid counts
exact.
"""

import pytest
import torch

import oracle
from topk_parity import assert_topk_exact_up_to_ties

pytestmark = pytest.mark.gpu


def _run(B, S, H, D, T, k, ratio, seed=0, w_dtype=torch.float32, mask=False):
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(B, S, H, D, T, seed=seed, w_dtype=w_dtype)
    cm = None
    if mask:
        g = torch.Generator().manual_seed(seed + 1)
        cm = torch.rand((B, S, T), generator=g) < 0.6
    gi, gv = si.chunked_indexer_topk(q.cuda(), kk.cuda(), w.cuda(), k,
                                     causal_ratio=ratio, causal_mask=None if cm is None else cm.cuda())
    torch.cuda.synchronize()
    oi, ov = oracle.materialize_topk(q, kk, w, k, ratio=ratio, causal_mask=cm)
    assert_topk_exact_up_to_ties(q, kk, w, gi.cpu(), gv.cpu(), oi, ov)
    return gi.cpu(), gv.cpu(), oi, ov


@pytest.mark.parametrize("H,D", [(64, 128), (128, 128), (16, 64), (32, 32)])
def test_indexer_topk_small(H, D):
    _run(1, 300, H, D, 75, 16, ratio=4, seed=H + D)


def test_indexer_topk_config1():
    """B=1, S=4096, H_I=64, D_I=128, T=1024, k=512, ratio 4, seed 0."""
    _run(1, 4096, 64, 128, 1024, 512, ratio=4, seed=0)


@pytest.mark.parametrize("S", [2048, 8192])
def test_indexer_topk_v4_flash_published_parity_sizes(S):
    """The published parity points at V4-Flash dims (S = 2048 and 8192 beside
    config 1's 4096; benchmarks/results/2026-04-27/parity_v4_flash_indexer_final.log:6-8):
    H_I=64, D_I=128, T=S/4, k=512, ratio 4, CPU-generated from seed 0."""
    _run(1, S, 64, 128, S // 4, 512, ratio=4, seed=0)


def test_indexer_topk_no_mask_and_bf16_weights():
    _run(2, 130, 64, 128, 520, 40, ratio=None, seed=3, w_dtype=torch.bfloat16)


def test_indexer_topk_explicit_mask():
    _run(1, 96, 64, 128, 300, 32, ratio=None, seed=4, mask=True)


def test_indexer_topk_k_larger_than_T_and_unaligned():
    """Reference test shape: S=47, T=73 with k > legal count (padding)."""
    _run(1, 47, 16, 32, 73, 100, ratio=1, seed=901)


def test_indexer_score_materialised():
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(1, 200, 64, 128, 333, seed=9)
    got = si.indexer_score(q.cuda(), kk.cuda(), w.cuda()).cpu()
    ref = oracle.lightning_indexer(q, kk, w)
    assert oracle.score_close(got, ref, 1e-2)
    assert oracle.norm_corr(got, ref) < 5e-3


def test_indexer_topk_v4_pro_dims():
    """BASELINE config 3 dims at small S: H_I=128, top_k=1024, ratio 4."""
    _run(1, 8192, 128, 128, 2048, 1024, ratio=4, seed=2)


def test_run_host_pipelined_matches_device_path():
    """Host-buffer pipelined path (query slices, overlapped copies) == device path, bit for bit."""
    from streamindex_b200.indexer import IndexerTopk

    S, H, D, T, k = 3000, 64, 128, 750, 64
    q, kk, w = oracle.indexer_inputs(1, S, H, D, T, seed=21)
    plan = IndexerTopk(1, S, T, H, D, k, causal_ratio=4, device="cuda")
    di, dv = plan.run(q.cuda(), kk.cuda(), w.cuda())
    di, dv = di.cpu().clone(), dv.cpu().clone()
    hq, hk, hw = q.pin_memory(), kk.pin_memory(), w.pin_memory()
    hi = torch.empty((1, S, k), dtype=torch.int64).pin_memory()
    hs = torch.empty((1, S, k), dtype=torch.float32).pin_memory()
    for chunks in (1, 5):
        plan.run_host(hq, hk, hw, hi, hs, chunks=chunks)
        assert torch.equal(hi, di) and torch.equal(hs, dv)


@pytest.mark.parametrize("H,k", [(64, 512), (128, 1024)])
def test_full_size_config2_properties_and_sampled_rows(H, k):
    """BASELINE configs[1] (H_I=64, k=512) and configs[2] (V4-Pro: H_I=128,
    k=1024) at their largest size, S=1,048,576 (T=262,144):
    size-independent properties on every row (sorted descending, indices legal
    under t < (s+1)//4 and distinct, exact valid counts min(k, (s+1)//4), pads
    -1/-inf) plus exact oracle parity on sampled rows spread over S."""
    from streamindex_b200.indexer import IndexerTopk

    S, D, r = 1 << 20, 128, 4
    T = S // r
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    kk = torch.randn((1, T, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    w = torch.randn((1, S, H), generator=g, device=dev)
    plan = IndexerTopk(1, S, T, H, D, k, causal_ratio=r, device=dev)
    idx, sc = plan.run(q, kk, w)
    torch.cuda.synchronize()
    assert plan.status() == 0
    s = torch.arange(S, device=dev).view(1, S, 1)
    lim = torch.clamp((s + 1) // r, max=T)
    valid = idx >= 0
    assert torch.equal(valid.sum(-1, keepdim=True), torch.clamp(lim, max=k))
    assert bool(((idx < lim) | ~valid).all())
    assert torch.equal(valid, torch.isfinite(sc))
    assert bool((sc[..., :-1] >= sc[..., 1:]).all())
    srt, _ = torch.where(valid, idx, torch.full_like(idx, -1)).sort(dim=-1)
    dup = (srt[..., 1:] == srt[..., :-1]) & (srt[..., 1:] >= 0)
    assert not bool(dup.any())
    # oracle on sampled rows (full key range of each): per-row recall >= 0.999
    # unless every difference is a certified fp32 tie
    rows = [5, 2047, 2048, 100003, 524287, 777777, S - 1]
    kc = kk.cpu()
    recalls = []
    for s_ in rows:
        qs = q[:, s_:s_ + 1].cpu()
        ws = w[:, s_:s_ + 1].cpu()
        n = min(T, (s_ + 1) // r)
        sc_ref = oracle.lightning_indexer(qs, kc[:, :n], ws)
        oi, ov = oracle.topk_desc_stable(sc_ref, min(k, n))
        gi = idx[:, s_:s_ + 1, : min(k, n)].cpu()
        gv = sc[:, s_:s_ + 1, : min(k, n)].cpu()
        assert_topk_exact_up_to_ties(qs, kc, ws, gi, gv, oi, ov, s_rows=[0], check_mean_recall=False)
        recalls.append(float(oracle.set_recall(oi, gi)))
    assert sum(recalls) / len(recalls) >= 0.999, recalls


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_devices_one_process():
    """Kernel attributes are set per device: the same process can run on cuda:0 then cuda:1."""
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(1, 256, 64, 128, 64, seed=8)
    out = [si.chunked_indexer_topk(q.to(d), kk.to(d), w.to(d), 16, causal_ratio=4)[0].cpu()
           for d in ("cuda:0", "cuda:1")]
    assert torch.equal(out[0], out[1])


@pytest.mark.parametrize("H,D", [(16, 64), (128, 128)])
def test_indexer_score_other_heads(H, D):
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(2, 70, H, D, 150, seed=H)
    got = si.indexer_score(q.cuda(), kk.cuda(), w.cuda()).cpu()
    ref = oracle.lightning_indexer(q, kk, w)
    assert oracle.score_close(got, ref, 1e-2)


def test_indexer_score_topk_width_and_mask():
    """indexer_score_topk returns width min(top_k, T); -1/-inf where no legal key."""
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(1, 64, 64, 128, 40, seed=31)
    cm = torch.rand((1, 64, 40), generator=torch.Generator().manual_seed(3)) < 0.5
    gi, gv = si.indexer_score_topk(q.cuda(), kk.cuda(), w.cuda(), 100, causal_mask=cm.cuda())
    assert gi.shape == (1, 64, 40)
    oi, ov = oracle.materialize_topk(q, kk, w, 100, causal_mask=cm, pad=False)
    assert_topk_exact_up_to_ties(q, kk, w, gi.cpu(), gv.cpu(), oi, ov)


def test_indexer_fp16_operands():
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(1, 256, 64, 128, 64, seed=41)
    q16, k16 = q.float().half(), kk.float().half()
    gi, gv = si.chunked_indexer_topk(q16.cuda(), k16.cuda(), w.cuda(), 24, causal_ratio=4)
    oi, ov = oracle.materialize_topk(q16, k16, w, 24, ratio=4)
    assert_topk_exact_up_to_ties(q16, k16, w, gi.cpu(), gv.cpu(), oi, ov)


def test_exact_ties_prefer_smaller_index():
    """Exact score ties resolve toward the smaller key index
    (docs/streaming_topk.md:48-66, 301-305): keys 32..63 duplicate keys 0..31,
    so every score occurs twice; whenever key j >= 32 is selected, key j - 32
    must be selected too and placed before it."""
    import streamindex_b200 as si

    q, kk, w = oracle.indexer_inputs(1, 200, 64, 128, 64, seed=71)
    kk[:, 32:] = kk[:, :32]
    gi, gv = si.chunked_indexer_topk(q.cuda(), kk.cuda(), w.cuda(), 40, causal_ratio=None)
    gi, gv = gi.cpu(), gv.cpu()
    for s in range(gi.shape[1]):
        row = gi[0, s].tolist()
        pos = {t: i for i, t in enumerate(row)}
        for t in row:
            if t >= 32:
                assert t - 32 in pos and pos[t - 32] < pos[t], (s, t)
                assert gv[0, s, pos[t]] == gv[0, s, pos[t - 32]]
    oi, ov = oracle.materialize_topk(q, kk, w, 40)
    assert_topk_exact_up_to_ties(q, kk, w, gi, gv, oi, ov)


def test_sharded_slices_equal_whole_sequence():
    """The S-sharded indexer (work-balanced contiguous slices with a global
    query offset, as each rank runs them) concatenates to the single-call
    result bit for bit; chunk_s / chunk_t do not change results."""
    import streamindex_b200 as si
    from streamindex_b200.dist import INDEXER_QUERY_COST_PAIRS, balanced_bounds
    from streamindex_b200.indexer import indexer_topk_slice

    S, H, D, T, k = 4096, 64, 128, 1024, 256
    q, kk, w = oracle.indexer_inputs(2, S, H, D, T, seed=72)
    q, kk, w = q.cuda(), kk.cuda(), w.cuda()
    full_i, full_v = si.chunked_indexer_topk(q, kk, w, k, causal_ratio=4)
    alt_i, alt_v = si.chunked_indexer_topk(q, kk, w, k, causal_ratio=4, chunk_s=512, chunk_t=128)
    assert torch.equal(full_i, alt_i) and torch.equal(full_v, alt_v)
    bounds = balanced_bounds(S, 5, T, 4, extra_per_query=INDEXER_QUERY_COST_PAIRS)
    parts = [indexer_topk_slice(q[:, a:b], kk, w[:, a:b], k, 4, a) for a, b in zip(bounds, bounds[1:])]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat([p[0] for p in parts], dim=1), full_i)
    assert torch.equal(torch.cat([p[1] for p in parts], dim=1), full_v)
