"""GPU parity of the CSA layer pieces against the oracle and the reference
golden fixtures (window/index build, compressor, score top-k, full CSA)."""

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_window_and_csa_index_golden(golden):
    from streamindex_b200.csa import build_csa_topk_idxs, sliding_window_idxs

    d = golden("window")
    got = sliding_window_idxs(d["B"], d["S"], d["n_win"], "cuda").cpu()
    assert torch.equal(got.long(), d["idx"].long())
    d = golden("csa_idx")
    got = build_csa_topk_idxs(d["scores"].cuda(), d["n_win"], d["top_k"], seq_len=40, n_compressed=10,
                              m=d["m"]).cpu()
    ref = d["idx"]
    nw = d["n_win"]
    assert got.dtype == torch.int32 and got.shape == ref.shape
    assert torch.equal(got[..., :nw], ref[..., :nw])
    assert float(oracle.set_recall(ref[..., nw:], got[..., nw:]).min()) == 1.0


def test_compressor_golden(golden):
    from streamindex_b200.csa import mean_pool_compress

    d = golden("compress")
    got = mean_pool_compress(d["x"].to(torch.bfloat16).cuda(), d["m"]).float().cpu()
    ref = oracle.mean_pool_compress(d["x"].to(torch.bfloat16), d["m"]).float()
    assert (got - ref).abs().max().item() <= 1e-2
    assert (got - d["out"]).abs().max().item() <= 2e-2


def test_scores_topk_matches_oracle():
    from streamindex_b200.csa import scores_topk

    g = torch.Generator().manual_seed(3)
    sc = torch.randn((2, 300, 700), generator=g)
    gi, gv = scores_topk(sc.cuda(), 96, causal_ratio=4)
    legal = torch.arange(700).view(1, 1, -1) < ((torch.arange(300) + 1) // 4).view(1, -1, 1)
    oi, ov = oracle.topk_desc_stable(sc.masked_fill(~legal, float("-inf")), 96)
    oi = torch.where(torch.isinf(ov), torch.full_like(oi, -1), oi)
    assert torch.equal(gi.cpu(), oi)  # distinct random scores: exact order
    assert torch.equal(gv.cpu(), ov)


@pytest.mark.parametrize("d_v", [512, None])
def test_flash_csa_forward_small(d_v):
    """Config-5 shape at small S: compressor -> indexer -> index build -> attention."""
    from streamindex_b200.csa import flash_csa_forward, mean_pool_compress

    B, S, H, D, HI, DI, m, nwin, k = 2, 256, 64, 576, 64, 128, 4, 16, 32
    g = torch.Generator().manual_seed(0)
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).bfloat16()
    x_kv = (torch.randn((B, S, D), generator=g) * D ** -0.5).bfloat16()
    q_idx = (torch.randn((B, S, HI, DI), generator=g) * DI ** -0.5).bfloat16()
    x_k = (torch.randn((B, S, DI), generator=g) * DI ** -0.5).bfloat16()
    w = torch.randn((B, S, HI), generator=g)
    sink = torch.randn(H, generator=g)
    kvc = mean_pool_compress(x_kv.cuda(), m)
    kc = mean_pool_compress(x_k.cuda(), m)
    o = flash_csa_forward(q.cuda(), x_kv.cuda(), kvc, q_idx.cuda(), kc, w.cuda(), sink.cuda(), n_win=nwin, top_k=k,
                          m=m, d_v=d_v)
    torch.cuda.synchronize()
    ro, _, _ = oracle.csa_forward(q, x_kv, kvc.cpu(), q_idx, kc.cpu(), w, sink, nwin, k, m, d_v=d_v)
    assert o.shape == ro.shape
    assert (o.float().cpu() - ro).abs().max().item() <= 2e-2


def test_hca_golden_and_oracle(golden):
    from streamindex_b200.hca import build_hca_topk_idxs, flash_hca_forward

    d = golden("hca")
    B, S = d["q"].shape[:2]
    nc = d["kv_c"].shape[1]
    idx = build_hca_topk_idxs(B=B, seq_len=S, n_win=d["n_win"], n_compressed=nc, m_prime=d["m_prime"],
                              device="cuda").cpu()
    assert torch.equal(idx, oracle.build_hca_topk_idxs(B, S, d["n_win"], nc, d["m_prime"]))
    o = flash_hca_forward(d["q"].cuda(), d["kv"].cuda(), d["kv_c"].cuda(), d["sink"].cuda(), n_win=d["n_win"],
                          m_prime=d["m_prime"])
    torch.cuda.synchronize()
    assert (o.float().cpu() - d["o"]).abs().max().item() <= 2e-2


def test_hca_v4_dims():
    """HCA at V4 dims (D=576/512, m'=128, n_win=128) against the oracle."""
    from streamindex_b200.hca import flash_hca_forward

    B, S, H, D, mp, nw = 1, 1024, 64, 576, 128, 128
    g = torch.Generator().manual_seed(17)
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).bfloat16()
    kv = (torch.randn((B, S, D), generator=g) * D ** -0.5).bfloat16()
    kvc = (torch.randn((B, S // mp, D), generator=g) * D ** -0.5).bfloat16()
    sink = torch.zeros(H)
    o = flash_hca_forward(q.cuda(), kv.cuda(), kvc.cuda(), sink.cuda(), n_win=nw, m_prime=mp, d_v=512)
    torch.cuda.synchronize()
    ro, _, _ = oracle.hca_forward(q, kv, kvc, sink, nw, mp, d_v=512)
    assert (o.float().cpu() - ro).abs().max().item() <= 2e-2


def test_csa_forward_slices_equal_whole_sequence():
    """S-sharding: per-slice CSA forwards (global offsets) concatenate to the
    whole-sequence forward exactly (same kernels, same inputs per query)."""
    from streamindex_b200.csa import csa_forward_slice, flash_csa_forward, mean_pool_compress
    from streamindex_b200.dist import balanced_bounds

    B, S, H, D, HI, DI, m, nwin, k = 2, 512, 64, 576, 64, 128, 4, 16, 32
    g = torch.Generator().manual_seed(5)
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).bfloat16().cuda()
    x_kv = (torch.randn((B, S, D), generator=g) * D ** -0.5).bfloat16().cuda()
    q_idx = (torch.randn((B, S, HI, DI), generator=g) * DI ** -0.5).bfloat16().cuda()
    x_k = (torch.randn((B, S, DI), generator=g) * DI ** -0.5).bfloat16().cuda()
    w = torch.randn((B, S, HI), generator=g).cuda()
    sink = torch.randn(H, generator=g).cuda()
    kvc, kc = mean_pool_compress(x_kv, m), mean_pool_compress(x_k, m)
    full = flash_csa_forward(q, x_kv, kvc, q_idx, kc, w, sink, n_win=nwin, top_k=k, m=m, d_v=512)
    bounds = balanced_bounds(S, 3, S // m, m, align=64, extra_per_query=nwin + k)
    parts = [csa_forward_slice(q[:, a:b], x_kv, kvc, q_idx[:, a:b], kc, w[:, a:b], sink, s_offset=a, n_win=nwin,
                               top_k=k, m=m, d_v=512) for a, b in zip(bounds, bounds[1:])]
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(parts, dim=1), full)


def test_gated_compressor_golden_and_overlap(golden):
    from streamindex_b200.csa import token_compressor

    d = golden("compress_gated")
    got = token_compressor(d["c"].cuda(), d["z"].cuda(), d["b"].cuda(), d["m"]).cpu()
    torch.testing.assert_close(got, d["out"], rtol=1e-4, atol=1e-5)
    g = torch.Generator().manual_seed(23)
    B, S, C, m = 2, 42, 40, 4
    ca, za, cb, zb = (torch.randn((B, S, C), generator=g) for _ in range(4))
    ba, bb = torch.randn((m, C), generator=g), torch.randn((m, C), generator=g)
    got = token_compressor(ca.bfloat16().cuda(), za.bfloat16().cuda(), ba.bfloat16().cuda(), m,
                           c_b=cb.bfloat16().cuda(), z_b=zb.bfloat16().cuda(), b_b=bb.bfloat16().cuda(),
                           overlap=True).float().cpu()
    ref = oracle.token_compressor(ca.bfloat16(), za.bfloat16(), ba.bfloat16(), m, cb.bfloat16(), zb.bfloat16(),
                                  bb.bfloat16(), overlap=True).float()
    assert (got - ref).abs().max().item() <= 2e-2


def test_flash_sparse_reference_module(golden):
    import flash_sparse.reference as R

    d = golden("idx_v4")
    sc = R.reference_lightning_indexer(d["q"].cuda(), d["k"].cuda(), d["w"].cuda()).cpu()
    assert oracle.score_close(sc, d["scores"], 1e-2)
    d = golden("attn_128")
    o = R.reference_sparse_attn(d["q"].cuda(), d["kv"].cuda(), d["sink"].cuda(), d["idx"].cuda())
    assert (o.float().cpu() - d["o"]).abs().max().item() <= 2e-2
    d = golden("hca")
    o = R.reference_hca_forward(d["q"].cuda(), d["kv"].cuda(), d["kv_c"].cuda(), d["sink"].cuda(), d["n_win"],
                                m_prime=d["m_prime"])
    assert (o.float().cpu() - d["o"]).abs().max().item() <= 2e-2
    # CSA with an explicit compressed mask vs the oracle's index build
    g = torch.Generator().manual_seed(29)
    B, S, H, D, T, nw, k = 1, 40, 8, 64, 10, 4, 6
    q = (torch.randn((B, S, H, D), generator=g) * D ** -0.5).bfloat16()
    kv = torch.randn((B, S, D), generator=g).bfloat16()
    kvc = torch.randn((B, T, D), generator=g).bfloat16()
    scores = torch.randn((B, S, T), generator=g)
    legal = (torch.arange(S).view(1, -1, 1) >= (torch.arange(T) + 1).view(1, 1, -1) * 4 - 1)
    sink = torch.randn(H, generator=g)
    o = R.reference_csa_forward(q.cuda(), kv.cuda(), kvc.cuda(), scores.cuda(), sink.cuda(), nw, k,
                                causal_mask_for_compressed=legal.cuda()).float().cpu()
    idx = oracle.build_csa_topk_idxs(scores, nw, k, 4)
    ro, _ = oracle.sparse_attn(q, torch.cat([kv, kvc], dim=1), sink, idx)
    assert (o - ro).abs().max().item() <= 2e-2
