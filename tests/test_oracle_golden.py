"""Pin the CPU oracle against outputs of the reference's own functions.

The fixtures under tests/golden/ were produced by make_golden.py, which runs
flash_sparse/reference.py, eval/test_v4_indexer_parity.py and
flash_sparse/csa.py from the reference checkout on seeded inputs.
"""

import torch

import oracle


def test_indexer_scores_match_reference(golden):
    for name in ("idx_v4", "idx_unaligned", "idx_b2"):
        d = golden(name)
        got = oracle.lightning_indexer(d["q"], d["k"], d["w"])
        torch.testing.assert_close(got, d["scores"], rtol=1e-5, atol=1e-5)


def test_materialize_topk_sets_match_reference(golden):
    for name in ("idx_v4", "idx_unaligned", "idx_b2"):
        d = golden(name)
        idx, vals = oracle.materialize_topk(d["q"], d["k"], d["w"], d["top_k"], ratio=d["ratio"], pad=False)
        ref = d["topk_idx"]
        assert idx.shape == ref.shape
        # same valid counts per row, same sets (torch.topk's tie order is undefined)
        assert torch.equal((idx >= 0).sum(-1), (ref >= 0).sum(-1))
        rec = oracle.set_recall(ref, idx)
        assert float(rec.min()) == 1.0, name
        # oracle order: score descending, index ascending on ties
        v = torch.where(idx >= 0, vals, torch.full_like(vals, float("-inf")))
        assert bool((v[..., :-1] >= v[..., 1:]).all())


def test_chunked_equals_materialize_exactly():
    q, k, w = oracle.indexer_inputs(1, 200, 16, 32, 50, seed=5)
    mi, mv = oracle.materialize_topk(q, k, w, 24, ratio=4)
    for cs, ct in [(7, 5), (64, 16), (200, 50), (33, 49)]:
        ci, cv = oracle.chunked_indexer_topk(q, k, w, 24, ratio=4, chunk_s=cs, chunk_t=ct)
        assert torch.equal(ci, mi), (cs, ct)
        # the fp32 einsum over a different key-chunk shape may round differently
        torch.testing.assert_close(cv, mv, rtol=1e-6, atol=1e-6)


def test_sparse_attn_matches_reference(golden):
    for name in ("attn_576", "attn_128"):
        d = golden(name)
        o, lse = oracle.sparse_attn(d["q"].float(), d["kv"].float(), d["sink"], d["idx"])
        torch.testing.assert_close(o, d["o"], rtol=1e-5, atol=1e-5)
        assert torch.isfinite(lse).all()


def test_compressor_window_and_csa_index(golden):
    d = golden("compress")
    torch.testing.assert_close(oracle.mean_pool_compress(d["x"], d["m"]), d["out"], rtol=1e-6, atol=1e-6)
    d = golden("window")
    assert torch.equal(oracle.sliding_window_idxs(d["B"], d["S"], d["n_win"]), d["idx"])
    d = golden("csa_idx")
    got = oracle.build_csa_topk_idxs(d["scores"], d["n_win"], d["top_k"], d["m"])
    ref = d["idx"]
    assert got.dtype == ref.dtype == torch.int32
    nw = d["n_win"]
    assert torch.equal(got[..., :nw], ref[..., :nw])
    assert float(oracle.set_recall(ref[..., nw:], got[..., nw:]).min()) == 1.0


def test_hca_forward_matches_reference(golden):
    d = golden("hca")
    o, _, idx = oracle.hca_forward(d["q"].float(), d["kv"].float(), d["kv_c"].float(), d["sink"], d["n_win"],
                                   d["m_prime"])
    torch.testing.assert_close(o, d["o"], rtol=1e-5, atol=1e-5)
    assert idx.dtype == torch.int32


def test_gated_compressor_matches_reference(golden):
    d = golden("compress_gated")
    got = oracle.token_compressor(d["c"], d["z"], d["b"], d["m"])
    torch.testing.assert_close(got, d["out"], rtol=1e-5, atol=1e-5)
    # zero scores and bias reduce it to the mean pool
    z0 = torch.zeros_like(d["z"])
    torch.testing.assert_close(oracle.token_compressor(d["c"], z0, torch.zeros_like(d["b"]), d["m"]),
                               oracle.mean_pool_compress(d["c"], d["m"]), rtol=1e-6, atol=1e-6)


def test_tie_certificate_accepts_ties_and_rejects_a_dropped_winner():
    """The top-k parity rule used by the GPU tests: an fp32 reordering passes,
    one clear winner swapped for a loser fails even in one row of many."""
    import sys, os
    sys.path.insert(0, os.path.dirname(__file__))
    from topk_parity import assert_topk_exact_up_to_ties

    q, k, w = oracle.indexer_inputs(1, 512, 64, 128, 128, seed=5)
    oi, ov = oracle.materialize_topk(q, k, w, 16, ratio=4)
    # a candidate ranked by float64 scores (another rounding) passes
    sc64 = (torch.einsum("bshd,btd->bsht", q.double(), k.double()).clamp_min(0) * w.double()[..., None]).sum(2)
    legal = torch.arange(128).view(1, 1, -1) < ((torch.arange(512) + 1) // 4).view(1, -1, 1)
    ci, cv = oracle.topk_desc_stable(sc64.masked_fill(~legal, float("-inf")), 16)
    ci = torch.where(torch.isinf(cv), torch.full_like(ci, -1), ci)
    assert_topk_exact_up_to_ties(q, k, w, ci, cv.float(), oi, ov)
    # swap the best pick of one row for its best non-pick: must fail
    bad_i, bad_v = oi.clone(), ov.clone()
    s = 400
    sc = oracle.lightning_indexer(q[:, s:s + 1], k, w[:, s:s + 1])[0, 0]
    lim = (s + 1) // 4
    order = torch.sort(sc[:lim], descending=True, stable=True).indices
    loser = int(order[16])
    bad_i[0, s] = torch.cat([bad_i[0, s, 1:], torch.tensor([loser])])
    bad_v[0, s] = torch.cat([bad_v[0, s, 1:], sc[loser:loser + 1]])
    try:
        assert_topk_exact_up_to_ties(q, k, w, bad_i, bad_v, oi, ov)
    except AssertionError:
        return
    raise AssertionError("a dropped winner passed the tie certificate")


def test_kv_fp8_quant_matches_reference_simulation(golden):
    """FP8 KV rows: the oracle's dequantised NoPE dims equal the reference's
    act_quant_simulate(kv[..., :512], 64) bit for bit; rope dims pass through."""
    from oracle.kv_fp8 import dequantize_rows, quantize_rows, row_layout

    d = golden("kv_fp8")
    rows = quantize_rows(d["kv"], d["n_nope"])
    assert rows.shape[-1] == row_layout(576, 512)[1] == 672
    deq = dequantize_rows(rows, 576, d["n_nope"])
    assert torch.equal(deq[..., :512], d["deq"])
    assert torch.equal(deq[..., 512:], d["kv"][..., 512:])


def test_attention_grads_match_reference_autograd(golden):
    """The oracle's backward (autograd through its sparse attention) equals the
    gradients of the reference's own reference_sparse_attn."""
    for name in ("attn_bwd_576", "attn_bwd_128"):
        d = golden(name)
        dq, dkv, ds = oracle.sparse_attn_grads(d["q"], d["kv"], d["sink"], d["idx"], d["do"], d_v=d["d_v"])
        torch.testing.assert_close(dq, d["dq"], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(dkv, d["dkv"], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(ds, d["dsink"], atol=1e-4, rtol=1e-4)
