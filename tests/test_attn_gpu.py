"""GPU parity: sparse attention forward against the CPU oracle and the
reference golden fixtures.  Tolerance (north star): output atol 2e-2; LSE
atol 1e-3 (fp32)."""

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _check(q, kv, sink, idx, d_v=None, scale=None, rtol=0.0):
    from streamindex_b200.attention import sparse_attn_fwd

    o, lse = sparse_attn_fwd(q.cuda(), kv.cuda(), sink.cuda(), idx.cuda(), scale, d_v=d_v)
    torch.cuda.synchronize()
    ro, rl = oracle.sparse_attn(q, kv, sink, idx, scale, d_v=d_v)
    o = o.float().cpu()
    assert o.shape == ro.shape
    err = ((o - ro).abs() - rtol * ro.abs()).max().item()
    assert err <= 2e-2, err
    assert oracle.norm_corr(o, ro) < 5e-3
    torch.testing.assert_close(lse.cpu(), rl, atol=1e-3, rtol=1e-4)
    return o, ro


@pytest.mark.parametrize("name", ["attn_576", "attn_128"])
def test_sparse_attn_golden(golden, name):
    d = golden(name)
    from streamindex_b200.attention import sparse_attn_fwd

    o, _ = sparse_attn_fwd(d["q"].cuda(), d["kv"].cuda(), d["sink"].cuda(), d["idx"].cuda())
    assert (o.float().cpu() - d["o"]).abs().max().item() <= 2e-2


def test_mla_576_512_config4_shape():
    """Config-4 layout at small S: H=64, D=576, value = first 512 dims, K=512."""
    q, kv, sink, idx = oracle.attn_inputs(1, 96, 64, 576, 2048, 512, ratio=1, seed=0)
    _check(q, kv, sink, idx, d_v=512)


def test_causal_random_idx_zero_sink():
    q, kv, sink, idx = oracle.attn_inputs(1, 200, 64, 576, 64, 64, ratio=4, seed=1, sink="zeros")
    _check(q, kv, sink, idx, d_v=512)


@pytest.mark.parametrize("H,D,K", [(16, 128, 40), (128, 128, 70), (64, 512, 96), (8, 64, 17)])
def test_heads_dims_and_ragged_k(H, D, K):
    q, kv, sink, idx = oracle.attn_inputs(2, 33, H, D, 150, K, ratio=1, seed=H + D)
    idx[:, :, 3::4] = -1            # every 4th slot masked
    idx[0, 5] = -1                  # one all-masked query -> output 0
    o, ro = _check(q, kv, sink, idx)
    assert o[0, 5].abs().max().item() < 1e-3


def test_large_score_range_rescales():
    """Scores growing along the index list force the running-shift rescale."""
    q, kv, sink, idx = oracle.attn_inputs(1, 8, 64, 128, 512, 256, ratio=1, seed=5)
    kv = (kv.float() * torch.linspace(0.1, 6.0, 512).view(1, -1, 1)).to(torch.bfloat16)
    idx = torch.arange(256, dtype=torch.int32).view(1, 1, -1).expand(1, 8, 256).contiguous() * 2
    # outputs reach ~18 here, where one bf16 ulp is 0.125: allow 1% relative on top of atol
    _check(q * 8, kv, sink, idx, rtol=1e-2)


def test_config4_full_size_sampled_queries():
    """BASELINE configs[3] at full size (S=65536, H=64, D=576/512, N_kv=16384,
    K=512 causal random indices): outputs finite, all-masked rows zero, and
    sampled queries spread over S match the oracle (atol 2e-2)."""
    from streamindex_b200.attention import sparse_attn_fwd

    S, H, D, N, K = 65536, 64, 576, 16384, 512
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    kv = torch.randn((1, N, D), generator=g, device=dev, dtype=torch.bfloat16)
    sink = torch.zeros(H, device=dev)
    # per query s: min(K, (s+1)//4) distinct indices from [0, (s+1)//4), -1 padded
    idx = torch.full((1, S, K), -1, dtype=torch.int32, device=dev)
    t = torch.arange(N, device=dev)
    for s0 in range(0, S, 4096):
        lim = torch.clamp((torch.arange(s0, s0 + 4096, device=dev) + 1) // 4, max=N)
        rnd = torch.rand((4096, N), generator=g, device=dev).masked_fill(t.unsqueeze(0) >= lim.unsqueeze(1), -1.0)
        v, i = rnd.topk(K, dim=-1)
        idx[0, s0:s0 + 4096] = torch.where(v >= 0, i, torch.full_like(i, -1)).int()
    o, lse = sparse_attn_fwd(q, kv, sink, idx, d_v=512)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(o.float()).all()) and bool(torch.isfinite(lse).all())
    assert o[0, 0:3].abs().max().item() == 0.0  # queries 0..2 have no legal key
    rows = [3, 1000, 4095, 20000, 40000, 65535]
    for s_ in rows:
        ro, _ = oracle.sparse_attn(q[:, s_:s_ + 1].cpu(), kv.cpu(), sink.cpu(), idx[:, s_:s_ + 1].cpu(), D ** -0.5,
                                   d_v=512)
        assert (o[:, s_:s_ + 1].float().cpu() - ro).abs().max().item() <= 2e-2


@pytest.mark.parametrize("B,S,H,D,K", [(2, 600, 64, 896, 48), (2, 700, 64, 200, 40), (1, 400, 128, 576, 64)])
def test_q_atom_ring_many_items(B, S, H, D, K):
    """Q sits in tensor memory in a ring of 14 atom slots (64 qk columns each);
    each CTA walks many work items here, so the ring wraps many times: D=896
    fills all 14 slots (no atom of the next item can be preloaded), D=200 is
    not a multiple of 64 (zero-filled tail atom, 10 atoms preloadable), and
    H=128 gives two 64-head items per query."""
    q, kv, sink, idx = oracle.attn_inputs(B, S, H, D, 300, K, ratio=1, seed=D + H)
    idx[:, :, 5::7] = -1
    _check(q, kv, sink, idx)


def test_sink_far_above_scores():
    """A sink ~100 nats above every score: the shift is max(m, sink), so the
    denominator stays finite; O ~ 0 and LSE ~ sink (sparse_attn_fwd.py:152-156)."""
    q, kv, sink, idx = oracle.attn_inputs(1, 16, 64, 128, 64, 32, ratio=1, seed=7)
    sink = torch.full((64,), 100.0)
    sink[::2] = -100.0  # even heads: far below
    o, ro = _check(q, kv, sink, idx)
    assert o[..., 1::2, :].abs().max().item() < 1e-3  # odd heads carry the +100 sink


def test_no_kv_rows_all_masked():
    """N_kv = 0: every slot is masked, O = 0 and LSE = sink, nothing is gathered."""
    from streamindex_b200.attention import sparse_attn_fwd

    H, D = 64, 576
    g = torch.Generator().manual_seed(3)
    q = torch.randn((1, 8, H, D), generator=g).bfloat16().cuda()
    kv = torch.empty((1, 0, D), dtype=torch.bfloat16, device="cuda")
    sink = torch.randn(H, generator=g).cuda()
    idx = torch.randint(0, 4, (1, 8, 16), dtype=torch.int32, device="cuda")
    o, lse = sparse_attn_fwd(q, kv, sink, idx, d_v=512)
    torch.cuda.synchronize()
    assert o.abs().max().item() == 0.0
    torch.testing.assert_close(lse, sink.view(1, 1, H).expand_as(lse), atol=1e-5, rtol=1e-5)


def test_sparse_attn_autograd_wrapper():
    """flash_sparse.triton.sparse_attn (triton/__init__.py:50-61): forward equals
    sparse_attn_fwd's output and carries a grad_fn when an input requires grad
    (the backward is checked in test_attn_bwd_gpu.py)."""
    from flash_sparse.triton import sparse_attn
    from streamindex_b200.attention import sparse_attn_fwd

    q, kv, sink, idx = oracle.attn_inputs(1, 24, 64, 576, 128, 48, ratio=1, seed=9)
    q, kv, sink, idx = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    o_ref, _ = sparse_attn_fwd(q, kv, sink, idx, d_v=512)
    o = sparse_attn(q, kv, sink, idx, d_v=512)
    assert torch.equal(o, o_ref)
    out = sparse_attn(q.clone().requires_grad_(True), kv, sink, idx, d_v=512)
    assert out.requires_grad and out.grad_fn is not None


@pytest.mark.parametrize("D,n_nope", [(576, 512), (512, 448)])
def test_kv_fp8_quantiser_bit_exact(golden, D, n_nope):
    """si_kv_quant_fp8 writes the oracle's FP8 rows byte for byte (e4m3 codes,
    fp32 scales, bf16 rope dims, zero pads); at D=576 on the reference golden."""
    from oracle.kv_fp8 import quantize_rows
    from streamindex_b200.attention import quantize_kv_fp8

    if D == 576:
        kv = golden("kv_fp8")["kv"]
    else:
        g = torch.Generator().manual_seed(31)
        kv = (torch.randn((3, 50, D), generator=g) * torch.logspace(-3, 2, 50).view(1, -1, 1)).bfloat16()
    got = quantize_kv_fp8(kv.cuda(), n_nope).cpu()
    assert torch.equal(got, quantize_rows(kv, n_nope))


@pytest.mark.parametrize("D,n_nope,d_v", [(576, 512, 512), (576, 512, None), (512, 448, 448)])
def test_sparse_attn_fp8_rows(D, n_nope, d_v):
    """Attention over FP8 KV rows equals attention over the dequantised bf16 kv
    (same tile contents: bit-identical to the bf16 kernel) and the oracle on the
    dequantised kv (atol 2e-2); masked slots and an all-masked query included."""
    from oracle.kv_fp8 import dequantize_rows
    from streamindex_b200.attention import quantize_kv_fp8, sparse_attn_fwd, sparse_attn_fwd_fp8kv

    q, kv, sink, idx = oracle.attn_inputs(1, 150, 64, D, 300, 96, ratio=1, seed=D + n_nope)
    idx[:, :, 5::6] = -1
    idx[0, 7] = -1
    rows = quantize_kv_fp8(kv.cuda(), n_nope)
    deq = dequantize_rows(rows.cpu(), D, n_nope)
    dvk = d_v if d_v is not None else D
    o8, l8 = sparse_attn_fwd_fp8kv(q.cuda(), rows, n_nope, sink.cuda(), idx.cuda(), d_v=dvk)
    ob, lb = sparse_attn_fwd(q.cuda(), deq.cuda(), sink.cuda(), idx.cuda(), d_v=dvk)
    torch.cuda.synchronize()
    assert torch.equal(o8, ob) and torch.equal(l8, lb)
    ro, rl = oracle.sparse_attn(q, deq, sink, idx, d_v=dvk)
    assert (o8.float().cpu() - ro).abs().max().item() <= 2e-2
    torch.testing.assert_close(l8.cpu(), rl, atol=1e-3, rtol=1e-4)


def test_full_width_576_single_pass_matches_two_width_passes():
    """The default full-width output (D_v = D = 576) runs as one pass (value
    columns 512..575 accumulate beside S in tensor memory); it equals the
    d_v=512 output on the first 512 columns and the oracle on all 576."""
    from streamindex_b200.attention import sparse_attn_fwd

    q, kv, sink, idx = oracle.attn_inputs(2, 300, 64, 576, 700, 80, ratio=1, seed=57)
    idx[:, :, 2::9] = -1
    o, lse = sparse_attn_fwd(q.cuda(), kv.cuda(), sink.cuda(), idx.cuda())
    o512, lse512 = sparse_attn_fwd(q.cuda(), kv.cuda(), sink.cuda(), idx.cuda(), d_v=512)
    torch.cuda.synchronize()
    assert o.shape[-1] == 576
    assert torch.equal(o[..., :512], o512) and torch.equal(lse, lse512)
    ro, _ = oracle.sparse_attn(q, kv, sink, idx)
    assert (o.float().cpu() - ro).abs().max().item() <= 2e-2


@pytest.mark.parametrize("D,d_v", [(576, 512), (128, None)])
def test_fp16_inputs(D, d_v):
    """fp16 q / kv (sparse_attn_fwd.py:207 accepts bf16 or fp16): fp16 output,
    oracle parity at atol 2e-2 on the same fp16 inputs."""
    from streamindex_b200.attention import sparse_attn_fwd

    q, kv, sink, idx = oracle.attn_inputs(2, 60, 64, D, 200, 48, ratio=1, seed=D + 3)
    q16, kv16 = q.float().half(), kv.float().half()
    idx[:, :, 4::5] = -1
    o, lse = sparse_attn_fwd(q16.cuda(), kv16.cuda(), sink.cuda(), idx.cuda(), d_v=d_v)
    torch.cuda.synchronize()
    assert o.dtype == torch.float16
    ro, rl = oracle.sparse_attn(q16, kv16, sink, idx, d_v=d_v)
    assert (o.float().cpu() - ro).abs().max().item() <= 2e-2
    torch.testing.assert_close(lse.cpu(), rl, atol=1e-3, rtol=1e-4)
