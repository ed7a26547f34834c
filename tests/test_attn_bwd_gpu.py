"""GPU parity of the sparse-attention backward (dq, dkv, dsink) against the
reference golden gradients (autograd through reference_sparse_attn) and the
oracle.  Tolerances: the reference's own backward gate
(tests/test_triton_sparse_attn_bwd.py:83-90 of the reference: normalized
correlation difference < 1e-2 for dq / dkv, < 5e-2 for dsink), plus a
max-error bound of 3% of the gradient's largest magnitude."""

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _close(got, ref, corr_tol):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert got.shape == ref.shape
    assert oracle.norm_corr(got, ref) < corr_tol, oracle.norm_corr(got, ref)
    assert (got - ref).abs().max().item() <= 3e-2 * ref.abs().max().item() + 1e-4


def _bwd(q, kv, sink, idx, do, d_v):
    from streamindex_b200.attention import sparse_attn_bwd, sparse_attn_fwd

    q, kv, sink, idx, do = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda(), do.cuda()
    o, lse = sparse_attn_fwd(q, kv, sink, idx, d_v=d_v)
    dq, dkv, ds = sparse_attn_bwd(q, kv, sink, idx, o, lse, do)
    torch.cuda.synchronize()
    return dq, dkv, ds


@pytest.mark.parametrize("name", ["attn_bwd_576", "attn_bwd_128"])
def test_bwd_golden(golden, name):
    d = golden(name)
    dq, dkv, ds = _bwd(d["q"], d["kv"], d["sink"], d["idx"], d["do"], d["d_v"])
    assert dq.dtype == torch.bfloat16 and dkv.dtype == torch.bfloat16 and ds.dtype == torch.float32
    _close(dq, d["dq"], 1e-2)
    _close(dkv, d["dkv"], 1e-2)
    _close(ds, d["dsink"], 5e-2)


@pytest.mark.parametrize("B,S,H,D,N,K,dv", [(1, 96, 64, 576, 2048, 512, 512), (2, 40, 24, 256, 300, 70, 256),
                                            (1, 64, 128, 512, 500, 100, 448), (1, 33, 16, 64, 100, 40, 64),
                                            (1, 20, 80, 128, 64, 64, 96)])
def test_bwd_oracle(B, S, H, D, N, K, dv):
    """Config-4 layout (H=64, D=576/512, K=512) at small S, ragged K, H not a
    multiple of 16, masked slots and an all-masked query."""
    q, kv, sink, idx = oracle.attn_inputs(B, S, H, D, N, K, ratio=1, seed=D + K)
    idx[:, :, 3::5] = -1
    idx[0, 1] = -1
    do = torch.randn((B, S, H, dv), generator=torch.Generator().manual_seed(7)).bfloat16()
    dq, dkv, ds = _bwd(q, kv, sink, idx, do, dv)
    rq, rkv, rs = oracle.sparse_attn_grads(q, kv, sink, idx, do, d_v=dv)
    _close(dq, rq, 1e-2)
    _close(dkv, rkv, 1e-2)
    _close(ds, rs, 5e-2)
    assert dq[0, 1].abs().max().item() == 0.0  # all-masked query: no gradient to q


def test_autograd_wrapper_backward():
    """flash_sparse.triton.sparse_attn through torch.autograd: gradients of q,
    kv and attn_sink equal the oracle's."""
    from flash_sparse.triton import sparse_attn

    q, kv, sink, idx = oracle.attn_inputs(1, 32, 64, 576, 400, 96, ratio=1, seed=77)
    do = torch.randn((1, 32, 64, 512), generator=torch.Generator().manual_seed(8)).bfloat16()
    qg = q.cuda().requires_grad_(True)
    kvg = kv.cuda().requires_grad_(True)
    sg = sink.cuda().requires_grad_(True)
    o = sparse_attn(qg, kvg, sg, idx.cuda(), d_v=512)
    (o.float() * do.cuda().float()).sum().backward()
    rq, rkv, rs = oracle.sparse_attn_grads(q, kv, sink, idx, do, d_v=512)
    _close(qg.grad, rq, 1e-2)
    _close(kvg.grad, rkv, 1e-2)
    _close(sg.grad, rs, 5e-2)
