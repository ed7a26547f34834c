"""Strided inputs are read in place (q / k / w of the indexer, q of the
attention): results are bit-identical to the same values passed contiguous.
The reference hands its Triton kernels arbitrary strides
(flash_sparse/triton/indexer_score.py:162-170, sparse_attn_fwd.py:267-270)."""

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_indexer_strided_q_k_w():
    import streamindex_b200 as si

    B, S, H, D, T, k = 2, 300, 64, 128, 120, 32
    q, kk, w = oracle.indexer_inputs(B, S, H, D, T, seed=41)
    q, kk, w = q.cuda(), kk.cuda(), w.cuda()
    ref_i, ref_v = si.chunked_indexer_topk(q, kk, w, k, causal_ratio=4)
    # q: padded head rows (h stride D+8) and a head-major layout viewed as [B,S,H,D]
    qpad = torch.zeros((B, S, H, D + 8), dtype=q.dtype, device="cuda")
    qpad[..., :D] = q
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)
    kpad = torch.zeros((B, T, 2 * D), dtype=kk.dtype, device="cuda")
    kpad[..., :D] = kk
    wpad = torch.zeros((B, S, H + 4), dtype=w.dtype, device="cuda")
    wpad[..., :H] = w
    for qv in (qpad[..., :D], qt):
        gi, gv = si.chunked_indexer_topk(qv, kpad[..., :D], wpad[..., :H], k, causal_ratio=4)
        torch.cuda.synchronize()
        assert torch.equal(gi, ref_i) and torch.equal(gv, ref_v)


@pytest.mark.parametrize("H", [64, 16])
def test_attention_strided_q(H):
    from streamindex_b200.attention import sparse_attn_fwd

    q, kv, sink, idx = oracle.attn_inputs(2, 100, H, 576, 400, 64, ratio=1, seed=H)
    q, kv, sink, idx = q.cuda(), kv.cuda(), sink.cuda(), idx.cuda()
    o_ref, l_ref = sparse_attn_fwd(q, kv, sink, idx, d_v=512)
    qpad = torch.zeros((2, 100, H, 584), dtype=q.dtype, device="cuda")
    qpad[..., :576] = q
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)
    for qv in (qpad[..., :576], qt):
        assert not qv.is_contiguous()
        o, lse = sparse_attn_fwd(qv, kv, sink, idx, d_v=512)
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(lse, l_ref)
