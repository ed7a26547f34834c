"""Oracle: sparse attention with attention sink, MQA layout (CPU, fp32).  Test infrastructure.

Restates ``reference_sparse_attn`` (``flash_sparse/reference.py:44-130``)
without its shipped defects (``.dim``/``.exp`` missing their call
parentheses, body nested under ``if softmax_scale is None``):

* gather ``kv[idx]`` with ``-1`` clamped to row 0 and zeroed (``:93-105``);
* ``scores = q . kv * scale`` masked to ``-inf`` where ``idx < 0`` (``:108-109``);
* shift by ``max(scores U {sink})`` (``-inf`` shift replaced by 0, ``:117-122``);
* ``denom = sum exp(scores - m) + exp(sink - m)``; sink is in the denominator
  only (``:124-126``);
* ``out = sum exp(scores - m) * v / denom`` (``:129``).

The log-sum-exp returned alongside is the one ``sparse_attn_fwd`` stores,
``lse = log(l) + m`` with ``-1e30`` when ``l == 0``
(``flash_sparse/triton/sparse_attn_fwd.py:175``).

``d_v`` selects how many leading dims of a kv row are the value (the caller
slices ``[..., :512]`` for the 576/512 MLA layout, ``reference.py:68-72``).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch


def sparse_attn(
    q: torch.Tensor,
    kv: torch.Tensor,
    attn_sink: torch.Tensor,
    topk_idxs: torch.Tensor,
    softmax_scale: Optional[float] = None,
    d_v: Optional[int] = None,
    s_chunk: int = 64,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns ``(o fp32 [B,S,H,d_v], lse fp32 [B,S,H])``."""
    assert q.dim() == 4 and kv.dim() == 3
    B, S, H, D = q.shape
    assert kv.shape[0] == B and kv.shape[2] == D
    assert attn_sink.shape == (H,)
    assert topk_idxs.shape[:2] == (B, S)
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    dv = D if d_v is None else int(d_v)
    o = torch.empty((B, S, H, dv), dtype=torch.float32)
    lse = torch.empty((B, S, H), dtype=torch.float32)
    sink = attn_sink.float().view(1, 1, H, 1)
    kvf = kv.float()
    for s0 in range(0, S, s_chunk):
        s1 = min(S, s0 + s_chunk)
        idx = topk_idxs[:, s0:s1].long()
        valid = idx >= 0
        safe = idx.clamp_min(0)
        g = torch.stack([kvf[b][safe[b]] for b in range(B)])  # [B, s, K, D]
        g = g * valid.unsqueeze(-1).float()
        sc = torch.einsum("bshd,bskd->bshk", q[:, s0:s1].float(), g) * softmax_scale
        sc = sc.masked_fill(~valid.unsqueeze(2), float("-inf"))
        m = torch.maximum(sc.amax(dim=-1, keepdim=True), sink)
        m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
        p = (sc - m).exp()
        denom = p.sum(dim=-1) + (sink - m).exp().squeeze(-1)
        o[:, s0:s1] = torch.einsum("bshk,bskd->bshd", p, g[..., :dv]) / denom.unsqueeze(-1)
        mm = m.squeeze(-1)
        lse[:, s0:s1] = torch.where(denom > 0, torch.log(denom) + mm, torch.full_like(denom, -1.0e30))
    return o, lse


def sparse_attn_grads(q, kv, attn_sink, topk_idxs, do, softmax_scale=None, d_v=None):
    """``(dq, dkv, dsink)`` of ``sum(sparse_attn(...)[0] * do)`` by autograd through :func:`sparse_attn`
    in fp32 (the reference's backward math, ``flash_sparse/triton/sparse_attn_bwd.py:1-30``)."""
    qf = q.detach().float().requires_grad_(True)
    kvf = kv.detach().float().requires_grad_(True)
    sf = attn_sink.detach().float().clone().requires_grad_(True)
    o, _ = sparse_attn(qf, kvf, sf, topk_idxs, softmax_scale, d_v=d_v)
    (o * do.float()).sum().backward()
    return qf.grad, kvf.grad, sf.grad
