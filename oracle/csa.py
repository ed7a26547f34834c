"""Oracle: CSA index build, mean-pool compressor and CSA forward (CPU).  Test infrastructure.

* ``sliding_window_idxs`` — ``_build_sliding_window_idxs``,
  ``flash_sparse/reference.py:460-475``: window ``[max(0,s-n_win+1), s]``,
  absolute positions, ``-1`` when out of range.
* ``build_csa_topk_idxs`` — ``flash_sparse/csa.py:30-83`` (legal iff
  ``(i+1)*m - 1 <= s``, top-k(min(k,T)), ``-1`` on -inf picks, pad to
  ``top_k``, compressed index ``+S``, window first, int32).
* ``mean_pool_compress`` — ``reference_token_compressor(overlap=False)``
  (``reference.py:234-240``) with zero scores and zero bias, i.e. uniform
  softmax weights ``1/m`` over each block of ``m`` tokens; trailing
  ``S % m`` tokens dropped (``reference.py:227-231``).
* ``build_hca_topk_idxs`` / ``hca_forward`` — ``flash_sparse/hca.py:24-51`` and
  ``reference_hca_forward`` (``flash_sparse/reference.py:411-452``): window plus
  every compressed block with ``(i+1)*m' - 1 <= s``.
* ``csa_forward`` — ``flash_csa_forward`` (``flash_sparse/csa.py:86-207``)
  on the reference path: indexer -> index build -> ``cat[kv; kv_compressed]``
  -> sparse attention.
"""

from __future__ import annotations

from typing import Optional

import torch

from .attention import sparse_attn
from .indexer import materialize_topk


def sliding_window_idxs(B: int, S: int, n_win: int) -> torch.Tensor:
    base = torch.arange(S).unsqueeze(-1)
    offs = torch.arange(n_win).unsqueeze(0)
    idx = (base - n_win + 1) + offs
    legal = (idx >= 0) & (idx <= base)
    idx = torch.where(legal, idx, torch.full_like(idx, -1))
    return idx.unsqueeze(0).expand(B, -1, -1).contiguous()


def compressed_to_global(top_idx_in_comp: torch.Tensor, S: int) -> torch.Tensor:
    return torch.where(top_idx_in_comp >= 0, top_idx_in_comp + S, torch.full_like(top_idx_in_comp, -1))


def build_csa_topk_idxs(indexer_scores: torch.Tensor, n_win: int, top_k: int, m: int) -> torch.Tensor:
    """``csa.py:55-83`` on a materialised ``[B,S,T]`` score tensor."""
    from .indexer import topk_desc_stable

    B, S, T = indexer_scores.shape
    block_last = (torch.arange(T) + 1) * m - 1
    legal = torch.arange(S).unsqueeze(-1) >= block_last
    sc = indexer_scores.masked_fill(~legal.unsqueeze(0), float("-inf"))
    k_eff = min(top_k, T)
    ti, tv = topk_desc_stable(sc, k_eff)
    ti = ti.masked_fill(torch.isinf(tv) & (tv < 0), -1)
    if k_eff < top_k:
        ti = torch.cat([ti, torch.full((B, S, top_k - k_eff), -1, dtype=ti.dtype)], dim=-1)
    win = sliding_window_idxs(B, S, n_win)
    return torch.cat([win.long(), compressed_to_global(ti, S).long()], dim=-1).int()


def mean_pool_compress(x: torch.Tensor, m: int) -> torch.Tensor:
    """``[B,S,c]`` -> ``[B,S//m,c]`` mean over each block of m tokens, fp32 math, x's dtype out."""
    B, S, c = x.shape
    nb = S // m
    return x[:, : nb * m].float().reshape(B, nb, m, c).mean(dim=2).to(x.dtype)


def csa_forward(
    q: torch.Tensor,
    kv: torch.Tensor,
    kv_compressed: torch.Tensor,
    q_idx: torch.Tensor,
    k_idx_compressed: torch.Tensor,
    indexer_weights: torch.Tensor,
    attn_sink: torch.Tensor,
    n_win: int,
    top_k: int,
    m: int = 4,
    softmax_scale: Optional[float] = None,
    d_v: Optional[int] = None,
):
    """Reference CSA forward.  Returns ``(o fp32, lse, topk_idxs int32)``."""
    B, S, H, D = q.shape
    T = kv_compressed.shape[1]
    ti, _ = materialize_topk(q_idx, k_idx_compressed, indexer_weights, top_k, ratio=m, pad=True)
    win = sliding_window_idxs(B, S, n_win)
    idxs = torch.cat([win.long(), compressed_to_global(ti, S).long()], dim=-1).int()
    kv_full = torch.cat([kv, kv_compressed], dim=1)
    o, lse = sparse_attn(q, kv_full, attn_sink, idxs, softmax_scale, d_v=d_v)
    return o, lse, idxs


def build_hca_topk_idxs(B: int, S: int, n_win: int, n_compressed: int, m_prime: int) -> torch.Tensor:
    win = sliding_window_idxs(B, S, n_win)
    block_last = (torch.arange(n_compressed) + 1) * m_prime - 1
    legal = torch.arange(S).unsqueeze(-1) >= block_last
    base = torch.arange(n_compressed).view(1, 1, -1).expand(B, S, -1)
    comp = torch.where(legal.unsqueeze(0).expand(B, -1, -1), base, torch.full_like(base, -1))
    return torch.cat([win.long(), compressed_to_global(comp, S).long()], dim=-1).int()


def hca_forward(q, kv, kv_compressed, attn_sink, n_win: int, m_prime: int, softmax_scale=None, d_v=None):
    """Reference HCA forward.  Returns ``(o fp32, lse, idx int32)``."""
    B, S, H, D = q.shape
    idx = build_hca_topk_idxs(B, S, n_win, kv_compressed.shape[1], m_prime)
    kv_full = torch.cat([kv, kv_compressed], dim=1)
    o, lse = sparse_attn(q, kv_full, attn_sink, idx, softmax_scale, d_v=d_v)
    return o, lse, idx


def token_compressor(c_a, z_a, b_a, m, c_b=None, z_b=None, b_b=None, overlap=False):
    """Softmax-gated pooling of m tokens per block (``flash_sparse/reference.py:176-272``).

    overlap=False: ``softmax_m(z_a + b_a)`` weights over each block of m tokens.
    overlap=True: a joint 2m-way softmax over the block's a-stream (``z_a + b_a``)
    and the previous block's b-stream (``z_b + b_b``, -inf / zero value for block
    0).  The shipped reference nests the overlap body under its shape check
    (dead code); this restates the code as written there, un-nested.
    Returns ``[B, S//m, c]`` in c_a's dtype (fp32 math).
    """
    B, S, c = c_a.shape
    nb = S // m
    if nb == 0:
        return c_a.new_zeros(B, 0, c)
    cut = nb * m
    ca = c_a[:, :cut].float().reshape(B, nb, m, c)
    za = z_a[:, :cut].float().reshape(B, nb, m, c) + b_a.float()
    if not overlap:
        return (ca * za.softmax(dim=2)).sum(dim=2).to(c_a.dtype)
    cb = c_b[:, :cut].float().reshape(B, nb, m, c)
    zb = z_b[:, :cut].float().reshape(B, nb, m, c) + b_b.float()
    cbs = torch.zeros_like(cb)
    cbs[:, 1:] = cb[:, :-1]
    zbs = torch.full_like(zb, float("-inf"))
    zbs[:, 1:] = zb[:, :-1]
    cj = torch.cat([ca, cbs], dim=2)
    zj = torch.cat([za, zbs], dim=2)
    return (cj * zj.softmax(dim=2)).sum(dim=2).to(c_a.dtype)
