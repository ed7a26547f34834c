"""``flash_sparse.reference`` import path (reference ``flash_sparse/reference.py``),
backed by the B200 kernels.

The reference module is its pure-PyTorch ground truth; code that imports
these names to *compute* (e.g. ``reference_token_compressor`` to build the
compressed kv, ``_build_sliding_window_idxs`` for index lists) gets the CUDA
implementations with the same signatures and results.  ``reference_hc_split_sinkhorn``
(hyper-connection mixing) is not part of the CSA hot path and is not provided.
"""

from __future__ import annotations

from typing import Optional

import torch

from streamindex_b200.attention import sparse_attn_fwd
from streamindex_b200.csa import csa_index_list, scores_topk, sliding_window_idxs, token_compressor
from streamindex_b200.hca import flash_hca_forward
from streamindex_b200.indexer import indexer_score

__all__ = [
    "reference_sparse_attn",
    "reference_lightning_indexer",
    "reference_token_compressor",
    "reference_csa_forward",
    "reference_hca_forward",
]


def reference_sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale: Optional[float] = None):
    """``reference.py:44-130``: full-D output in q's dtype."""
    o, _ = sparse_attn_fwd(q, kv, attn_sink, topk_idxs, softmax_scale)
    return o.to(q.dtype)


def reference_lightning_indexer(q_idx, k_idx, weights):
    """``reference.py:138-168``: ``[B,S,T]`` fp32 scores."""
    return indexer_score(q_idx, k_idx, weights)


def reference_token_compressor(c_a, z_a, b_a, m, *, c_b=None, z_b=None, b_b=None, overlap):
    """``reference.py:176-272``."""
    return token_compressor(c_a, z_a, b_a, m, c_b=c_b, z_b=z_b, b_b=b_b, overlap=overlap)


def reference_csa_forward(q, kv, kv_compressed, indexer_scores, attn_sink, n_win, top_k, *,
                          softmax_scale: Optional[float] = None, causal_mask_for_compressed=None):
    """``reference.py:338-408``: top-k over the given scores (optionally masked),
    window + compressed index list, attention over ``cat[kv; kv_compressed]``."""
    B, S, H, D = q.shape
    n_comp = kv_compressed.shape[1]
    if tuple(indexer_scores.shape) != (B, S, n_comp):
        raise ValueError(f"indexer_scores must be [{B},{S},{n_comp}], got {tuple(indexer_scores.shape)}")
    k = min(top_k, n_comp)
    comp, _ = scores_topk(indexer_scores, k, causal_mask=causal_mask_for_compressed)
    idx = csa_index_list(comp, n_win)
    kv_full = torch.cat([kv, kv_compressed], dim=1)
    o, _ = sparse_attn_fwd(q, kv_full, attn_sink, idx, softmax_scale)
    return o.to(q.dtype)


def reference_hca_forward(q, kv, kv_compressed, attn_sink, n_win, *, m_prime, softmax_scale=None):
    """``reference.py:411-452``."""
    return flash_hca_forward(q, kv, kv_compressed, attn_sink, n_win=n_win, m_prime=m_prime,
                             softmax_scale=softmax_scale).to(q.dtype)


def _build_sliding_window_idxs(B: int, S: int, n_win: int, device) -> torch.Tensor:
    """``reference.py:460-475`` (int64, like the reference)."""
    return sliding_window_idxs(B, S, n_win, device).long()
