"""StreamIndex-B200: the StreamIndex CSA hot path as hand-written sm_100a CUDA.

Public API (same names and signatures as the reference's Python API):

* indexer:   :func:`chunked_indexer_topk`, :func:`indexer_score`, :func:`indexer_score_topk`
* attention: :func:`sparse_attn_fwd`, :func:`sparse_attn`
* CSA layer: :func:`flash_csa_forward`, :func:`build_csa_topk_idxs`
* HCA layer: :func:`flash_hca_forward`, :func:`build_hca_topk_idxs`
"""

from .attention import sparse_attn, sparse_attn_fwd  # noqa: F401
from .csa import build_csa_topk_idxs, flash_csa_forward, mean_pool_compress  # noqa: F401
from .hca import build_hca_topk_idxs, flash_hca_forward  # noqa: F401
from .indexer import chunked_indexer_topk, indexer_score, indexer_score_topk  # noqa: F401

__all__ = ["chunked_indexer_topk", "indexer_score", "indexer_score_topk", "sparse_attn_fwd", "sparse_attn",
           "flash_csa_forward", "build_csa_topk_idxs", "mean_pool_compress", "flash_hca_forward",
           "build_hca_topk_idxs"]
