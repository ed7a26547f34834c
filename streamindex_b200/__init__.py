"""StreamIndex-B200: the StreamIndex CSA hot path as hand-written sm_100a CUDA.

Public API (same names and signatures as the reference's Python API):

* :func:`chunked_indexer_topk`, :func:`indexer_score`, :func:`indexer_score_topk`
"""

from .indexer import chunked_indexer_topk, indexer_score, indexer_score_topk  # noqa: F401

__all__ = ["chunked_indexer_topk", "indexer_score", "indexer_score_topk"]
