"""``flash_sparse.triton.indexer_score`` (reference path) -> B200 indexer kernels."""

from streamindex_b200.indexer import indexer_score, indexer_score_topk  # noqa: F401

__all__ = ["indexer_score", "indexer_score_topk"]
