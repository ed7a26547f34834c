"""``flash_sparse.triton.chunked_indexer`` (reference path) -> fused B200 indexer + streaming top-k."""

from streamindex_b200.indexer import chunked_indexer_topk  # noqa: F401

__all__ = ["chunked_indexer_topk"]
