"""``flash_sparse.triton.sparse_attn_fwd`` (reference path) -> B200 sparse attention forward."""

from streamindex_b200.attention import sparse_attn_fwd  # noqa: F401

__all__ = ["sparse_attn_fwd"]
