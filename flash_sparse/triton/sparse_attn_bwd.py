"""``flash_sparse.triton.sparse_attn_bwd`` import path of the reference: the B200 backward kernel."""

from streamindex_b200.attention import sparse_attn_bwd  # noqa: F401

__all__ = ["sparse_attn_bwd"]
