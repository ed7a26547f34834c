"""``flash_sparse.triton`` import path of the reference (``flash_sparse/triton/__init__.py``).

``sparse_attn_fwd`` / ``sparse_attn_bwd`` / ``sparse_attn`` run the B200 CUDA
kernels (forward and backward, the latter behind the autograd wrapper).
"""

from streamindex_b200.attention import sparse_attn, sparse_attn_bwd, sparse_attn_fwd  # noqa: F401

__all__ = ["sparse_attn", "sparse_attn_fwd", "sparse_attn_bwd"]
