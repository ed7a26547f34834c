"""``flash_sparse.triton`` import path of the reference (``flash_sparse/triton/__init__.py``).

``sparse_attn_fwd`` / ``sparse_attn`` run the B200 CUDA kernel.  The
backward pass is out of scope: ``sparse_attn_bwd`` raises ``NotImplementedError``.
"""

from streamindex_b200.attention import sparse_attn, sparse_attn_fwd  # noqa: F401


def sparse_attn_bwd(*args, **kwargs):
    raise NotImplementedError("sparse attention backward is not part of the B200 build (forward only)")


__all__ = ["sparse_attn", "sparse_attn_fwd", "sparse_attn_bwd"]
