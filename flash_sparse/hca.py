"""``flash_sparse.hca`` (reference ``flash_sparse/hca.py``): HCA layer forward."""

from streamindex_b200.hca import build_hca_topk_idxs, flash_hca_forward  # noqa: F401

__all__ = ["flash_hca_forward", "build_hca_topk_idxs"]
