"""``flash_sparse.csa`` (reference ``flash_sparse/csa.py``): CSA layer forward."""

from streamindex_b200.csa import build_csa_topk_idxs, flash_csa_forward  # noqa: F401

__all__ = ["flash_csa_forward", "build_csa_topk_idxs"]
