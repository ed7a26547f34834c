"""Drop-in import paths of the reference package (``flash_sparse``), backed by
the B200 implementation in :mod:`streamindex_b200`.

``flash_sparse.triton.*`` keeps the reference's module names so existing
imports work unchanged; no Triton code is involved.
"""

__version__ = "0.1.0+b200"
__all__ = ["__version__"]
