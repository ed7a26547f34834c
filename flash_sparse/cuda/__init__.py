"""``flash_sparse.cuda``: the hand-written sm_100a kernels (C ABI in ``include/streamindex_b200.h``)."""

from streamindex_b200 import (  # noqa: F401
    chunked_indexer_topk,
    flash_csa_forward,
    indexer_score,
    indexer_score_topk,
    sparse_attn,
    sparse_attn_fwd,
)
