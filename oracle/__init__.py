"""CPU oracle for the StreamIndex CSA hot path — TEST INFRASTRUCTURE ONLY.

This package is a defect-free CPU restatement of the reference's math
(tsukimia-hoshi/StreamIndex, ``flash_sparse/reference.py``,
``flash_sparse/triton/chunked_indexer.py``, ``flash_sparse/csa.py`` and
``eval/test_v4_indexer_parity.py``).  It is the checker the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it;
the product package (``streamindex_b200``) never does, and it has no CPU
fallback that could route through here.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
functions (with a shim that restores the call parentheses dropped from the
shipped source) on seeded inputs and stores their outputs as fixtures;
``tests/test_oracle_golden.py`` checks this restatement against them.
"""

from .indexer import (  # noqa: F401
    causal_limit,
    lightning_indexer,
    materialize_topk,
    chunked_indexer_topk,
    topk_desc_stable,
)
from .attention import sparse_attn, sparse_attn_grads  # noqa: F401
from .csa import (  # noqa: F401
    sliding_window_idxs,
    build_csa_topk_idxs,
    mean_pool_compress,
    csa_forward,
    build_hca_topk_idxs,
    hca_forward,
    token_compressor,
)
from .metrics import (  # noqa: F401
    set_recall, norm_corr, score_close, exact_pair_scores, measured_score_error, topk_tie_violations,
)
from .inputs import indexer_inputs, attn_inputs  # noqa: F401
