"""CPU checks of the Python API surface: the reference import paths resolve,
ops refuse CPU tensors (no CPU fallback), and argument errors match the
reference's exception types."""

import pytest
import torch


def test_flash_sparse_import_paths():
    from flash_sparse.csa import build_csa_topk_idxs, flash_csa_forward  # noqa: F401
    from flash_sparse.hca import build_hca_topk_idxs, flash_hca_forward  # noqa: F401
    from flash_sparse.reference import reference_csa_forward, reference_token_compressor  # noqa: F401
    from flash_sparse.triton import sparse_attn, sparse_attn_bwd, sparse_attn_fwd  # noqa: F401
    from flash_sparse.triton.chunked_indexer import chunked_indexer_topk  # noqa: F401
    from flash_sparse.triton.indexer_score import indexer_score, indexer_score_topk  # noqa: F401
    from flash_sparse.triton.sparse_attn_bwd import sparse_attn_bwd as bwd2

    assert bwd2 is sparse_attn_bwd
    z = torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):  # CPU tensors: no fallback
        sparse_attn_bwd(z, torch.zeros(1, 3, 64, dtype=torch.bfloat16), torch.zeros(4),
                        torch.zeros(1, 2, 2, dtype=torch.int32), z, torch.zeros(1, 2, 4), z)


def test_no_cpu_fallback():
    from streamindex_b200 import chunked_indexer_topk, sparse_attn_fwd

    q = torch.zeros(1, 8, 64, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 128, dtype=torch.bfloat16)
    w = torch.zeros(1, 8, 64)
    with pytest.raises(AssertionError):
        chunked_indexer_topk(q, k, w, 4, causal_ratio=4)
    with pytest.raises(AssertionError):
        sparse_attn_fwd(torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16), torch.zeros(1, 3, 64, dtype=torch.bfloat16),
                        torch.zeros(4), torch.zeros(1, 2, 2, dtype=torch.int32))


def test_mask_and_ratio_are_exclusive():
    from streamindex_b200 import chunked_indexer_topk

    q = torch.zeros(1, 8, 64, 128, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        chunked_indexer_topk(q, torch.zeros(1, 2, 128, dtype=torch.bfloat16), torch.zeros(1, 8, 64), 4,
                             causal_mask=torch.ones(1, 8, 2, dtype=torch.bool), causal_ratio=4)
