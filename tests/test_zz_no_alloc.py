"""GPU test of the allocation-free indexer + top-k entry point.

si_indexer_topk_noalloc serves callers that cannot allocate device memory
themselves (a host runtime that owns the allocator, or code that must not
allocate while other work is in flight): its workspace is a fixed device
array inside the library.  This test calls it through the C ABI, twice in a
row (the array keeps the previous call's contents, so the second call checks
that nothing stale leaks through), and compares each result with the
regular si_indexer_topk given a caller-allocated workspace and with the CPU
oracle, using the same tie-exact parity rule as the other indexer tests, and
reads the path's own status word after each call.  The file name sorts last so a run
that stops at the first failure has already run every other test.
"""

import ctypes

import pytest
import torch

import oracle
from topk_parity import assert_topk_exact_up_to_ties

pytestmark = pytest.mark.gpu


def _regular(lib, _lib, q, k, w, B, S, T, H, D, top_k, ratio):
    oi = torch.empty((B, S, top_k), dtype=torch.int64, device="cuda")
    ov = torch.empty((B, S, top_k), dtype=torch.float32, device="cuda")
    ws_bytes = lib.si_indexer_topk_ws_bytes(B, S, T, H, D, top_k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.si_indexer_topk(q.data_ptr(), k.data_ptr(), w.data_ptr(), 0, 0, B, S, T, H, D, top_k, ratio,
                                   None, oi.data_ptr(), ov.data_ptr(), ws.data_ptr(), ws_bytes,
                                   _lib.stream_handle(q.device)))
    return oi, ov


def _noalloc(lib, _lib, q, k, w, B, S, T, H, D, top_k, ratio):
    oi = torch.empty((B, S, top_k), dtype=torch.int64, device="cuda")
    ov = torch.empty((B, S, top_k), dtype=torch.float32, device="cuda")
    _lib.check(lib.si_indexer_topk_noalloc(q.data_ptr(), k.data_ptr(), w.data_ptr(), 0, 0, B, S, T, H, D, top_k,
                                           ratio, None, oi.data_ptr(), ov.data_ptr(), _lib.stream_handle(q.device)))
    return oi, ov


def test_noalloc_matches_regular_entry_point_twice():
    from streamindex_b200 import _lib

    lib = _lib.load()
    cases = [(1, 2048, 64, 128, 512, 256, 4, 11), (2, 300, 128, 128, 400, 64, 1, 12)]
    for B, S, H, D, T, top_k, ratio, seed in cases:
        qc, kc, wc = oracle.indexer_inputs(B, S, H, D, T, seed=seed)
        oi, ov = oracle.materialize_topk(qc, kc, wc, top_k, ratio=ratio)
        q, k, w = qc.cuda(), kc.cuda(), wc.cuda()
        ri, rv = _regular(lib, _lib, q, k, w, B, S, T, H, D, top_k, ratio)
        for _ in range(2):
            ni, nv = _noalloc(lib, _lib, q, k, w, B, S, T, H, D, top_k, ratio)
            st = ctypes.c_int(-1)
            _lib.check(lib.si_indexer_topk_noalloc_read_status(ctypes.byref(st), _lib.stream_handle(q.device)))
            assert st.value == 0
            # same kernel as the regular entry point: identical results
            assert torch.equal(ni, ri) and torch.equal(nv, rv)
            # and parity with the CPU oracle
            assert_topk_exact_up_to_ties(qc, kc, wc, ni.cpu(), nv.cpu(), oi, ov)


def test_noalloc_rejects_oversized_workspace():
    from streamindex_b200 import _lib

    lib = _lib.load()
    z = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    # H_I=16 keeps 32 queries per SM; top_k=2048 makes the workspace far larger than the array
    rc = lib.si_indexer_topk_noalloc(z.data_ptr(), z.data_ptr(), z.data_ptr(), 0, 0, 1, 1 << 16, 1 << 14, 16, 128,
                                     2048, 4, None, z.data_ptr(), z.data_ptr(), _lib.stream_handle(z.device))
    assert rc == -1
    assert "maximum" in lib.si_last_error().decode()
