"""Failure detection on the GPU without a GPU fault: a kernel wait whose
partner never arrives gives up after its limit, reports a status code the
host reads, and the context stays usable for the next launch."""

import time

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports_status():
    import streamindex_b200 as si
    from streamindex_b200 import _lib

    lib = _lib.load()
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    t0 = time.perf_counter()
    _lib.check(lib.si_selftest_wait_timeout(ws.data_ptr(), 20_000_000, _lib.stream_handle(ws.device)))  # 20 ms
    status = _lib.read_status(ws, ws.device)
    elapsed = time.perf_counter() - t0
    assert status == 1
    assert elapsed < 5.0
    # the context is intact: a real call right after gives correct results
    q, kk, w = oracle.indexer_inputs(1, 128, 64, 128, 32, seed=2)
    gi, _ = si.chunked_indexer_topk(q.cuda(), kk.cuda(), w.cuda(), 8, causal_ratio=4)
    oi, _ = oracle.materialize_topk(q, kk, w, 8, ratio=4)
    assert float(oracle.set_recall(oi, gi.cpu()).mean()) >= 0.999
