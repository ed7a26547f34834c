"""Host-side S-sharding logic on CPU: balanced boundaries and a world-size-2
gloo run of the key broadcast and the rank-0 gather used by bench.py."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from streamindex_b200.dist import balanced_bounds, legal_pairs


def test_legal_pairs_closed_form():
    S, T, r = 1000, 250, 4
    s = np.arange(S)
    assert legal_pairs(S, T, r) == int(np.minimum(T, (s + 1) // r).sum())
    assert legal_pairs(S, T, None) == S * T
    assert legal_pairs(S, T, r, 100, 300) == int(np.minimum(T, (s[100:300] + 1) // r).sum())


@pytest.mark.parametrize("N", [2, 4, 8])
def test_balanced_bounds_split_work_evenly(N):
    S, T = 1 << 20, 1 << 18
    b = balanced_bounds(S, N, T, 4)
    assert b[0] == 0 and b[-1] == S and all(x <= y for x, y in zip(b, b[1:]))
    assert all(x % 128 == 0 for x in b[:-1])
    work = [legal_pairs(S, T, 4, lo, hi) for lo, hi in zip(b, b[1:])]
    assert max(work) / min(work) < 1.01
    # equal-length slices would be far from balanced under the causal mask
    eq = [legal_pairs(S, T, 4, i * S // N, (i + 1) * S // N) for i in range(N)]
    assert max(eq) / min(eq) > 2


def test_csa_bounds_weight_the_attention():
    """CSA slices: the per-query attention cost (weighted by the kernels'
    measured relative speed) moves queries off the early, attention-heavy
    ranks; each slice's modelled work is equal."""
    from streamindex_b200.dist import csa_query_cost_pairs

    S, m = 131072, 4
    e = csa_query_cost_pairs(64, 576, 512, 64, 128, 128, 512)
    flops_only = (128 + 512) * 64 * (576 + 512) / (64 * 128)
    assert e > flops_only
    b = balanced_bounds(S, 8, S // m, m, align=128, extra_per_query=e)
    b0 = balanced_bounds(S, 8, S // m, m, align=128, extra_per_query=flops_only)
    assert b[1] < b0[1]
    work = [legal_pairs(S, S // m, m, lo, hi) + e * (hi - lo) for lo, hi in zip(b, b[1:])]
    assert max(work) / min(work) < 1.02  # 128-query alignment


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, S, k, q):
    import torch.distributed as dist

    from streamindex_b200.dist import balanced_bounds, broadcast_keys, gather_to_rank0

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        keys = torch.arange(12.0) if rank == 0 else torch.zeros(12)
        broadcast_keys(keys)
        assert torch.equal(keys, torch.arange(12.0))
        b = balanced_bounds(S, world, S // 4, 4, align=8)
        lo, hi = b[rank], b[rank + 1]
        local = (torch.arange(lo, hi, dtype=torch.int64).view(1, -1, 1) * 10).expand(1, hi - lo, k).contiguous()
        full = torch.empty((1, S, k), dtype=torch.int64) if rank == 0 else None
        gather_to_rank0(local, b, full)
        if rank == 0:
            ref = (torch.arange(S, dtype=torch.int64).view(1, -1, 1) * 10).expand(1, S, k)
            q.put(bool(torch.equal(full, ref)))
    finally:
        dist.destroy_process_group()


def test_gloo_broadcast_and_gather_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 200, 3, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True


def _failing_worker(rank, world, port, q):
    """A rank that raises before the collective: the survivor's collective must
    end with an error within the process-group timeout instead of hanging."""
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(3)  # injected failure: leaves before the broadcast
    try:
        t = torch.zeros(4)
        dist.broadcast(t, src=1)
        q.put("no-error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert q.get(timeout=5) != "no-error"
