"""Per-tile timeline of the fused indexer kernel (debug build).

Builds ``libstreamindex_b200_trace.so`` (``SI_IDX_TRACE``: %globaltimer
stamps of CTA 0's first query block, up to 512 key tiles) and runs one launch
of the V4-Flash shape at the given S.  CTA 0's first block is the last block
of the sequence, so it sees every key tile.  Prints per-tile durations and
where they go for the producer (0), MMA issuer (1) and epilogue warp 2
(group g: 4g+0 wait for the accumulator, 4g+1 accumulator ready, 4g+2
accumulator released, 4g+3 top-k step done, including any flush).

    python -m streamindex_b200.trace_indexer [S]
"""

from __future__ import annotations

import ctypes
import statistics
import sys

import torch

from . import build as _build
from ._lib import SIGNATURES


def main(S: int = 131072):
    path = _build.build(trace=True, force=True)
    lib = ctypes.CDLL(path)
    for n, (r, a) in SIGNATURES.items():
        f = getattr(lib, n)
        f.restype, f.argtypes = r, a
    lib.si_debug_set_idx_trace.argtypes = [ctypes.c_void_p]
    H, D, k, ratio = 64, 128, 512, 4
    T = S // ratio
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    kk = torch.randn((1, T, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    w = torch.randn((1, S, H), generator=g, device=dev)
    oi = torch.empty((1, S, k), dtype=torch.int64, device=dev)
    ov = torch.empty((1, S, k), dtype=torch.float32, device=dev)
    wsb = lib.si_indexer_topk_ws_bytes(1, S, T, H, D, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    tr = torch.zeros(3 * 512 * 8, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def run():
        rc = lib.si_indexer_topk(q.data_ptr(), kk.data_ptr(), w.data_ptr(), 0, 0, 1, S, T, H, D, k, ratio, None,
                                 oi.data_ptr(), ov.data_ptr(), ws.data_ptr(), wsb, st)
        assert rc == 0, lib.si_last_error()

    run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    print(f"S={S}: {e0.elapsed_time(e1):.3f} ms per launch (untraced stamps off)")
    lib.si_debug_set_idx_trace(tr.data_ptr())
    run()
    torch.cuda.synchronize()
    t = tr.view(3, 512, 8).cpu().double()
    ntiles = int((t[2, :, 0] > 0).sum())
    ep = t[2, :ntiles]
    tile = (ep[1:, 0] - ep[:-1, 0]).tolist()
    wait = [(ep[i, 1] - ep[i, 0] + ep[i, 5] - ep[i, 4]).item() for i in range(ntiles)]
    score = [(ep[i, 2] - ep[i, 1] + ep[i, 6] - ep[i, 5]).item() for i in range(ntiles)]
    topk = [(ep[i, 3] - ep[i, 2] + ep[i, 7] - ep[i, 6]).item() for i in range(ntiles)]
    print(f"tiles traced: {ntiles}; per tile (ns): median {statistics.median(tile):.0f}, mean {statistics.mean(tile):.0f}")
    print(f"  epilogue warp 2, both groups: wait {statistics.mean(wait):.0f}, scores {statistics.mean(score):.0f}, "
          f"top-k {statistics.mean(topk):.0f} (mean ns)")
    slow = sorted(range(ntiles - 1), key=lambda i: -tile[i])[:12]
    print("  slowest tiles (tile, ns, top-k ns):", [(i, int(tile[i]), int(topk[i])) for i in slow])
    print("  top-k ns over tiles (every 16th):", [int(x) for x in topk[::16]])
    # the slice's warps meet every 4th tile (flush decision); other tiles only insert
    for ph in range(4):
        sel = [i for i in range(ntiles) if i % 4 == ph]
        tk0 = [(ep[i, 3] - ep[i, 2]).item() for i in sel]
        tk1 = [(ep[i, 7] - ep[i, 6]).item() for i in sel]
        print(f"  tiles t % 4 == {ph}: top-k step median g0 {statistics.median(tk0):.0f} ns, "
              f"g1 {statistics.median(tk1):.0f} ns")


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 131072)
