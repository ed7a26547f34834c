"""Per-tile timeline of the sparse-attention kernel (debug build).

Builds ``libstreamindex_b200_trace.so`` (the same sources with
``SI_ATTN_TRACE``: %globaltimer stamps of CTA 0's first four work items, 16
tiles each, for the gather, MMA-issue and softmax roles), runs one config-4
shaped launch and prints the stamps of item 2 relative to the first stamp (ns).

    python -m streamindex_b200.trace_attn [S]

Softmax points: 0 wait for S | 1 S and mask ready | 2 S loaded from TMEM |
5 max / exp / sum done | 3 P buffer free (P.V of an earlier tile complete) |
4 P published.  Issuers: 0 Q.K^T waits | 3 Q.K^T committed | 4 P ready for
P.V | 5 P.V committed.  Gather: 0 index wait | 1 stage free | 2 copies issued.
"""

from __future__ import annotations

import ctypes
import sys

import torch

from . import build as _build
from ._lib import SIGNATURES


def main(S: int = 16384):
    path = _build.build(trace=True, force=True)
    lib = ctypes.CDLL(path)
    for n, (r, a) in SIGNATURES.items():
        f = getattr(lib, n)
        f.restype, f.argtypes = r, a
    lib.si_debug_set_attn_trace.argtypes = [ctypes.c_void_p]
    H, D, DV, NKV, K = 64, 576, 512, 16384, 512
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    kv = torch.randn((1, NKV, D), generator=g, device=dev, dtype=torch.bfloat16)
    sink = torch.zeros(H, device=dev)
    idx = torch.randint(0, NKV, (1, S, K), generator=g, device=dev, dtype=torch.int32)
    o = torch.empty((1, S, H, DV), device=dev, dtype=torch.bfloat16)
    lse = torch.empty((1, S, H), device=dev)
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    tr = torch.zeros(3 * 4 * 16 * 8, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def run():
        rc = lib.si_sparse_attn_fwd(q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), 1, S, H, D, NKV, K,
                                    DV, D ** -0.5, o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256, st)
        assert rc == 0, lib.si_last_error()

    for _ in range(3):
        run()
    lib.si_debug_set_attn_trace(tr.data_ptr())
    run()
    torch.cuda.synchronize()
    t = tr.view(3, 4, 16, 8).cpu()
    base = int(t[t > 0].min())
    for role, name in [(2, "softmax"), (1, "issuers"), (0, "gather")]:
        print(name)
        for tile in range(16):
            print(tile, [(int(x) - base) if x > 0 else -1 for x in t[role, 2, tile]])


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 16384)
