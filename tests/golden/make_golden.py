"""Generate golden fixtures by running the reference's own Python functions.

Run where a checkout of the reference exists, naming it by argument or by
``$STREAMINDEX_REF``::

    python tests/golden/make_golden.py <path-to-reference-checkout>

The shipped reference drops the empty call parentheses of some method calls
(``q.dim != 4``, ``qk.relu_``, ``(x).exp``, ``c_a.dim != 3``).  Rather than
editing its source, the inputs are wrapped in a ``torch.Tensor`` subclass
whose ``dim`` / ``relu_`` / ``exp`` attributes evaluate eagerly and return
objects that are also callable (calling them returns themselves), so the
reference's own lines run unchanged with their intended meaning.  Functions
whose bodies were moved into dead branches are called with arguments that
reach the live branch (``softmax_scale=None`` for ``reference_sparse_attn``;
``n_compressed < top_k`` for ``build_csa_topk_idxs``).

Outputs are written next to this script as ``*.pt``; the tests read only
those files (the reference is never read at test time).
"""

from __future__ import annotations

import importlib.util
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class _CallableInt(int):
    def __call__(self):
        return int(self)


class Fixed(torch.Tensor):
    """Tensor whose dropped-parenthesis attributes behave as the calls they meant."""

    def __call__(self):
        return self

    @property
    def dim(self):  # type: ignore[override]
        return _CallableInt(torch.Tensor.dim(self))

    @property
    def relu_(self):  # type: ignore[override]
        torch.Tensor.relu_(self)
        return self

    @property
    def exp(self):  # type: ignore[override]
        return torch.Tensor.exp(self)

    @property
    def abs(self):  # type: ignore[override]
        return torch.Tensor.abs(self)


def fx(t: torch.Tensor) -> torch.Tensor:
    return t.as_subclass(Fixed)


def plain(t):
    return t.as_subclass(torch.Tensor) if isinstance(t, torch.Tensor) else t


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STREAMINDEX_REF")
    if not REF or not os.path.isdir(REF):
        raise SystemExit("usage: make_golden.py <reference checkout> (or set $STREAMINDEX_REF)")
    sys.path.insert(0, REF)
    from flash_sparse import reference as R  # noqa: E402
    from flash_sparse import csa as C  # noqa: E402

    parity = _load("ref_parity", os.path.join(REF, "eval", "test_v4_indexer_parity.py"))
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.inputs import indexer_inputs, attn_inputs  # noqa: E402

    out = {}

    # 1. lightning indexer + materialise-then-topk with post-mask (V4 dims, small S)
    cases = [
        ("idx_v4", dict(B=1, S=128, H=64, D=128, T=32), 16, 4, 0),
        ("idx_unaligned", dict(B=1, S=47, H=16, D=32, T=73), 16, 1, 901),
        ("idx_b2", dict(B=2, S=96, H=32, D=64, T=24), 8, 4, 7),
    ]
    for name, shp, top_k, ratio, seed in cases:
        q, k, w = indexer_inputs(shp["B"], shp["S"], shp["H"], shp["D"], shp["T"], seed=seed)
        scores = plain(R.reference_lightning_indexer(fx(q), fx(k), fx(w)))
        idx = plain(parity._materialize_topk(fx(q), fx(k), fx(w), top_k, ratio))
        out[name] = dict(q=q, k=k, w=w, top_k=top_k, ratio=ratio, scores=scores.float(), topk_idx=idx.long())

    # 2. sparse attention with sink, MLA-style D=576 (value = first 512 dims) and D=128
    for name, shp, seed in [
        ("attn_576", dict(B=1, S=24, H=16, D=576, N=64, K=32), 3),
        ("attn_128", dict(B=2, S=16, H=8, D=128, N=40, K=16), 4),
    ]:
        q, kv, sink, idx = attn_inputs(shp["B"], shp["S"], shp["H"], shp["D"], shp["N"], shp["K"], ratio=1, seed=seed)
        # one all-masked query and a masked slot pattern as in the reference tests
        idx[0, 0] = -1
        idx[:, :, 3::4] = -1
        o = plain(R.reference_sparse_attn(fx(q.float()), fx(kv.float()), fx(sink), fx(idx), softmax_scale=None))
        out[name] = dict(q=q, kv=kv, sink=sink, idx=idx, o=o.float())

    # 3. compressor (non-overlap, zero scores/bias == mean pool), window and CSA index build
    g = torch.Generator("cpu").manual_seed(11)
    x = torch.randn((2, 30, 16), generator=g)
    comp = plain(R.reference_token_compressor(fx(x), fx(torch.zeros_like(x)), fx(torch.zeros(4, 16)), 4, overlap=False))
    out["compress"] = dict(x=x, m=4, out=comp)
    out["window"] = dict(B=2, S=20, n_win=6, idx=plain(R._build_sliding_window_idxs(2, 20, 6, "cpu")))
    sc = torch.randn((1, 40, 10), generator=g)
    built = plain(C.build_csa_topk_idxs(sc, 8, 16, seq_len=40, n_compressed=10, m=4, device="cpu"))
    out["csa_idx"] = dict(scores=sc, n_win=8, top_k=16, m=4, idx=built)

    # 4. HCA forward (flash_sparse/reference.py:411-452): window + all legal compressed blocks
    g2 = torch.Generator("cpu").manual_seed(13)
    Bh, Sh, Hh, Dh, mp, nw = 1, 40, 8, 64, 8, 6
    qh = (torch.randn((Bh, Sh, Hh, Dh), generator=g2) * Dh ** -0.5).bfloat16()
    kvh = torch.randn((Bh, Sh, Dh), generator=g2).bfloat16()
    kvc = torch.randn((Bh, Sh // mp, Dh), generator=g2).bfloat16()
    sinkh = torch.randn(Hh, generator=g2)
    oh = plain(R.reference_hca_forward(fx(qh.float()), fx(kvh.float()), fx(kvc.float()), fx(sinkh), nw, m_prime=mp))
    out["hca"] = dict(q=qh, kv=kvh, kv_c=kvc, sink=sinkh, n_win=nw, m_prime=mp, o=oh.float())

    # 5. general softmax-gated compressor, non-overlapping mode (the overlapping
    #    mode's body is unreachable in the shipped reference)
    g3 = torch.Generator("cpu").manual_seed(19)
    cx = torch.randn((2, 37, 24), generator=g3)
    zx = torch.randn((2, 37, 24), generator=g3)
    bx = torch.randn((8, 24), generator=g3)
    comp8 = plain(R.reference_token_compressor(fx(cx), fx(zx), fx(bx), 8, overlap=False))
    out["compress_gated"] = dict(c=cx, z=zx, b=bx, m=8, out=comp8)

    # 6. FP8 KV quant-dequant of the NoPE dims, block 64 (flash_sparse/utils/quantization.py:19-36)
    Q = _load("ref_quant", os.path.join(REF, "flash_sparse", "utils", "quantization.py"))
    g4 = torch.Generator("cpu").manual_seed(23)
    kvq = torch.randn((2, 24, 576), generator=g4)
    kvq[0, :4] *= 40.0            # large rows
    kvq[1, :3, :64] *= 1e-6       # a block below the 1e-4 amax floor
    kvq[1, 5] = 0.0               # an all-zero row
    kvq = kvq.bfloat16()
    deq = plain(Q.act_quant_simulate(fx(kvq[..., :512].contiguous()), block_size=64))
    out["kv_fp8"] = dict(kv=kvq, n_nope=512, block=64, deq=deq)

    # 7. gradients of the reference's sparse attention (autograd through
    #    reference_sparse_attn itself): the backward's ground truth
    #    (the reference's Triton backward needs a GPU and a power-of-2 D)
    for name, shp, dv, seed in [("attn_bwd_576", dict(B=1, S=12, H=16, D=576, N=48, K=32), 512, 29),
                                ("attn_bwd_128", dict(B=2, S=10, H=20, D=128, N=40, K=24), 128, 31)]:
        q, kv, sink, idx = attn_inputs(shp["B"], shp["S"], shp["H"], shp["D"], shp["N"], shp["K"], ratio=1, seed=seed)
        idx[0, 0] = -1
        idx[:, :, 5::7] = -1
        gdo = torch.Generator("cpu").manual_seed(seed + 1)
        do = torch.randn((shp["B"], shp["S"], shp["H"], dv), generator=gdo).bfloat16()
        qf = q.float().requires_grad_(True)
        kvf = kv.float().requires_grad_(True)
        sf = sink.clone().requires_grad_(True)
        o = R.reference_sparse_attn(fx(qf), fx(kvf), fx(sf), fx(idx), softmax_scale=None)
        o = plain(o)[..., :dv]
        (o * do.float()).sum().backward()
        out[name] = dict(q=q, kv=kv, sink=sink, idx=idx, do=do, d_v=dv, o=o.detach().float(),
                         dq=qf.grad.detach(), dkv=kvf.grad.detach(), dsink=sf.grad.detach())

    only = os.environ.get("GOLDEN_ONLY")
    for name, d in out.items():
        if only and name not in only.split(","):
            continue
        torch.save(d, os.path.join(HERE, f"{name}.pt"))
        print("wrote", name)


if __name__ == "__main__":
    main()
