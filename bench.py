"""StreamIndex-B200 benchmark: V4-Flash lightning indexer + top-k.

Workload (benchmark configs[1], the headline point): B=1, S=1,048,576,
H_I=64, D_I=128, m=4 (T=S/4), top_k=512, causal t < (s+1)//4; synthetic
inputs q, k ~ N(0,1)*D^-0.5 (bf16), w ~ N(0,1) (fp32), seeded, generated on
the device.  One step = one indexer+top-k pass over the whole query range.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--S S]

With N > 1 it runs under torchrun, one rank per GPU: the query range is cut
into work-balanced contiguous slices (``streamindex_b200.dist``), each step
broadcasts the keys from rank 0 (NCCL), runs the rank's slice and gathers
the indices and scores to rank 0.  Total work is fixed as N grows
("scaling": "strong").  Rank 0 prints one JSON line.

``--impl reference`` times the reference's materialise-then-topk algorithm
(the CPU oracle restatement of eval/test_v4_indexer_parity.py:111-137) on the
host cores, on a bounded sample of the same workload's queries.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "V4-Flash indexer+top-k ms & Mqueries/s at S=256K/1M, 1/2/4/8 B200; % TC peak"
UNIT = "Mqueries/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--S", type=int, default=1 << 20)
    ap.add_argument("--H", type=int, default=64)
    ap.add_argument("--D", type=int, default=128)
    ap.add_argument("--k", type=int, default=512)
    ap.add_argument("--ratio", type=int, default=4)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-queries", type=int, default=96)
    ap.add_argument("--no-gather", action="store_true")
    ap.add_argument("--attn-heads", type=int, default=64, help="attention workload: query heads (64; 128 = V4-Pro)")
    ap.add_argument("--attn-k", type=int, default=512, help="attention workload: selected kv rows per query")
    ap.add_argument("--attn-dv", type=int, default=512, help="attention workload: value width (576 = full D)")
    ap.add_argument("--attn-nkv", type=int, default=16384,
                    help="attention workload: kv rows (16384 = configs[3]; a power of two above it is a KV cache "
                         "larger than L2, indices spread over all rows)")
    ap.add_argument("--kv-fp8", action="store_true",
                    help="attention workload: kv stored as FP8 rows (e4m3 NoPE + fp32 block scales + bf16 RoPE)")
    ap.add_argument("--workload", default="indexer", choices=["indexer", "attn", "attn_bwd", "csa"],
                    help="indexer: the headline metric (default); attn: benchmark configs[3] sparse attention")
    return ap.parse_args()


def config(a, world):
    return {
        "workload": (f"V4-Flash indexer+top-k S={a.S} (configs[1])" if (a.H, a.k) == (64, 512)
                     else f"V4-Pro-dimension indexer+top-k S={a.S} H_I={a.H} top_k={a.k} (configs[2])"
                     if (a.H, a.k) == (128, 1024) else f"indexer+top-k S={a.S} H_I={a.H} top_k={a.k}"),
        "B": 1, "S": a.S, "H_I": a.H, "D_I": a.D, "T": a.S // a.ratio, "top_k": a.k, "causal_ratio": a.ratio,
        "chunk_s_chunk_t": "2048x8192 semantics (result is chunk-independent)",
        "parallelism": f"S-shard x{world}" if world > 1 else "single GPU",
        "l2": "inputs larger than L2 (q is S*H*D*2 bytes)",
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def gen_inputs(a, s_lo, s_hi, device, rank):
    """Seeded synthetic slice [s_lo, s_hi) of q / w plus the full keys (rank 0's copy is broadcast)."""
    T = a.S // a.ratio
    g = torch.Generator(device=device)
    g.manual_seed(1000 + rank)
    n = s_hi - s_lo
    q = torch.randn((1, n, a.H, a.D), generator=g, device=device, dtype=torch.bfloat16).mul_(a.D ** -0.5)
    w = torch.randn((1, n, a.H), generator=g, device=device, dtype=torch.float32)
    gk = torch.Generator(device=device)
    gk.manual_seed(0)
    k = torch.randn((1, T, a.D), generator=gk, device=device, dtype=torch.bfloat16).mul_(a.D ** -0.5)
    return q, k, w


def cpu_materialize_sample(a, q_rows, s_pos, k, w_rows, threads):
    """Reference materialise-then-topk (oracle port) on a sample of queries at global positions s_pos."""
    import oracle

    torch.set_num_threads(threads)
    T = k.shape[1]
    out = []
    step = 8
    for i in range(0, q_rows.shape[1], step):
        sc = oracle.lightning_indexer(q_rows[:, i:i + step], k, w_rows[:, i:i + step])
        lim = torch.clamp((s_pos[i:i + step] + 1) // a.ratio, max=T)
        illegal = torch.arange(T).unsqueeze(0) >= lim.unsqueeze(1)
        sc = sc.masked_fill(illegal.unsqueeze(0), float("-inf"))
        idx, vals = oracle.topk_desc_stable(sc, min(a.k, T))
        out.append(idx)
    return out


def cpu_sample_inputs(a, q, k, w, s_lo, n):
    """n queries evenly spread over the local slice (their global positions drive the mask)."""
    S_loc = q.shape[1]
    pos = torch.linspace(0, S_loc - 1, n).long()
    return (q[:, pos.to(q.device)].cpu(), (pos + s_lo), k.cpu(), w[:, pos.to(w.device)].cpu())


def time_cpu(a, qs, spos, kc, ws_, threads, reps=1):
    t0 = time.perf_counter()
    for _ in range(reps):
        cpu_materialize_sample(a, qs, spos, kc, ws_, threads)
    return (time.perf_counter() - t0) / reps


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(a, world, rank):
    """--impl reference: CPU materialise-then-topk on sampled queries of the same workload."""
    import oracle  # noqa: F401

    if rank != 0:
        return
    threads = os.cpu_count() or 1
    T = a.S // a.ratio
    g = torch.Generator().manual_seed(0)
    kc = (torch.randn((1, T, a.D), generator=g) * a.D ** -0.5).to(torch.bfloat16)
    n = max(8, a.cpu_queries // 4)
    pos = torch.linspace(0, a.S - 1, n).long()
    qs = (torch.randn((1, n, a.H, a.D), generator=g) * a.D ** -0.5).to(torch.bfloat16)
    ws_ = torch.randn((1, n, a.H), generator=g)
    for _ in range(a.warmup):
        cpu_materialize_sample(a, qs, pos, kc, ws_, threads)
    t = []
    for _ in range(a.steps):
        t.append(time_cpu(a, qs, pos, kc, ws_, threads))
    per_step = statistics.mean(t)
    value = n / per_step / 1e6
    sample = (f"{n} queries evenly spaced over S={a.S}, full T={T} keys each, materialise [n,H,T] fp32 + mask + "
              f"top-{a.k} (reference algorithm, oracle port); Mqueries/s = sampled queries / time")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config(a, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# published single-H200 Triton times for this workload (reference benchmarks/results/2026-04-27/scaling_v4_flash_indexer_final.log), ms
PUBLISHED_H200_MS = {32768: 30.8, 65536: 122.2, 131072: 484.7, 262144: 1935.3, 524288: 7730.1, 1048576: 30899.6}


def _max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier_sync(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def load_traffic():
    """Per-launch DRAM bytes of the fused kernel from the committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "indexer_topk_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


def run_ours(a, world, rank, local):
    from streamindex_b200.dist import (INDEXER_QUERY_COST_PAIRS, balanced_bounds, broadcast_keys, gather_to_rank0,
                                       legal_pairs)
    from streamindex_b200.indexer import IndexerTopk, chunked_indexer_topk

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    T = a.S // a.ratio
    bounds = balanced_bounds(a.S, world, T, a.ratio, extra_per_query=INDEXER_QUERY_COST_PAIRS * a.H / 64)
    s_lo, s_hi = bounds[rank], bounds[rank + 1]
    n_loc = s_hi - s_lo
    q, k, w = gen_inputs(a, s_lo, s_hi, device, rank)
    plan = IndexerTopk(1, n_loc, T, a.H, a.D, a.k, causal_ratio=a.ratio, s_offset=s_lo, device=device)
    full_idx = full_sc = None
    gather = world > 1 and not a.no_gather
    if gather and rank == 0:
        full_idx = torch.empty((1, a.S, a.k), dtype=torch.int64, device=device)
        full_sc = torch.empty((1, a.S, a.k), dtype=torch.float32, device=device)

    def step(ev=None):
        if world > 1:
            broadcast_keys(k)
        if ev is not None:
            ev[0].record()
        plan.run(q, k, w, sort=False)
        if ev is not None:
            ev[1].record()
        plan.sort()
        if ev is not None:
            ev[2].record()
        if gather:
            gather_to_rank0(plan.out_idx, bounds, full_idx)
            gather_to_rank0(plan.out_scores, bounds, full_sc)

    for _ in range(a.warmup):
        step()
    st = plan.status()
    if st != 0:
        raise RuntimeError(f"kernel status {st} after warm-up")

    clocks = ClockSampler(local)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(a.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier_sync(world)
    clocks.start()
    t0.record()
    for i in range(a.steps):
        step(evs[i])
    t1.record()
    _barrier_sync(world)
    clk = clocks.stop()
    ms_local = t0.elapsed_time(t1) / a.steps
    ms = _max_over_ranks(ms_local, world, device)
    k_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    s_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)

    flops = 2.0 * a.H * a.D * legal_pairs(a.S, T, a.ratio, s_lo, s_hi)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak_tf = peaks.get("bf16_tflops_sustained")
    peak_src = "of measured (bf16_tflops_sustained, MEASURED_PEAKS.json)"
    if not peak_tf:
        peak_tf, peak_src = 1400.0, "of fallback (1.4 PFLOP/s sustained)"
    achieved_tf = flops / (k_ms * 1e-3) / 1e12
    tr = load_traffic()
    traffic = None
    if tr and tr.get("bytes_per_query") and a.H == 64 and a.D == 128 and a.k == 512:
        traffic = tr["bytes_per_query"] * n_loc  # ncu capture scaled by queries per launch
    sort_bytes = n_loc * a.k * (8 + 8 + 4)
    sort_gbs = sort_bytes / (s_ms * 1e-3) / 1e9
    hbm_peak = peaks.get("hbm_gbs") or 6650.0

    # peak HBM of one public-API call, measured like the reference (max_memory_allocated delta)
    torch.cuda.synchronize()
    del plan
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats(device)
    base = torch.cuda.memory_allocated(device)
    if world == 1:
        oi, osc = chunked_indexer_topk(q, k, w, a.k, causal_ratio=a.ratio, chunk_s=2048, chunk_t=8192)
        torch.cuda.synchronize()
        peak_gb = (torch.cuda.max_memory_allocated(device) - base) / 1e9
        del oi, osc
    else:
        peak_gb = None

    line = None
    if rank == 0:
        value = a.S / (ms * 1e-3) / 1e6
        pub = PUBLISHED_H200_MS.get(a.S) if a.H == 64 and a.k == 512 and a.ratio == 4 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": (value / (a.S / (pub * 1e-3) / 1e6)) if pub else None,
            "vs_baseline_note": "published 1x H200 Triton chunked path" if pub else None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1)*D^-0.5 bf16 q/k, N(0,1) fp32 w, on device)",
            "config": config(a, world),
            "gpu_launches": 2 * a.steps,
            "kernels": {
                "indexer_topk_fused_ms": k_ms, "row_sort_ms": s_ms,
                "row_sort_gbs": sort_gbs, "row_sort_frac_hbm": sort_gbs / hbm_peak,
                "legal_pairs_rank0": legal_pairs(a.S, T, a.ratio, s_lo, s_hi),
            },
            "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved_tf / peak_tf, "peak_source": peak_src, "traffic": traffic,
                         "algorithmic": "2*H_I*D_I flops per causally legal (s,t) pair"},
            "peak_hbm_gb": peak_gb,
            "clocks": clk,
        }
    return line, (q, k, w, s_lo, device)


def run_e2e(a, world, rank, q, k, w, s_lo, device):
    """Same step through the C-ABI call with HOST (pinned) inputs and outputs; copies inside the timed region."""
    from streamindex_b200.indexer import IndexerTopk

    T = a.S // a.ratio
    n_loc = q.shape[1]
    hq = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    hk = torch.empty(k.shape, dtype=k.dtype, pin_memory=True)
    hw = torch.empty(w.shape, dtype=w.dtype, pin_memory=True)
    hq.copy_(q)
    hk.copy_(k)
    hw.copy_(w)
    plan = IndexerTopk(1, n_loc, T, a.H, a.D, a.k, causal_ratio=a.ratio, s_offset=s_lo, device=device)
    hi = torch.empty(plan.out_idx.shape, dtype=torch.int64, pin_memory=True)
    hs = torch.empty(plan.out_scores.shape, dtype=torch.float32, pin_memory=True)
    del q, k, w  # the host-buffer path owns its device staging buffers

    def step():
        plan.run_host(hq, hk, hw, hi, hs, chunks=16)

    step()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier_sync(world)
    t0.record()
    for _ in range(a.e2e_steps):
        step()
    t1.record()
    _barrier_sync(world)
    ms = _max_over_ranks(t0.elapsed_time(t1) / a.e2e_steps, world, device)
    h2d = hq.numel() * hq.element_size() + hk.numel() * hk.element_size() + hw.numel() * hw.element_size()
    d2h = hi.numel() * 8 + hs.numel() * 4
    if world > 1:
        t = torch.tensor([h2d, d2h], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        h2d, d2h = int(t[0].item()), int(t[1].item())
    return {"value": a.S / (ms * 1e-3) / 1e6, "unit": UNIT, "ms_per_step": ms, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": a.e2e_steps,
            "path": "IndexerTopk.run_host: pinned host q/k/w -> 16 query slices, H2D of slice c+1 and D2H of slice c-1 overlapped with the C-ABI kernel call on slice c; all copies inside the timed region"}


def run_cpu_baseline(a, q, k, w, s_lo):
    threads = os.cpu_count() or 1
    n = a.cpu_queries
    qs, spos, kc, ws_ = cpu_sample_inputs(a, q, k, w, s_lo, n)
    cpu_materialize_sample(a, qs[:, :8], spos[:8], kc, ws_[:, :8], threads)  # warm-up
    t = time_cpu(a, qs, spos, kc, ws_, threads)
    return {"value": n / t / 1e6, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"{n} queries evenly spaced over S={a.S} with their causal limits, full T={a.S // a.ratio} "
                       f"keys: materialise [n,H,T] fp32 einsum + ReLU*w + head-sum + mask + top-{a.k} "
                       f"(eval/test_v4_indexer_parity.py:111-137 restated), {t:.2f} s, torch threads={threads}")}


def gen_attn_idx(S, K, n_kv, ratio, device, seed=0, chunk=4096):
    """Per query, min(K, (s+1)//ratio) distinct indices drawn uniformly from [0, (s+1)//ratio), -1 padded."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = torch.full((1, S, K), -1, dtype=torch.int32, device=device)
    t = torch.arange(n_kv, device=device)
    for s0 in range(0, S, chunk):
        s1 = min(S, s0 + chunk)
        lim = torch.clamp((torch.arange(s0, s1, device=device) + 1) // ratio, max=n_kv)
        r = torch.rand((s1 - s0, n_kv), generator=g, device=device)
        r = r.masked_fill(t.unsqueeze(0) >= lim.unsqueeze(1), -1.0)
        v, i = r.topk(K, dim=-1)
        out[0, s0:s1] = torch.where(v >= 0, i, torch.full_like(i, -1)).to(torch.int32)
    return out


def gen_spread_idx(S, K, n_kv, device, seed=0):
    """K distinct rows per query spread over a power-of-two pool: (a_s + j * c_s) mod n_kv with a random
    offset a_s and a random odd stride c_s (odd strides are coprime with n_kv, so the K rows are distinct)."""
    assert n_kv & (n_kv - 1) == 0 and K <= n_kv
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    a0 = torch.randint(0, n_kv, (S, 1), generator=g, device=device)
    c = torch.randint(0, n_kv // 2, (S, 1), generator=g, device=device) * 2 + 1
    j = torch.arange(K, device=device).unsqueeze(0)
    return ((a0 + j * c) % n_kv).to(torch.int32).unsqueeze(0)


def run_attn(a):
    """benchmark configs[3]: sparse attention forward, B=1, S=65536, H=64, D=576/512, N_kv=16384, K=512."""
    from streamindex_b200 import _lib

    S, H, D, DV, NKV, K = a.S, a.attn_heads, 576, a.attn_dv, a.attn_nkv, a.attn_k
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=device, dtype=torch.bfloat16).mul_(D ** -0.5)
    kv = torch.randn((1, NKV, D), generator=g, device=device, dtype=torch.bfloat16)
    sink = torch.zeros(H, dtype=torch.float32, device=device)
    idx = gen_attn_idx(S, K, NKV, 4, device) if NKV == 16384 else gen_spread_idx(S, K, NKV, device)
    o = torch.empty((1, S, H, DV), dtype=torch.bfloat16, device=device)
    lse = torch.empty((1, S, H), dtype=torch.float32, device=device)
    ws = torch.empty(256, dtype=torch.uint8, device=device)
    lib = _lib.load()
    st = _lib.stream_handle(device)

    row_bytes = 2 * D
    if a.kv_fp8:
        from streamindex_b200.attention import quantize_kv_fp8

        kv_rows = quantize_kv_fp8(kv, 512)  # the KV cache as stored (quantised once, outside the timed region)
        row_bytes = kv_rows.shape[-1]

        def step():
            _lib.check(lib.si_sparse_attn_fwd_fp8kv(q.data_ptr(), kv_rows.data_ptr(), NKV, None, 0, 512,
                                                    sink.data_ptr(), idx.data_ptr(), 1, S, H, D, K, DV, D ** -0.5,
                                                    o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256, st))
    else:
        def step():
            _lib.check(lib.si_sparse_attn_fwd(q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), 1, S, H,
                                              D, NKV, K, DV, D ** -0.5, o.data_ptr(), lse.data_ptr(), ws.data_ptr(),
                                              256, st))

    for _ in range(a.warmup):
        step()
    assert _lib.read_status(ws, device) == 0
    clocks = ClockSampler(0)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    clocks.start()
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / a.steps
    V = int((idx >= 0).sum().item())
    flops = 2.0 * H * V * (D + DV)
    gather_bytes = V * row_bytes
    uniq = q.numel() * 2 + o.numel() * 2 + idx.numel() * 4 + kv.numel() * 2 + lse.numel() * 4
    peaks = _load_peaks()
    tf_peak = peaks.get("bf16_tflops") or 1590.0
    hbm_peak = peaks.get("hbm_gbs") or 6650.0
    attn_src = ("of measured (bf16_tflops burst, MEASURED_PEAKS.json)" if peaks.get("bf16_tflops")
                else "of fallback (1.59 PFLOP/s burst)")
    tf = flops / (ms * 1e-3) / 1e12
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "sparse_attn_traffic.json")) as f:
            tr = json.load(f)
        if (H, K, DV) == (tr["H"], tr["K"], tr["Dv"]) and not a.kv_fp8:
            traffic = tr["bytes_per_query"] * S  # ncu capture at S=4096 scaled by the queries of a launch
    except Exception:
        pass
    # CPU oracle on a small sample of the same queries
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    n = 2048
    pos = torch.linspace(0, S - 1, n).long()
    t = time.perf_counter()
    oracle.sparse_attn(q[:, pos.to(device)].cpu(), kv.cpu(), sink.cpu(), idx[:, pos.to(device)].cpu(), D ** -0.5,
                       d_v=DV)
    cpu_s = time.perf_counter() - t
    line = {
        "metric": "sparse attention forward (benchmark configs[3]) Mqueries/s", "value": S / (ms * 1e-3) / 1e6,
        "unit": "Mqueries/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; causal uniform indices without replacement)",
        "config": {"workload": "sparse_attn_fwd%s B=1 S=%d H=%d D_qk=576 D_v=%d N_kv=%d K=%d" % (
                       "_fp8kv" if a.kv_fp8 else "", S, H, DV, NKV, K),
                   "kv_row_bytes": row_bytes,
                   "valid_slots": V,
                   "l2": ("q/o larger than L2; kv (18.9 MB) L2-resident by design" if NKV == 16384 else
                          "q/o and kv (%.1f GB as stored) larger than L2; indices spread over all rows" % (
                              NKV * row_bytes / 1e9))},
        "gpu_launches": a.steps,
        "roofline": {"bound": "tensor", "achieved": tf, "peak": tf_peak, "unit": "TFLOP/s", "frac": tf / tf_peak,
                     "peak_source": attn_src, "traffic": traffic,
                     "hbm_unique_gbs": uniq / (ms * 1e-3) / 1e9, "hbm_frac": uniq / (ms * 1e-3) / 1e9 / hbm_peak,
                     "gather_gbs_from_l2": gather_bytes / (ms * 1e-3) / 1e9},
        "cpu_baseline": {"value": n / cpu_s / 1e6, "unit": "Mqueries/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{n} queries, reference_sparse_attn restated (oracle), {cpu_s:.2f} s"},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_attn_bwd(a):
    """Sparse attention backward at the benchmark config-4 shape (B=1, S=65536, H=64, D=576/512,
    N_kv=16384, K=512): one step = si_sparse_attn_bwd (dq, dkv, dsink) given the forward's o / lse."""
    from streamindex_b200 import _lib
    from streamindex_b200.attention import sparse_attn_fwd

    S, H, D, DV, NKV, K = a.S, a.attn_heads, 576, a.attn_dv, 16384, a.attn_k
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=device, dtype=torch.bfloat16).mul_(D ** -0.5)
    kv = torch.randn((1, NKV, D), generator=g, device=device, dtype=torch.bfloat16)
    sink = torch.zeros(H, dtype=torch.float32, device=device)
    idx = gen_attn_idx(S, K, NKV, 4, device)
    o, lse = sparse_attn_fwd(q, kv, sink, idx, d_v=DV)
    do = torch.randn(o.shape, generator=g, device=device, dtype=torch.bfloat16)
    dq = torch.zeros_like(q)
    dkv = torch.zeros((1, NKV, D), dtype=torch.float32, device=device)
    dsink = torch.zeros(H, dtype=torch.float32, device=device)
    lib = _lib.load()
    st = _lib.stream_handle(device)

    def step():
        dkv.zero_()
        dsink.zero_()
        _lib.check(lib.si_sparse_attn_bwd(q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), o.data_ptr(),
                                          lse.data_ptr(), do.data_ptr(), 1, S, H, D, NKV, K, DV, D ** -0.5,
                                          dq.data_ptr(), dkv.data_ptr(), dsink.data_ptr(), st))

    for _ in range(a.warmup):
        step()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / a.steps
    V = int((idx >= 0).sum().item())
    flops = 2.0 * H * V * (3 * D + 2 * DV)  # S, dO.V^T, dq, dkv (q and do parts)
    peaks = _load_peaks()
    tf_peak = peaks.get("bf16_tflops") or 1590.0
    bwd_src = ("of measured (bf16_tflops burst, tcgen05 cuBLAS)" if peaks.get("bf16_tflops")
               else "of fallback (1.59 PFLOP/s burst)")
    tf = flops / (ms * 1e-3) / 1e12
    print(json.dumps({
        "metric": "sparse attention backward (benchmark configs[3] shape) Mqueries/s", "value": S / (ms * 1e-3) / 1e6,
        "unit": "Mqueries/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"sparse_attn_bwd B=1 S={S} H={H} D=576 D_v={DV} N_kv=16384 K={K}",
                   "valid_slots": V},
        "gpu_launches": 3 * a.steps,
        "roofline": {"bound": "tensor", "achieved": tf, "peak": tf_peak, "unit": "TFLOP/s", "frac": tf / tf_peak,
                     "peak_source": bwd_src + "; this kernel uses the "
                                    "warp-level mma.sync path", "traffic": None},
    }), flush=True)


def _csa_slots(S, lo, hi, nwin, k, m):
    """Valid attention slots of queries [lo, hi): window min(n_win, s+1) + compressed min(k, (s+1)//m)."""
    import numpy as np

    s = np.arange(lo, hi, dtype=np.int64)
    return int(np.minimum(nwin, s + 1).sum() + np.minimum(k, np.minimum(S // m, (s + 1) // m)).sum())


def _load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def run_csa(a, world=1, rank=0, local=0):
    """benchmark configs[4]: CSA layer forward, B=2, S=131072, H=64, D=576/512, H_I=64, D_I=128, m=4, k=512, n_win=128.

    One step = mean-pool compressors (kv and indexer keys) -> fused indexer + top-k
    -> sparse attention with the window + compressed index list built in the
    kernel.  With N GPUs the query range is S-sharded (work-balanced slices):
    every rank holds the full x_kv / x_k, computes both compressors itself (no
    broadcast), runs its slice (``csa_forward_slice``) and keeps its attention
    output (the next layer consumes it sharded); the compressed top-k indices
    are gathered to rank 0 (NCCL point-to-point), the one exchange the
    north-star contract names.  Timed twice: with the index gather (the
    headline) and without it."""
    from streamindex_b200.attention import _csa_attn_call
    from streamindex_b200.csa import csa_forward_slice, flash_csa_forward, mean_pool_compress
    from streamindex_b200.dist import balanced_bounds, csa_query_cost_pairs, gather_to_rank0, legal_pairs
    from streamindex_b200.indexer import indexer_topk_slice

    B, S, H, D, DV, HI, DI, m, k, nwin = 2, a.S, 64, 576, 512, 64, 128, 4, 512, 128
    T = S // m
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    x_kv = torch.randn((B, S, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    x_k = torch.randn((B, S, DI), generator=g, device=dev, dtype=torch.bfloat16).mul_(DI ** -0.5)
    # per-query work beyond the indexer's key pairs (its own fixed cost and the attention), in pair units
    extra = csa_query_cost_pairs(H, D, DV, HI, DI, nwin, k)
    bounds = balanced_bounds(S, world, T, m, align=128, extra_per_query=extra)
    lo, hi = bounds[rank], bounds[rank + 1]
    gq = torch.Generator(device=dev)
    gq.manual_seed(100 + rank)
    q = torch.randn((B, hi - lo, H, D), generator=gq, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    q_idx = torch.randn((B, hi - lo, HI, DI), generator=gq, device=dev, dtype=torch.bfloat16).mul_(DI ** -0.5)
    w = torch.randn((B, hi - lo, HI), generator=gq, device=dev, dtype=torch.float32)
    sink = torch.zeros(H, dtype=torch.float32, device=dev)
    comp_full = torch.empty((B, S, k), dtype=torch.int64, device=dev) if (world > 1 and rank == 0) else None

    def step(gather):
        kvc = mean_pool_compress(x_kv, m)
        kc = mean_pool_compress(x_k, m)
        if world == 1:
            return flash_csa_forward(q, x_kv, kvc, q_idx, kc, w, sink, n_win=nwin, top_k=k, m=m, d_v=DV)
        o, comp = csa_forward_slice(q, x_kv, kvc, q_idx, kc, w, sink, s_offset=lo, n_win=nwin, top_k=k, m=m, d_v=DV,
                                    return_indices=True)
        if gather:
            gather_to_rank0(comp, bounds, comp_full, dim=1)
        return o

    def timed(gather, clocks=None):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _barrier_sync(world)
        if clocks:
            clocks.start()
        t0.record()
        for _ in range(a.steps):
            step(gather)
        t1.record()
        _barrier_sync(world)
        clk = clocks.stop() if clocks else None
        return _max_over_ranks(t0.elapsed_time(t1) / a.steps, world, dev), clk

    gather = world > 1 and not a.no_gather
    for _ in range(a.warmup):
        step(gather)
    ms, clk = timed(gather, ClockSampler(local))
    ms_nogather = timed(False)[0] if gather else ms

    # per-kernel split on this rank (same calls, events between them)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    kern = {"mean_pool_x2_ms": 0.0, "indexer_topk_ms": 0.0, "csa_attention_ms": 0.0}
    reps = max(1, min(a.steps, 5))
    for _ in range(reps):
        ev[0].record()
        kvc = mean_pool_compress(x_kv, m)
        kc = mean_pool_compress(x_k, m)
        ev[1].record()
        comp, _ = indexer_topk_slice(q_idx, kc, w, k, m, lo)
        ev[2].record()
        _csa_attn_call(q, x_kv, kvc, sink, comp, nwin, lo, D ** -0.5, DV)
        ev[3].record()
        torch.cuda.synchronize()
        kern["mean_pool_x2_ms"] += ev[0].elapsed_time(ev[1]) / reps
        kern["indexer_topk_ms"] += ev[1].elapsed_time(ev[2]) / reps
        kern["csa_attention_ms"] += ev[2].elapsed_time(ev[3]) / reps

    # algorithmic work of this rank's slice (rank 0 reports its own; all ranks are balanced)
    idx_flops = B * 2.0 * HI * DI * legal_pairs(S, T, m, lo, hi)
    att_flops = B * 2.0 * H * (D + DV) * _csa_slots(S, lo, hi, nwin, k, m)
    peaks = _load_peaks()
    tf_peak = peaks.get("bf16_tflops_sustained") or 1400.0
    src = ("of measured (bf16_tflops_sustained, MEASURED_PEAKS.json: the step repeats for seconds under the power cap)"
           if peaks.get("bf16_tflops_sustained") else "of fallback (1.4 PFLOP/s sustained)")
    step_local_ms = kern["mean_pool_x2_ms"] + kern["indexer_topk_ms"] + kern["csa_attention_ms"]
    achieved = (idx_flops + att_flops) / (step_local_ms * 1e-3) / 1e12

    peak_gb = None
    if world == 1:
        del comp, kvc, kc
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        base = torch.cuda.memory_allocated(dev)
        o = step(False)
        torch.cuda.synchronize()
        peak_gb = (torch.cuda.max_memory_allocated(dev) - base) / 1e9
        del o

    e2e = None if (a.no_e2e or world > 1) else run_csa_e2e(a, q, q_idx, w, x_kv, x_k, sink, dev)
    cpu = None if (a.no_cpu or world > 1 or rank != 0) else run_csa_cpu(q, q_idx, w, x_kv, x_k, sink, m, nwin, k)
    if rank == 0:
        line = {
            "metric": "CSA layer forward (benchmark configs[4]) Mqueries/s", "value": B * S / (ms * 1e-3) / 1e6,
            "unit": "Mqueries/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "ms_per_step_no_gather": ms_nogather, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1)*D^-0.5 bf16 activations, N(0,1) fp32 head weights, on device)",
            "config": {"workload": f"flash_csa_forward B=2 S={S} H=64 D=576/512 H_I=64 D_I=128 m=4 top_k=512 n_win=128",
                       "path": "mean-pool x2 -> fused indexer+top-k -> sparse attention with the index list built "
                               "in the kernel (window + compressed picks)",
                       "parallelism": (f"S-shard x{world}: compressors on every rank, output kept sharded, "
                                       f"compressed top-k indices gathered to rank 0"
                                       + (" (gather off)" if a.no_gather else "")) if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (q is 19 GB)"},
            "gpu_launches": 5 * a.steps,
            "kernels": kern,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": achieved / tf_peak, "peak_source": src, "traffic": None,
                         "algorithmic": "indexer 2*H_I*D_I per legal (s,t) pair + attention 2*H*(D+D_v) per valid "
                                        "slot, over the step's summed kernel times on rank 0",
                         "indexer_tflops": idx_flops / (kern["indexer_topk_ms"] * 1e-3) / 1e12,
                         "attention_tflops": att_flops / (kern["csa_attention_ms"] * 1e-3) / 1e12},
            "peak_hbm_gb": peak_gb,
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def run_csa_e2e(a, q, q_idx, w, x_kv, x_k, sink, dev, chunk=8192):
    """CSA step through the public API with HOST (pinned) inputs and output.

    Each step copies x_kv / x_k to the device, compresses them, then walks the
    query range in chunks of one batch row: H2D of chunk c+1 (copy stream) and
    D2H of chunk c-1's output (second copy stream) overlap the layer forward of
    chunk c (``csa_forward_slice`` with the chunk's global offset)."""
    from streamindex_b200.csa import csa_forward_slice, mean_pool_compress

    B, S, H, D = q.shape
    DV, m, k, nwin = 512, 4, 512, 128
    pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t)  # noqa: E731
    hq, hqi, hw, hkv, hk = pin(q), pin(q_idx), pin(w), pin(x_kv), pin(x_k)
    ho = torch.empty((B, S, H, DV), dtype=torch.bfloat16, pin_memory=True)
    del q, q_idx, w
    torch.cuda.empty_cache()
    cs = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    chunks = [(b, s0, min(S, s0 + chunk)) for b in range(B) for s0 in range(0, S, chunk)]
    kvd = torch.empty_like(x_kv)
    kd = torch.empty_like(x_k)

    def one():
        kvd.copy_(hkv, non_blocking=True)
        kd.copy_(hk, non_blocking=True)
        kvc, kc = mean_pool_compress(kvd, m), mean_pool_compress(kd, m)
        staged = {}

        def stage(i):
            b, s0, s1 = chunks[i]
            with torch.cuda.stream(up):
                t = (hq[b:b + 1, s0:s1].to(dev, non_blocking=True), hqi[b:b + 1, s0:s1].to(dev, non_blocking=True),
                     hw[b:b + 1, s0:s1].to(dev, non_blocking=True))
                e = torch.cuda.Event()
                e.record(up)
            staged[i] = (t, e)

        stage(0)
        for i, (b, s0, s1) in enumerate(chunks):
            if i + 1 < len(chunks):
                stage(i + 1)
            (tq, tqi, tw), e = staged.pop(i)
            cs.wait_event(e)
            for t in (tq, tqi, tw):
                t.record_stream(cs)
            o = csa_forward_slice(tq, kvd[b:b + 1], kvc[b:b + 1], tqi, kc[b:b + 1], tw, sink, s_offset=s0,
                                  n_win=nwin, top_k=k, m=m, d_v=DV)
            down.wait_stream(cs)
            with torch.cuda.stream(down):
                ho[b:b + 1, s0:s1].copy_(o, non_blocking=True)
            o.record_stream(down)
        cs.wait_stream(down)

    one()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(a.e2e_steps):
        one()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / a.e2e_steps
    h2d = sum(t.numel() * t.element_size() for t in (hq, hqi, hw, hkv, hk))
    d2h = ho.numel() * ho.element_size()
    return {"value": B * S / (ms * 1e-3) / 1e6, "unit": "Mqueries/s", "ms_per_step": ms,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": a.e2e_steps,
            "path": f"pinned host inputs -> x_kv/x_k H2D + mean-pool, then {len(chunks)} query chunks: H2D of "
                    "chunk c+1 and D2H of chunk c-1's output overlapped with csa_forward_slice on chunk c"}


def run_csa_cpu(q, q_idx, w, x_kv, x_k, sink, m, nwin, k, n=384):
    """The reference's CSA forward (oracle restatement of flash_sparse/csa.py:86-207) on n sampled queries of
    batch 0: compressors over the whole sequence, materialised indexer scores over all compressed keys, mask,
    top-k, window + compressed index list, sparse attention."""
    import oracle
    from oracle.csa import compressed_to_global

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    S = q.shape[1]
    D = q.shape[-1]
    pos = torch.linspace(0, S - 1, n).long()
    qs, qis, ws_ = (t[0:1, pos.to(t.device)].cpu() for t in (q, q_idx, w))
    xkv, xk = x_kv[0:1].cpu(), x_k[0:1].cpu()
    t = time.perf_counter()
    kvc = oracle.mean_pool_compress(xkv, m)
    kc = oracle.mean_pool_compress(xk, m)
    T = kc.shape[1]
    sc = oracle.lightning_indexer(qis, kc, ws_)
    lim = torch.clamp((pos + 1) // m, max=T)
    sc = sc.masked_fill((torch.arange(T).view(1, -1) >= lim.view(-1, 1)).unsqueeze(0), float("-inf"))
    ti, tv = oracle.topk_desc_stable(sc, min(k, T))
    ti = torch.where(torch.isinf(tv), torch.full_like(ti, -1), ti)
    win = (pos.view(-1, 1) - nwin + 1 + torch.arange(nwin).view(1, -1))
    win = torch.where(win >= 0, win, torch.full_like(win, -1)).unsqueeze(0)
    idx = torch.cat([win, compressed_to_global(ti, S)], dim=-1).int()
    oracle.sparse_attn(qs, torch.cat([xkv, kvc], dim=1), sink.cpu(), idx, D ** -0.5, d_v=512)
    dt = time.perf_counter() - t
    return {"value": n / dt / 1e6, "unit": "Mqueries/s", "cores": threads, "kind": "port",
            "sample": f"{n} queries of batch 0 evenly spaced over S={S}: oracle compressors + materialised indexer "
                      f"over all {T} compressed keys + mask + top-{k} + window/compressed list + sparse attention, "
                      f"{dt:.2f} s, torch threads={threads}"}


def main():
    a = parse()
    if a.workload == "csa":
        if a.S == 1 << 20:
            a.S = 131072
        world, rank, local = init_dist()
        run_csa(a, world, rank, local)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if a.workload in ("attn", "attn_bwd"):
        if a.S == 1 << 20:
            a.S = 65536
        run_attn(a) if a.workload == "attn" else run_attn_bwd(a)
        return
    if a.impl == "reference":
        # CPU-only arm: rank 0 alone measures on the host cores; other ranks exit
        # at once (no process group, so nothing spins beside the measurement)
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(a, world, rank)
        return
    world, rank, local = init_dist()
    line, (q, k, w, s_lo, device) = run_ours(a, world, rank, local)
    e2e = None if a.no_e2e else run_e2e(a, world, rank, q, k, w, s_lo, device)
    if rank == 0:
        line["e2e"] = e2e
        if world == 1 and not a.no_cpu:
            line["cpu_baseline"] = run_cpu_baseline(a, q, k, w, s_lo)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
