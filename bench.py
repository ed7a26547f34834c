"""StreamIndex-B200 benchmark: V4-Flash lightning indexer + top-k.

Workload (the headline point): B=1, S=1,048,576,
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
    ap.add_argument("--workload", default="indexer", choices=["indexer", "attn", "csa"],
                    help="indexer: the headline metric (default); attn: BASELINE configs[3] sparse attention")
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


# published single-H200 Triton times for this workload, ms
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
    from streamindex_b200.dist import balanced_bounds, broadcast_keys, gather_to_rank0, legal_pairs
    from streamindex_b200.indexer import IndexerTopk, chunked_indexer_topk

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    T = a.S // a.ratio
    bounds = balanced_bounds(a.S, world, T, a.ratio)
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


def run_attn(a):
    """sparse attention forward, B=1, S=65536, H=64, D=576/512, N_kv=16384, K=512."""
    from streamindex_b200 import _lib

    S, H, D, DV, NKV, K = a.S, a.attn_heads, 576, 512, 16384, a.attn_k
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(0)
    q = torch.randn((1, S, H, D), generator=g, device=device, dtype=torch.bfloat16).mul_(D ** -0.5)
    kv = torch.randn((1, NKV, D), generator=g, device=device, dtype=torch.bfloat16)
    sink = torch.zeros(H, dtype=torch.float32, device=device)
    idx = gen_attn_idx(S, K, NKV, 4, device)
    o = torch.empty((1, S, H, DV), dtype=torch.bfloat16, device=device)
    lse = torch.empty((1, S, H), dtype=torch.float32, device=device)
    ws = torch.empty(256, dtype=torch.uint8, device=device)
    lib = _lib.load()
    st = _lib.stream_handle(device)

    def step():
        _lib.check(lib.si_sparse_attn_fwd(q.data_ptr(), kv.data_ptr(), sink.data_ptr(), idx.data_ptr(), 1, S, H, D,
                                          NKV, K, DV, D ** -0.5, o.data_ptr(), lse.data_ptr(), ws.data_ptr(), 256, st))

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
    gather_bytes = V * D * 2
    uniq = q.numel() * 2 + o.numel() * 2 + idx.numel() * 4 + kv.numel() * 2 + lse.numel() * 4
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    tf_peak = peaks.get("bf16_tflops", 1590.0)
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    tf = flops / (ms * 1e-3) / 1e12
    # CPU oracle on a small sample of the same queries
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    n = 8
    pos = torch.linspace(0, S - 1, n).long()
    t = time.perf_counter()
    oracle.sparse_attn(q[:, pos.to(device)].cpu(), kv.cpu(), sink.cpu(), idx[:, pos.to(device)].cpu(), D ** -0.5,
                       d_v=DV)
    cpu_s = time.perf_counter() - t
    line = {
        "metric": "sparse attention forward (BASELINE configs[3]) Mqueries/s", "value": S / (ms * 1e-3) / 1e6,
        "unit": "Mqueries/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; causal uniform indices without replacement)",
        "config": {"workload": "sparse_attn_fwd B=1 S=%d H=%d D_qk=576 D_v=512 N_kv=16384 K=%d" % (S, H, K),
                   "valid_slots": V, "l2": "q/o larger than L2; kv (18.9 MB) L2-resident by design"},
        "gpu_launches": a.steps,
        "roofline": {"bound": "tensor", "achieved": tf, "peak": tf_peak, "unit": "TFLOP/s", "frac": tf / tf_peak,
                     "peak_source": "of measured (bf16_tflops burst, MEASURED_PEAKS.json)", "traffic": None,
                     "hbm_unique_gbs": uniq / (ms * 1e-3) / 1e9, "hbm_frac": uniq / (ms * 1e-3) / 1e9 / hbm_peak,
                     "gather_gbs_from_l2": gather_bytes / (ms * 1e-3) / 1e9},
        "cpu_baseline": {"value": n / cpu_s / 1e6, "unit": "Mqueries/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{n} queries, reference_sparse_attn restated (oracle), {cpu_s:.2f} s"},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_csa(a, world=1, rank=0, local=0):
    """CSA layer forward, B=2, S=131072, H=64, D=576/512, H_I=64, D_I=128, m=4, k=512, n_win=128.

    One step = mean-pool compressor (kv and indexer keys) -> fused indexer + top-k
    -> index build -> sparse attention.  With N GPUs the query range is
    S-sharded (work-balanced slices): rank 0 compresses and broadcasts the
    compressed kv / keys, every rank runs its slice (``csa_forward_slice``) and
    the outputs are gathered to rank 0."""
    from streamindex_b200.csa import csa_forward_slice, flash_csa_forward, mean_pool_compress
    from streamindex_b200.dist import balanced_bounds, broadcast_keys, gather_to_rank0

    B, S, H, D, DV, HI, DI, m, k, nwin = 2, a.S, 64, 576, 512, 64, 128, 4, 512, 128
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    x_kv = torch.randn((B, S, D), generator=g, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    x_k = torch.randn((B, S, DI), generator=g, device=dev, dtype=torch.bfloat16).mul_(DI ** -0.5)
    # attention work per query relative to one indexer key: (n_win + k) * H * (D + DV) vs H_I * D_I flops
    extra = (nwin + k) * H * (D + DV) / (HI * DI)
    bounds = balanced_bounds(S, world, S // m, m, align=128, extra_per_query=extra)
    lo, hi = bounds[rank], bounds[rank + 1]
    gq = torch.Generator(device=dev)
    gq.manual_seed(100 + rank)
    q = torch.randn((B, hi - lo, H, D), generator=gq, device=dev, dtype=torch.bfloat16).mul_(D ** -0.5)
    q_idx = torch.randn((B, hi - lo, HI, DI), generator=gq, device=dev, dtype=torch.bfloat16).mul_(DI ** -0.5)
    w = torch.randn((B, hi - lo, HI), generator=gq, device=dev, dtype=torch.float32)
    sink = torch.zeros(H, dtype=torch.float32, device=dev)
    kvc = torch.empty((B, S // m, D), dtype=torch.bfloat16, device=dev)
    kc = torch.empty((B, S // m, DI), dtype=torch.bfloat16, device=dev)
    full = torch.empty((B, S, H, DV), dtype=torch.bfloat16, device=dev) if (world > 1 and rank == 0) else None

    def step():
        if world == 1:
            kvc.copy_(mean_pool_compress(x_kv, m))
            kc.copy_(mean_pool_compress(x_k, m))
            return flash_csa_forward(q, x_kv, kvc, q_idx, kc, w, sink, n_win=nwin, top_k=k, m=m, d_v=DV)
        if rank == 0:
            kvc.copy_(mean_pool_compress(x_kv, m))
            kc.copy_(mean_pool_compress(x_k, m))
        broadcast_keys(kvc)
        broadcast_keys(kc)
        o = csa_forward_slice(q, x_kv, kvc, q_idx, kc, w, sink, s_offset=lo, n_win=nwin, top_k=k, m=m, d_v=DV)
        gather_to_rank0(o, bounds, full, dim=1)
        return o

    for _ in range(a.warmup):
        step()
    clocks = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier_sync(world)
    clocks.start()
    t0.record()
    for _ in range(a.steps):
        step()
    t1.record()
    _barrier_sync(world)
    clk = clocks.stop()
    ms = _max_over_ranks(t0.elapsed_time(t1) / a.steps, world, dev)
    if rank == 0:
        line = {
            "metric": "CSA layer forward (BASELINE configs[4]) Mqueries/s", "value": B * S / (ms * 1e-3) / 1e6,
            "unit": "Mqueries/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"flash_csa_forward B=2 S={S} H=64 D=576/512 H_I=64 D_I=128 m=4 top_k=512 n_win=128",
                       "path": "mean-pool x2 -> fused indexer+top-k -> index build -> split-kv sparse attention",
                       "parallelism": f"S-shard x{world} (compressed kv/keys broadcast, output gathered)"
                       if world > 1 else "single GPU"},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)


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
    if a.workload == "attn":
        if a.S == 1 << 20:
            a.S = 65536
        run_attn(a)
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
