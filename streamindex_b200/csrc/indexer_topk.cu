// Fused indexer score + streaming top-k kernel, row-sort kernel and launchers.
// Design notes are in indexer_topk.cuh.
#include <cstdio>
#include <mutex>
#include <cuda_bf16.h>

#include "indexer_topk.cuh"

namespace si {

// ------------------------------------------------------------------ scheduling
// Query blocks are visited in decreasing causal work (the last block of a
// batch has the most legal keys) and dealt to CTAs in a zig-zag, so a static
// schedule is balanced without an atomic work counter.
__device__ __forceinline__ void block_coords(const IndexerParams& p, int i, int& b, int& blk) {
  const int r = i / p.B;
  b = i - r * p.B;
  blk = p.nblk_per_batch - 1 - r;
}

__device__ __forceinline__ int block_index(int round, int cta, int grid) {
  return round * grid + ((round & 1) ? (grid - 1 - cta) : cta);
}

// Number of legal keys of query s (mode-dependent upper bound on t).
__device__ __forceinline__ int key_limit(const IndexerParams& p, int s) {
  if (s >= p.S) return 0;
  if (p.ratio > 0) {
    const long long l = ((long long)s + p.s_offset + 1) / p.ratio;
    return l < p.T ? (int)l : p.T;
  }
  return p.T;
}

__device__ __forceinline__ int block_key_tiles(const IndexerParams& p, int QC, int blk) {
  const int s_last = min(p.S, (blk + 1) * QC) - 1;
  return ceil_div(key_limit(p, s_last), kKeysPerTile);
}

// ------------------------------------------------------------------ warp radix select
__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, m);
  hi = __shfl_xor_sync(0xffffffffu, hi, m);
  return ((unsigned long long)hi << 32) | lo;
}

// Loads of the candidate buffer are issued kSelBatch at a time per lane
// (independent loads, one latency per batch) — the buffer lives in global
// memory (L1/L2 resident) and a dependent load per iteration would make every
// pass latency-bound.
constexpr int kSelBatch = 8;

template <typename F>
__device__ __forceinline__ void for_each_key(const unsigned long long* buf, int n, uint32_t lane, F&& f) {
  for (int base = 0; base < n; base += 32 * kSelBatch) {
    unsigned long long k[kSelBatch];
#pragma unroll
    for (int u = 0; u < kSelBatch; ++u) {
      const int i = base + u * 32 + (int)lane;
      k[u] = i < n ? buf[i] : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kSelBatch; ++u) {
      const int i = base + u * 32 + (int)lane;
      if (i < n) f(k[u]);
    }
  }
}

// One warp: keep the `ksel` largest of the n (> ksel) distinct keys in buf,
// compacted to buf[0, ksel), and return the smallest kept key.  hist is a
// 256-entry shared scratch owned by this warp.
#ifdef SI_IDX_TRACE
__device__ unsigned long long* g_sel_trace = nullptr;  // [event < 4096][point < 8]
__device__ unsigned int g_sel_count = 0;
#define SEL_T(pt) do { if (tslot >= 0 && lane == 0) g_sel_trace[tslot * 8 + (pt)] = globaltimer(); } while (0)
#else
#define SEL_T(pt) do { } while (0)
#endif
__device__ unsigned long long warp_select_topk(unsigned long long* buf, int n, int ksel, uint32_t* hist) {
  const uint32_t lane = lane_id();
#ifdef SI_IDX_TRACE
  int tslot = -1;
  if (g_sel_trace && blockIdx.x == 0) {
    if (lane == 0) tslot = (int)atomicAdd(&g_sel_count, 1u);
    tslot = __shfl_sync(0xffffffffu, tslot, 0);
    if (tslot >= 4096) tslot = -1;
    if (tslot >= 0 && lane == 0) g_sel_trace[tslot * 8 + 7] = (unsigned long long)n;
  }
#endif
  SEL_T(0);
  unsigned long long a = ~0ull, o = 0ull;
  for_each_key(buf, n, lane, [&](unsigned long long k) {
    a &= k;
    o |= k;
  });
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    a &= shfl_xor_u64(a, m);
    o |= shfl_xor_u64(o, m);
  }
  SEL_T(1);
  const unsigned long long diff = a ^ o;  // nonzero: keys are distinct and n >= 2
  const int hb = 63 - __clzll((long long)diff);
  unsigned long long mask = (hb == 63) ? 0ull : ~((2ull << hb) - 1ull);
  unsigned long long prefix = a & mask;
  int need = ksel;
  int shift = hb >= 7 ? hb - 7 : 0;
  while (true) {
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
    __syncwarp();
    for_each_key(buf, n, lane, [&](unsigned long long k) {
      if ((k & mask) == prefix) atomicAdd(&hist[(uint32_t)(k >> shift) & 255u], 1u);
    });
    __syncwarp();
    uint32_t c[8];
    uint32_t local = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[lane * 8 + j];
      local += c[j];
    }
    // inclusive suffix sum over lanes (lane 31 holds the highest digits)
    uint32_t suf = local;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
      const uint32_t v = __shfl_down_sync(0xffffffffu, suf, m);
      if (lane + m < 32) suf += v;
    }
    const uint32_t above_lane = suf - local;  // count in higher lanes
    // the crossing lane: above_lane < need <= suf
    const bool mine = above_lane < (uint32_t)need && (uint32_t)need <= suf;
    int digit = 0;
    uint32_t above = above_lane, eq = 0;
    if (mine) {
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        if (above + c[j] >= (uint32_t)need) {
          digit = (int)lane * 8 + j;
          eq = c[j];
          break;
        }
        above += c[j];
      }
    }
    const uint32_t who = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
    digit = __shfl_sync(0xffffffffu, digit, who);
    above = __shfl_sync(0xffffffffu, above, who);
    eq = __shfl_sync(0xffffffffu, eq, who);
    need -= (int)above;
    prefix |= (unsigned long long)digit << shift;
    mask |= 0xFFull << shift;
    __syncwarp();
    if ((int)eq == need || shift == 0) break;
    shift = shift >= 8 ? shift - 8 : 0;
#ifdef SI_IDX_TRACE
    if (tslot >= 0 && lane == 0) g_sel_trace[tslot * 8 + 6] += 1;  // extra passes
#endif
  }
  SEL_T(2);
  // keys >= prefix are exactly the top ksel; compact in place (never writes
  // ahead of the batch being read: all loads of a batch precede its stores)
  const unsigned long long theta = prefix;
  int out = 0;
  unsigned long long kmin = ~0ull;
  const uint32_t lt = (1u << lane) - 1u;
  for (int base = 0; base < n; base += 32 * kSelBatch) {
    unsigned long long k[kSelBatch];
#pragma unroll
    for (int u = 0; u < kSelBatch; ++u) {
      const int i = base + u * 32 + (int)lane;
      k[u] = i < n ? buf[i] : 0ull;
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < kSelBatch; ++u) {
      const int i = base + u * 32 + (int)lane;
      const bool sel = i < n && k[u] >= theta;
      const uint32_t bal = __ballot_sync(0xffffffffu, sel);
      if (sel) {
        buf[out + __popc(bal & lt)] = k[u];
        kmin = k[u] < kmin ? k[u] : kmin;
      }
      out += __popc(bal);
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const unsigned long long v = shfl_xor_u64(kmin, m);
    kmin = v < kmin ? v : kmin;
  }
  __syncwarp();
  SEL_T(3);
  return kmin;
}

}  // namespace si

namespace si {

struct __align__(16) IndexerSmemMisc {
  uint64_t k_full[4], k_empty[4];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t q_full, q_empty;
  unsigned long long thr[kMaxQC];
  int cnt[kMaxQC];
  int lim[kMaxQC];
  uint32_t tmem_base;
  int abort_flag;
  alignas(16) float w[kQRows];
  uint32_t hist[kEpiWarps][256];
  unsigned long long xch[4][16];  // per-slice exchange words of the cooperative select
};

__host__ __device__ inline int indexer_stages(int D) { return D <= 64 ? 4 : 2; }
__host__ __device__ inline size_t indexer_smem_bytes(int D) {
  const int na = D / 64;
  return 1024 /*alignment slack*/ + (size_t)na * kQRows * 128 + (size_t)indexer_stages(D) * na * kKeysPerTile * 128 +
         sizeof(IndexerSmemMisc);
}

// Packed fp32 helpers (sm_100 fma.rn.f32x2 on a 64-bit register pair).
__device__ __forceinline__ unsigned long long relu2(float x, float y) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(fmaxf(x, 0.f)), "f"(fmaxf(y, 0.f)));
  return r;
}
__device__ __forceinline__ void ffma2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float sum2(unsigned long long v) {
  float x, y;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(v));
  return x + y;
}

// Cooperative exact top-k select by the 4 warps (128 threads) of one epilogue
// slice, used when the candidate buffer fits in registers (n <= 128 * E).
// One coalesced read of the buffer into registers, radix passes (8-bit
// digits over the 64-bit key, starting below the keys' common prefix) with
// per-warp shared histograms, and an in-place compaction from registers.
// hist4: the slice's 4 warp histograms (4 x 256 words); xch: 16 words of
// exchange space; bar: the slice's named barrier id.  Returns the smallest
// kept key.  All 128 threads must call it with the same arguments.
template <int E>
__device__ unsigned long long slice_select_topk(unsigned long long* buf, int n, int ksel, uint32_t* hist4,
                                                unsigned long long* xch, int wi, uint32_t bar) {
  const uint32_t lane = lane_id();
  const int tid = wi * 32 + (int)lane;
  unsigned long long k[E];
  unsigned long long a = ~0ull, o = 0ull;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 128 + tid;
    k[e] = i < n ? buf[i] : 0ull;
    if (i < n) {
      a &= k[e];
      o |= k[e];
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    a &= shfl_xor_u64(a, m);
    o |= shfl_xor_u64(o, m);
  }
  if (lane == 0) {
    xch[wi] = a;
    xch[4 + wi] = o;
  }
  named_bar(bar, 128);
  a = xch[0] & xch[1] & xch[2] & xch[3];
  o = xch[4] | xch[5] | xch[6] | xch[7];
  const unsigned long long diff = a ^ o;
  const int hb = 63 - __clzll((long long)diff);
  unsigned long long mask = (hb == 63) ? 0ull : ~((2ull << hb) - 1ull);
  unsigned long long prefix = a & mask;
  int need = ksel;
  int shift = hb >= 7 ? hb - 7 : 0;
  uint32_t* myh = hist4 + wi * 256;
  while (true) {
#pragma unroll
    for (int j = 0; j < 8; ++j) myh[lane * 8 + j] = 0;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = e * 128 + tid;
      if (i < n && (k[e] & mask) == prefix) atomicAdd(&myh[(uint32_t)(k[e] >> shift) & 255u], 1u);
    }
    named_bar(bar, 128);  // histograms complete (and the previous round's xch reads done)
    if (wi == 0) {
      uint32_t c[8];
      uint32_t local = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane * 8 + j;
        c[j] = hist4[d] + hist4[256 + d] + hist4[512 + d] + hist4[768 + d];
        local += c[j];
      }
      uint32_t suf = local;
#pragma unroll
      for (int m = 1; m < 32; m <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, suf, m);
        if (lane + m < 32) suf += v;
      }
      const uint32_t above_lane = suf - local;
      const bool mine = above_lane < (uint32_t)need && (uint32_t)need <= suf;
      if (mine) {
        uint32_t above = above_lane;
#pragma unroll
        for (int j = 7; j >= 0; --j) {
          if (above + c[j] >= (uint32_t)need) {
            xch[8] = (unsigned long long)(lane * 8 + j);
            xch[9] = above;
            xch[10] = c[j];
            break;
          }
          above += c[j];
        }
      }
    }
    named_bar(bar, 128);  // digit published
    const int digit = (int)xch[8];
    const int above = (int)xch[9];
    const int eq = (int)xch[10];
    need -= above;
    prefix |= (unsigned long long)digit << shift;
    mask |= 0xFFull << shift;
    if (eq == need || shift == 0) break;
    shift = shift >= 8 ? shift - 8 : 0;
  }
  // compaction: keys >= prefix are exactly the top ksel
  const unsigned long long theta = prefix;
  int cnt = 0;
  unsigned long long kmin = ~0ull;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 128 + tid;
    if (i < n && k[e] >= theta) {
      ++cnt;
      kmin = k[e] < kmin ? k[e] : kmin;
    }
  }
  int incl = cnt;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, m);
    if ((int)lane >= m) incl += v;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const unsigned long long v = shfl_xor_u64(kmin, m);
    kmin = v < kmin ? v : kmin;
  }
  named_bar(bar, 128);  // everyone has read xch[8..10]
  if (lane == 31) xch[wi] = (unsigned long long)incl;
  if (lane == 0) xch[4 + wi] = kmin;
  named_bar(bar, 128);
  int base = 0;
  for (int w = 0; w < wi; ++w) base += (int)xch[w];
  int pos = base + incl - cnt;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = e * 128 + tid;
    if (i < n && k[e] >= theta) buf[pos++] = k[e];
  }
  unsigned long long m0 = xch[4], m1 = xch[5], m2 = xch[6], m3 = xch[7];
  kmin = m0 < m1 ? m0 : m1;
  kmin = m2 < kmin ? m2 : kmin;
  kmin = m3 < kmin ? m3 : kmin;
  named_bar(bar, 128);  // compaction stores done, xch free
  return kmin;
}

// ------------------------------------------------------------------ epilogue
// Warps 2..9.  Per (key tile, group): TMEM -> fp32 scores (ReLU, w, sum over
// heads in-thread), release the accumulator, then feed the streaming top-k.
template <int H, int MODE>
// wst: element strides of w over (b, s, h) (x, y, z); passed beside the
// parameter struct rather than in it (a larger IndexerParams measurably
// changed the kernel's register allocation: more spills, ~3% slower)
__device__ __forceinline__ void indexer_epilogue(const IndexerParams& p, IndexerSmemMisc* ms, uint32_t tmem,
                                                 int warp, uint32_t lane, int nrounds, int nblocks, int grid,
                                                 int4 wst) {
  constexpr int QC = kQRows / H;
  constexpr int QG = kGroupCols / H;
  constexpr int NQH = EpiCfg<H>::NQW;      // queries per epilogue warp
  constexpr int CW = EpiCfg<H>::CW;        // columns per epilogue warp
  constexpr int NW = EpiCfg<H>::WARPS;
  const int e = warp - 2;
  const int qd = warp & 3;  // TMEM lane quadrant this warp may access
  const int hf = e >> 2;    // column slice of each group
  const int etid = e * 32 + (int)lane;
  const uint32_t lt = (1u << lane) - 1u;
  volatile int* abort_flag = &ms->abort_flag;
  volatile int* vcnt = ms->cnt;
  volatile unsigned long long* vthr = ms->thr;
  uint32_t* hist = ms->hist[e];
  uint32_t* hist4 = ms->hist[4 * hf];       // the slice's four warp histograms
  unsigned long long* xch = ms->xch[hf];
  // exact top-ksel of query j's buffer (n > ksel keys), compacted in place;
  // returns the new threshold.  Called uniformly by the slice's 4 warps.
  auto select = [&](int jj, unsigned long long* buf, int n) -> unsigned long long {
    constexpr int SR = (H == 128) ? 20 : kSelRegs;  // H_I = 128 runs 8 epilogue warps with a larger register budget
    if (n <= 128 * SR) return slice_select_topk<SR>(buf, n, p.ksel, hist4, xch, qd, 1 + hf);
    unsigned long long th = 0ull;
    if ((jj & 3) == qd) th = warp_select_topk(buf, n, p.ksel, hist);
    if (lane == 0 && (jj & 3) == qd) xch[15] = th;
    named_bar(1 + hf, 128);
    th = xch[15];
    named_bar(1 + hf, 128);
    return th;
  };
  unsigned long long* cand_cta = p.cand + (size_t)blockIdx.x * QC * p.cap;
  uint32_t aph[2] = {0, 0};
  unsigned long long thr_reg[2][NQH];  // per group: this warp's cached thresholds (change only at sync points)

  for (int r = 0; r < nrounds; ++r) {
    const int i = block_index(r, blockIdx.x, grid);
    if (i >= nblocks) continue;
    int b, blk;
    block_coords(p, i, b, blk);
    const int s0 = blk * QC;
    const int ntiles = (MODE == kModeTopk) ? block_key_tiles(p, QC, blk) : ceil_div(p.T, kKeysPerTile);

    named_bar(7, 32 * NW);  // the previous block is done with w / lim / thr / cnt
    for (int x = etid; x < QC * H; x += 32 * NW) {
      const int s = s0 + x / H;
      float wv = 0.f;
      if (s < p.S) {
        const int off = b * wst.x + s * wst.y + (x % H) * wst.z;
        wv = p.w_is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.w)[off])
                         : reinterpret_cast<const float*>(p.w)[off];
      }
      ms->w[x] = wv;
    }
    if (etid < QC) {
      ms->lim[etid] = key_limit(p, s0 + etid);
      ms->thr[etid] = 0ull;
      ms->cnt[etid] = 0;
    }
    named_bar(7, 32 * NW);
#pragma unroll
    for (int g = 0; g < 2; ++g)
#pragma unroll
      for (int jj = 0; jj < NQH; ++jj) thr_reg[g][jj] = 0ull;

    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const int tkey = t * kKeysPerTile + qd * 32 + (int)lane;
      for (int g = 0; g < 2; ++g) {
        if (warp == 2 && lane == 0) SI_ITRACE(2, r, t, 4 * g + 0);
        if (!mbar_wait(&ms->acc_full[g], aph[g], abort_flag, p.status, kErrWaitAccFull)) {
          ok = false;
          break;
        }
        if (warp == 2 && lane == 0) SI_ITRACE(2, r, t, 4 * g + 1);
        aph[g] ^= 1;
        tc_fence_after();
        // acc2[jj] holds two partial sums (even / odd heads) updated with the
        // packed fp32 FMA (fma.rn.f32x2): ReLU is one fmax per element, the
        // weight multiply-add half an instruction per element.
        // Four independent packed accumulators per query (by head index mod 8)
        // keep the FMA dependency chains short.
        unsigned long long acc2[NQH][4];
#pragma unroll
        for (int jj = 0; jj < NQH; ++jj)
#pragma unroll
          for (int u = 0; u < 4; ++u) acc2[jj][u] = 0ull;
        const uint32_t tbase = tmem + ((uint32_t)(qd * 32) << 16) + g * kGroupCols + hf * CW;
        const float* wrow = ms->w + g * kGroupCols + hf * CW;
#pragma unroll
        for (int c = 0; c < CW / 64; ++c) {
          float v0[32], v1[32];
          tmem_ld32x2_sync(tbase + c * 64, tbase + c * 64 + 32, v0, v1);
#pragma unroll
          for (int h4 = 0; h4 < 8; ++h4) {
            const ulonglong2 wa = reinterpret_cast<const ulonglong2*>(wrow + c * 64)[h4];
            const ulonglong2 wb = reinterpret_cast<const ulonglong2*>(wrow + c * 64 + 32)[h4];
            const int ca = c * 64 + h4 * 4, cb = c * 64 + 32 + h4 * 4;
            ffma2(acc2[ca / H][(h4 & 1) * 2 + 0], relu2(v0[h4 * 4 + 0], v0[h4 * 4 + 1]), wa.x);
            ffma2(acc2[ca / H][(h4 & 1) * 2 + 1], relu2(v0[h4 * 4 + 2], v0[h4 * 4 + 3]), wa.y);
            ffma2(acc2[cb / H][(h4 & 1) * 2 + 0], relu2(v1[h4 * 4 + 0], v1[h4 * 4 + 1]), wb.x);
            ffma2(acc2[cb / H][(h4 & 1) * 2 + 1], relu2(v1[h4 * 4 + 2], v1[h4 * 4 + 3]), wb.y);
          }
        }
        float acc[NQH];
#pragma unroll
        for (int jj = 0; jj < NQH; ++jj)
          acc[jj] = (sum2(acc2[jj][0]) + sum2(acc2[jj][1])) + (sum2(acc2[jj][2]) + sum2(acc2[jj][3]));
        tc_fence_before();
        __syncwarp();
        // The accumulator's TMEM reads completed in tcgen05.wait::ld; a relaxed
        // arrive keeps the release from waiting on this warp's candidate
        // stores of the previous group.
        if (lane == 0) mbar_arrive_relaxed(&ms->acc_empty[g]);
        if (warp == 2 && lane == 0) SI_ITRACE(2, r, t, 4 * g + 2);

        if (MODE == kModeScore) {
#pragma unroll
          for (int jj = 0; jj < NQH; ++jj) {
            const int s = s0 + g * QG + hf * NQH + jj;
            if (s < p.S && tkey < p.T) p.out_scores[((size_t)b * p.S + s) * p.T + tkey] = acc[jj];
          }
          continue;
        }

        // ---- streaming top-k.  Every kSyncTiles tiles the half's four warps
        // meet: a query whose buffer could not absorb kSyncTiles more tiles of
        // inserts is flushed by the slice (cooperative register select), and
        // thresholds are re-read.
        // In between, inserts only need the cached threshold and an atomic.
        if (t % kSyncTiles == 0) {
          named_bar(1 + hf, 128);
          const int room = p.cap - kSyncTiles * kKeysPerTile;
          bool any = false;
#pragma unroll
          for (int jj = 0; jj < NQH; ++jj) any |= vcnt[g * QG + hf * NQH + jj] > room;
          if (any) {
#pragma unroll
            for (int jj = 0; jj < NQH; ++jj) {
              const int j = g * QG + hf * NQH + jj;
              const int n = vcnt[j];
              if (n > room) {
                const unsigned long long th = select(jj, cand_cta + (size_t)j * p.cap, n);
                if (qd == 0 && lane == 0) {
                  vthr[j] = th;
                  vcnt[j] = p.ksel;
                }
              }
            }
          }
          // Every warp of the slice has read the counts before any of them
          // inserts this tile's keys: a count raised by an early insert would
          // otherwise send only some of the warps into the (barrier-using)
          // flush.
          named_bar(1 + hf, 128);
#pragma unroll
          for (int jj = 0; jj < NQH; ++jj) thr_reg[g][jj] = vthr[g * QG + hf * NQH + jj];
        }
#pragma unroll
        for (int jj = 0; jj < NQH; ++jj) {
          const int j = g * QG + hf * NQH + jj;
          bool legal = tkey < ms->lim[j];
          if (MODE == kModeTopkMask && legal)
            legal = p.mask[((size_t)b * p.S + (s0 + j)) * p.T + tkey] != 0;
          const unsigned long long key = make_key(acc[jj], tkey);
          const bool pass = legal && key > thr_reg[g][jj];
          const uint32_t bal = __ballot_sync(0xffffffffu, pass);
          if (bal) {
            const int leader = __ffs(bal) - 1;
            int base = 0;
            if ((int)lane == leader) base = atomicAdd(&ms->cnt[j], __popc(bal));
            base = __shfl_sync(0xffffffffu, base, leader);
            if (pass) cand_cta[(size_t)j * p.cap + base + __popc(bal & lt)] = key;
          }
        }
        if (warp == 2 && lane == 0) SI_ITRACE(2, r, t, 4 * g + 3);
      }
    }
    if (!ok) break;

    if (MODE != kModeScore) {
      // ---- final selection and (unsorted) key write-out for this block's queries
      named_bar(1 + hf, 128);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int jj = 0; jj < NQH; ++jj) {
          const int j = g * QG + hf * NQH + jj;
          const int s = s0 + j;
          if (s >= p.S) continue;  // uniform across the slice
          unsigned long long* buf = cand_cta + (size_t)j * p.cap;
          int n = vcnt[j];
          if (n > p.ksel) {
            select(jj, buf, n);
            n = p.ksel;
          }
          unsigned long long* dst = p.out_keys + ((size_t)b * p.S + s) * p.ksel;
          const int tid = qd * 32 + (int)lane;
          for (int x = tid; x < p.ksel; x += 128) dst[x] = x < n ? buf[x] : 0ull;
        }
      }
    }
  }
}

template <int H, int MODE>
__global__ void __launch_bounds__(EpiCfg<H>::THREADS, 1)
    indexer_topk_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        IndexerParams p, uint32_t idesc, int4 wst, int2 nd) {
  constexpr int QC = kQRows / H;         // queries per block
  constexpr int QG = kGroupCols / H;     // queries per group
  static_assert(EpiCfg<H>::NQW >= 1 && QC <= kMaxQC, "unsupported head count");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NA = p.D / 64;
  const int NST = indexer_stages(p.D);
  uint8_t* sQ = smem;                                    // [NA][512 rows][128 B]
  uint8_t* sK = smem + (size_t)NA * kQRows * 128;        // [NST][NA][128 rows][128 B]
  IndexerSmemMisc* ms = reinterpret_cast<IndexerSmemMisc*>(sK + (size_t)NST * NA * kKeysPerTile * 128);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const int grid = gridDim.x;
  const int nblocks = p.B * p.nblk_per_batch;
  const int nrounds = ceil_div(nblocks, grid);
  volatile int* abort_flag = &ms->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      mbar_init(&ms->k_full[i], 1);
      mbar_init(&ms->k_empty[i], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&ms->acc_full[g], 1);
      mbar_init(&ms->acc_empty[g], EpiCfg<H>::WARPS);
    }
    mbar_init(&ms->q_full, 1);
    mbar_init(&ms->q_empty, 1);
    ms->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_k);
  }
  if (warp == 1) {
    tmem_alloc(&ms->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ms->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t st = 0, kph = 0, qph = 0;
      const uint32_t qbytes = (uint32_t)NA * kQRows * 128;
      const uint32_t kbytes = (uint32_t)NA * kKeysPerTile * 128;
      for (int r = 0; r < nrounds; ++r) {
        const int i = block_index(r, blockIdx.x, grid);
        if (i >= nblocks) continue;
        int b, blk;
        block_coords(p, i, b, blk);
        const int ntiles = (MODE == kModeTopk) ? block_key_tiles(p, QC, blk) : ceil_div(p.T, kKeysPerTile);
        if (ntiles == 0) continue;
        if (!mbar_wait(&ms->q_empty, qph ^ 1, abort_flag, p.status, kErrWaitQ)) break;
        qph ^= 1;
        mbar_expect_tx(&ms->q_full, qbytes);
        // 256 (query, head) rows per box: 256/H queries x all H heads
        for (int a = 0; a < NA; ++a)
          for (int hh = 0; hh < 2; ++hh) {
            uint8_t* dq = sQ + (size_t)a * kQRows * 128 + hh * 256 * 128;
            if (nd.x)
              tma_load_4d(dq, &map_q, &ms->q_full, a * 64, 0, blk * QC + hh * (256 / H), b);
            else
              tma_load_2d(dq, &map_q, &ms->q_full, a * 64, (b * p.S + blk * QC) * H + hh * 256);
          }
        bool ok = true;
        for (int t = 0; t < ntiles; ++t) {
          SI_ITRACE(0, r, t, 0);
          if (!mbar_wait(&ms->k_empty[st], kph ^ 1, abort_flag, p.status, kErrWaitTmaEmpty)) {
            ok = false;
            break;
          }
          SI_ITRACE(0, r, t, 1);
          mbar_expect_tx(&ms->k_full[st], kbytes);
          uint8_t* dst = sK + (size_t)st * NA * kKeysPerTile * 128;
          for (int a = 0; a < NA; ++a) {
            if (nd.y)
              tma_load_3d(dst + (size_t)a * kKeysPerTile * 128, &map_k, &ms->k_full[st], a * 64, t * kKeysPerTile,
                          b);
            else
              tma_load_2d(dst + (size_t)a * kKeysPerTile * 128, &map_k, &ms->k_full[st], a * 64,
                          b * p.T + t * kKeysPerTile);
          }
          if (++st == (uint32_t)NST) {
            st = 0;
            kph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      uint32_t st = 0, kph = 0, qph = 0;
      uint32_t aph[2] = {0, 0};
      for (int r = 0; r < nrounds; ++r) {
        const int i = block_index(r, blockIdx.x, grid);
        if (i >= nblocks) continue;
        int b, blk;
        block_coords(p, i, b, blk);
        const int ntiles = (MODE == kModeTopk) ? block_key_tiles(p, QC, blk) : ceil_div(p.T, kKeysPerTile);
        if (ntiles == 0) continue;
        if (!mbar_wait(&ms->q_full, qph, abort_flag, p.status, kErrWaitQ)) break;
        qph ^= 1;
        tc_fence_after();
        bool ok = true;
        for (int t = 0; t < ntiles && ok; ++t) {
          SI_ITRACE(1, r, t, 0);
          if (!mbar_wait(&ms->k_full[st], kph, abort_flag, p.status, kErrWaitTmaFull)) {
            ok = false;
            break;
          }
          SI_ITRACE(1, r, t, 1);
          tc_fence_after();
          const uint32_t kbase = smem_u32(sK + (size_t)st * NA * kKeysPerTile * 128);
          for (int g = 0; g < 2; ++g) {
            if (!mbar_wait(&ms->acc_empty[g], aph[g] ^ 1, abort_flag, p.status, kErrWaitAccEmpty)) {
              ok = false;
              break;
            }
            aph[g] ^= 1;
            SI_ITRACE(1, r, t, 2 + g);
            tc_fence_after();
            const uint32_t qbase = smem_u32(sQ) + g * kGroupCols * 128;
            const uint32_t d_tmem = tmem + g * kGroupCols;
            for (int a = 0; a < NA; ++a) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t adesc = umma_desc_sw128(kbase + a * kKeysPerTile * 128 + kk * 32);
                const uint64_t bdesc = umma_desc_sw128(qbase + a * kQRows * 128 + kk * 32);
                umma_f16(d_tmem, adesc, bdesc, idesc, (a | kk) != 0);
              }
            }
            umma_commit(&ms->acc_full[g]);
          }
          umma_commit(&ms->k_empty[st]);
          if (++st == (uint32_t)NST) {
            st = 0;
            kph ^= 1;
          }
        }
        umma_commit(&ms->q_empty);
        if (!ok) break;
      }
    }
  } else {
    indexer_epilogue<H, MODE>(p, ms, tmem, warp, lane, nrounds, nblocks, grid, wst);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace si

namespace si {

// ------------------------------------------------------------------ row sort
// One warp per row: read ksel 64-bit keys (0 = empty slot), bitonic-sort them
// descending in registers (E keys per lane, element i = r*32 + lane), and
// decode into idx (int64, -1 for empty) and score (fp32, -inf for empty)
// in place of the keys.
template <int E>
__global__ void __launch_bounds__(256) topk_row_sort_kernel(unsigned long long* keys_io, float* scores_out,
                                                            long long rows, int ksel) {
  constexpr int P = E * 32;
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  unsigned long long* kr = keys_io + row * ksel;
  unsigned long long v[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < ksel ? kr[i] : 0ull;
  }
#pragma unroll
  for (int size = 2; size <= P; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j >= 1; j >>= 1) {
      if (j >= 32) {
        const int rj = j / 32;
#pragma unroll
        for (int r = 0; r < E; ++r) {
          if ((r & rj) == 0) {
            const int r2 = r | rj;
            const bool desc = (((r * 32 + lane) & size) == 0);
            const unsigned long long a = v[r], c = v[r2];
            const bool sw = desc ? (a < c) : (a > c);
            v[r] = sw ? c : a;
            v[r2] = sw ? a : c;
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < E; ++r) {
          const unsigned long long o = shfl_xor_u64(v[r], j);
          const int i = r * 32 + lane;
          const bool desc = ((i & size) == 0);
          const bool lower = (lane & j) == 0;
          const bool take_max = (lower == desc);
          v[r] = take_max ? (o > v[r] ? o : v[r]) : (o < v[r] ? o : v[r]);
        }
      }
    }
  }
  long long* ir = reinterpret_cast<long long*>(kr);
  float* sr = scores_out + row * ksel;
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const int i = r * 32 + lane;
    if (i < ksel) {
      const unsigned long long k = v[r];
      ir[i] = k ? (long long)(0xFFFFFFFFu - (uint32_t)k) : -1ll;
      sr[i] = k ? unord_f32((uint32_t)(k >> 32)) : -INFINITY;
    }
  }
}

}  // namespace si

// ==================================================================== host side
#include "capi_common.h"
#include "../../include/streamindex_b200.h"

namespace si {

static int pick_cap(int ksel) { return ((2 * ksel + kSyncTiles * kKeysPerTile + 31) / 32) * 32; }

static int indexer_grid(int nblocks) {
  const int sms = device_sm_count();
  return nblocks < sms ? nblocks : sms;
}

size_t indexer_ws_bytes(int B, int S, int H, int ksel) {
  const int QC = kQRows / H;
  const int nblocks = B * ceil_div(S, QC);
  const int grid = indexer_grid(nblocks > 0 ? nblocks : 1);
  return kStatusBytes + (size_t)grid * QC * pick_cap(ksel) * sizeof(unsigned long long);
}

template <int H, int MODE>
static cudaError_t launch_indexer_t(const CUtensorMap& mq, const CUtensorMap& mk, const IndexerParams& p, int grid,
                                    uint32_t idesc, int4 wst, int2 nd, cudaStream_t stream) {
  const size_t smem = indexer_smem_bytes(p.D);
  static unsigned long long configured = 0;  // devices on which the attribute is set
  cudaError_t e = set_smem_attr_once(reinterpret_cast<const void*>(indexer_topk_kernel<H, MODE>),
                                     (int)indexer_smem_bytes(128), &configured);
  if (e != cudaSuccess) return e;
  indexer_topk_kernel<H, MODE><<<grid, EpiCfg<H>::THREADS, smem, stream>>>(mq, mk, p, idesc, wst, nd);
  return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_indexer_h(const CUtensorMap& mq, const CUtensorMap& mk, const IndexerParams& p, int grid,
                                    uint32_t idesc, int4 wst, int2 nd, cudaStream_t stream) {
  switch (p.H) {
    case 16: return launch_indexer_t<16, MODE>(mq, mk, p, grid, idesc, wst, nd, stream);
    case 32: return launch_indexer_t<32, MODE>(mq, mk, p, grid, idesc, wst, nd, stream);
    case 64: return launch_indexer_t<64, MODE>(mq, mk, p, grid, idesc, wst, nd, stream);
    case 128: return launch_indexer_t<128, MODE>(mq, mk, p, grid, idesc, wst, nd, stream);
    default: return cudaErrorInvalidValue;
  }
}

static cudaError_t launch_row_sort(unsigned long long* keys, float* scores, long long rows, int ksel,
                                   cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  int p = 32;
  while (p < ksel) p <<= 1;
  switch (p / 32) {
    case 1: topk_row_sort_kernel<1><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 2: topk_row_sort_kernel<2><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 4: topk_row_sort_kernel<4><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 8: topk_row_sort_kernel<8><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 16: topk_row_sort_kernel<16><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 32: topk_row_sort_kernel<32><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    case 64: topk_row_sort_kernel<64><<<grid, 256, 0, stream>>>(keys, scores, rows, ksel); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Shared argument checks for the indexer entry points.
static int check_indexer_args(const void* q, const void* k, const void* w, int B, int S, int T, int H, int D) {
  if (!q || !k || !w) return fail("indexer: null input pointer");
  if (B < 1 || S < 0 || T < 0) return fail("indexer: bad B/S/T (B=%d S=%d T=%d)", B, S, T);
  if (H != 16 && H != 32 && H != 64 && H != 128) return fail("indexer: H_I must be 16, 32, 64 or 128 (got %d)", H);
  if (D < 8 || D > 128 || D % 8) return fail("indexer: D_I must be a multiple of 8 in [8,128] (got %d)", D);
  if (((uintptr_t)q | (uintptr_t)k) & 15) return fail("indexer: q and k must be 16-byte aligned");
  if ((long long)B * S * H + 1024 >= (1ll << 31) || (long long)B * T + 256 >= (1ll << 31))
    return fail("indexer: B*S*H or B*T exceeds the 2^31 TMA coordinate range");
  return 0;
}

#ifdef SI_IDX_TRACE
static unsigned long long* g_idx_trace = nullptr;
}  // namespace si
extern "C" SI_API void si_debug_set_idx_trace(unsigned long long* t) { si::g_idx_trace = t; }
extern "C" SI_API void si_debug_set_sel_trace(unsigned long long* t) {
  cudaMemcpyToSymbol(si::g_sel_trace, &t, sizeof(t));
  unsigned int z = 0;
  cudaMemcpyToSymbol(si::g_sel_count, &z, sizeof(z));
}
namespace si {
#endif

// Element strides of the indexer inputs (last dim contiguous).  Negative
// entries mean "contiguous" for that tensor.
struct IndexerStrides {
  long long q_b = -1, q_s = -1, q_h = -1, k_b = -1, k_t = -1, w_b = -1, w_s = -1, w_h = -1;
};

static int run_indexer(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                       int H, int D, int ksel, int ratio, const uint8_t* mask, int mode, int64_t* out_idx,
                       float* out_scores, void* ws, size_t ws_bytes, cudaStream_t stream, long long s_offset = 0,
                       unsigned flags = 0, IndexerStrides str = IndexerStrides()) {
  if (int rc = check_indexer_args(q, k, w, B, S, T, H, D)) return rc;
  if (str.q_h < 0) { str.q_h = D; str.q_s = (long long)H * D; str.q_b = (long long)S * H * D; }
  if (str.k_t < 0) { str.k_t = D; str.k_b = (long long)T * D; }
  if (str.w_h < 0) { str.w_h = 1; str.w_s = H; str.w_b = (long long)S * H; }
  if (s_offset < 0) return fail("indexer: negative s_offset");
  if (!ws) return fail("indexer: null workspace");
  const size_t need = mode == kModeScore ? kStatusBytes : indexer_ws_bytes(B, S, H, ksel);
  if (ws_bytes < need) return fail("indexer: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream)) return fail_cuda("indexer: status reset", e);
  const long long rows = (long long)B * S;
  if (rows == 0) return 0;
  if (mode != kModeScore && T == 0) {
    // no keys: every slot is padding
    return launch_fill_pad(out_idx, out_scores, rows * ksel, stream);
  }
  if (mode == kModeScore && T == 0) return 0;

  const int Dp = ((D + 63) / 64) * 64;
  CUtensorMap mq, mk;
  const int dt = ab_fp16 ? 1 : 0;
  // Evenly spaced rows (the contiguous layout, or padded rows) use a 2-D
  // [rows, D] map with the row pitch: measured ~3% faster at S=1M than the
  // 3-D key-tile map.  Other strides use 4-D / 3-D maps.
  const bool q_rows = str.q_s == (long long)H * str.q_h && str.q_b == (long long)S * str.q_s;
  const bool k_rows = str.k_b == (long long)T * str.k_t;
  if (q_rows) {
    const uint64_t qd[2] = {(uint64_t)D, (uint64_t)B * S * H};
    const uint64_t qs[1] = {(uint64_t)str.q_h * 2};
    const uint32_t qb[2] = {64, 256};
    if (int rc = make_tmap_nd_16b(&mq, q, 2, qd, qs, qb, dt)) return rc;
  } else {
    const uint64_t qd[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)S, (uint64_t)B};
    const uint64_t qs[3] = {(uint64_t)str.q_h * 2, (uint64_t)str.q_s * 2, (uint64_t)str.q_b * 2};
    const uint32_t qb[4] = {64, (uint32_t)H, (uint32_t)(256 / H), 1};
    if (int rc = make_tmap_nd_16b(&mq, q, 4, qd, qs, qb, dt)) return rc;
  }
  if (k_rows) {
    const uint64_t kd[2] = {(uint64_t)D, (uint64_t)B * T};
    const uint64_t ks[1] = {(uint64_t)str.k_t * 2};
    const uint32_t kb[2] = {64, (uint32_t)kKeysPerTile};
    if (int rc = make_tmap_nd_16b(&mk, k, 2, kd, ks, kb, dt)) return rc;
  } else {
    const uint64_t kd[3] = {(uint64_t)D, (uint64_t)T, (uint64_t)B};
    const uint64_t ks[2] = {(uint64_t)str.k_t * 2, (uint64_t)str.k_b * 2};
    const uint32_t kb[3] = {64, (uint32_t)kKeysPerTile, 1};
    if (int rc = make_tmap_nd_16b(&mk, k, 3, kd, ks, kb, dt)) return rc;
  }

  IndexerParams p{};
  p.B = B; p.S = S; p.T = T; p.H = H; p.D = Dp;
  p.ratio = ratio > 0 ? ratio : 0;
  p.ksel = ksel;
  p.cap = pick_cap(ksel > 0 ? ksel : 1);
  p.w_is_bf16 = w_is_bf16;
  p.w = w;
  p.mask = mask;
  p.out_keys = reinterpret_cast<unsigned long long*>(out_idx);
  p.out_scores = out_scores;
  p.cand = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(ws) + kStatusBytes);
  p.status = status;
  const int QC = kQRows / H;
  p.nblk_per_batch = ceil_div(S, QC);
  p.s_offset = s_offset;
  const int2 nd = make_int2(q_rows ? 0 : 1, k_rows ? 0 : 1);
  if ((long long)(B - 1) * str.w_b + (long long)(S - 1) * str.w_s + (long long)(H - 1) * str.w_h >= (1ll << 31))
    return fail("indexer: w strides address beyond 2^31 elements");
  const int4 wst = make_int4((int)str.w_b, (int)str.w_s, (int)str.w_h, 0);
#ifdef SI_IDX_TRACE
  p.trace = g_idx_trace;
#endif
  const int grid = indexer_grid(B * p.nblk_per_batch);
  const uint32_t idesc = umma_idesc_f16(kKeysPerTile, kGroupCols, ab_fp16 ? 0 : 1);
  cudaError_t e;
  if (mode == kModeTopk) e = launch_indexer_h<kModeTopk>(mq, mk, p, grid, idesc, wst, nd, stream);
  else if (mode == kModeTopkMask) e = launch_indexer_h<kModeTopkMask>(mq, mk, p, grid, idesc, wst, nd, stream);
  else e = launch_indexer_h<kModeScore>(mq, mk, p, grid, idesc, wst, nd, stream);
  if (e != cudaSuccess) return fail_cuda("indexer: kernel launch", e);
  if (mode != kModeScore && !(flags & SI_FLAG_SKIP_SORT)) {
    e = launch_row_sort(p.out_keys, out_scores, rows, ksel, stream);
    if (e != cudaSuccess) return fail_cuda("indexer: row-sort launch", e);
  }
  return 0;
}

}  // namespace si

extern "C" {

size_t si_indexer_topk_ws_bytes(int B, int S, int T, int H, int D, int top_k) {
  (void)T;
  (void)D;
  if (H != 16 && H != 32 && H != 64 && H != 128) H = 16;
  if (B < 1) B = 1;
  if (S < 1) S = 1;
  return si::indexer_ws_bytes(B, S, H, top_k > 0 ? top_k : 1);
}

int si_indexer_topk(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                    int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask, int64_t* out_idx,
                    float* out_scores, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("indexer_topk: top_k must be in [1, 2048] (got %d)", top_k);
  if (!out_idx || !out_scores) return si::fail("indexer_topk: null output pointer");
  const int mode = causal_ratio > 0 ? si::kModeTopk : (causal_mask ? si::kModeTopkMask : si::kModeTopk);
  return si::run_indexer(q, k, w, w_is_bf16, ab_fp16, B, S, T, H, D, top_k, causal_ratio > 0 ? causal_ratio : 0,
                         causal_mask, mode, out_idx, out_scores, ws, ws_bytes, stream);
}

int si_indexer_topk_ex(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                       int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask, long long s_offset,
                       unsigned flags, int64_t* out_idx, float* out_scores, void* ws, size_t ws_bytes,
                       cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("indexer_topk: top_k must be in [1, 2048] (got %d)", top_k);
  if (!out_idx || !out_scores) return si::fail("indexer_topk: null output pointer");
  const int mode = causal_ratio > 0 ? si::kModeTopk : (causal_mask ? si::kModeTopkMask : si::kModeTopk);
  return si::run_indexer(q, k, w, w_is_bf16, ab_fp16, B, S, T, H, D, top_k, causal_ratio > 0 ? causal_ratio : 0,
                         causal_mask, mode, out_idx, out_scores, ws, ws_bytes, stream, s_offset, flags);
}

int si_indexer_topk_strided(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                            const void* w, const long long* w_strides, int w_is_bf16, int ab_fp16, int B, int S,
                            int T, int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask,
                            long long s_offset, unsigned flags, int64_t* out_idx, float* out_scores, void* ws,
                            size_t ws_bytes, cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("indexer_topk: top_k must be in [1, 2048] (got %d)", top_k);
  if (!out_idx || !out_scores) return si::fail("indexer_topk: null output pointer");
  si::IndexerStrides st;
  if (q_strides) {
    st.q_b = q_strides[0]; st.q_s = q_strides[1]; st.q_h = q_strides[2];
    if (st.q_b < 0 || st.q_s < 0 || st.q_h < 0 || (st.q_b | st.q_s | st.q_h) % 8)
      return si::fail("indexer_topk: q strides must be non-negative multiples of 8 elements");
  }
  if (k_strides) {
    st.k_b = k_strides[0]; st.k_t = k_strides[1];
    if (st.k_b < 0 || st.k_t < 0 || (st.k_b | st.k_t) % 8)
      return si::fail("indexer_topk: k strides must be non-negative multiples of 8 elements");
  }
  if (w_strides) {
    st.w_b = w_strides[0]; st.w_s = w_strides[1]; st.w_h = w_strides[2];
    if (st.w_b < 0 || st.w_s < 0 || st.w_h < 0) return si::fail("indexer_topk: w strides must be non-negative");
  }
  const int mode = causal_ratio > 0 ? si::kModeTopk : (causal_mask ? si::kModeTopkMask : si::kModeTopk);
  return si::run_indexer(q, k, w, w_is_bf16, ab_fp16, B, S, T, H, D, top_k, causal_ratio > 0 ? causal_ratio : 0,
                         causal_mask, mode, out_idx, out_scores, ws, ws_bytes, stream, s_offset, flags, st);
}

int si_topk_row_sort(int64_t* idx_keys, float* out_scores, long long rows, int top_k, cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("topk_row_sort: top_k must be in [1, 2048] (got %d)", top_k);
  if (rows < 0 || (rows > 0 && (!idx_keys || !out_scores))) return si::fail("topk_row_sort: bad arguments");
  cudaError_t e = si::launch_row_sort(reinterpret_cast<unsigned long long*>(idx_keys), out_scores, rows, top_k, stream);
  return e == cudaSuccess ? 0 : si::fail_cuda("topk_row_sort: launch", e);
}

int si_indexer_score(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S, int T,
                     int H, int D, float* out, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!out) return si::fail("indexer_score: null output pointer");
  return si::run_indexer(q, k, w, w_is_bf16, ab_fp16, B, S, T, H, D, 1, 0, nullptr, si::kModeScore, nullptr, out,
                         ws, ws_bytes, stream);
}

}  // extern "C"

// ==================================================================== allocation-free variant
// For callers that cannot allocate device memory themselves (for example a
// host runtime that owns the device allocator and forbids cudaMalloc from
// plugins, or code that must not allocate while a latency-critical stream is
// running): the workspace lives in this file-scope device array instead of a
// caller buffer.  Every GPU that loads the library holds the array until the
// process exits.
namespace si {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, resolved once per device with
// that device current (the host-side symbol is not a device address).
static void* noalloc_scratch_ptr(int* rc) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = fail_cuda("indexer_topk_noalloc: cudaGetDevice", e);
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *rc = fail("indexer_topk_noalloc: device ordinal %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *rc = fail_cuda("indexer_topk_noalloc: cudaGetSymbolAddress", e);
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *rc = 0;
  return ptrs[dev];
}

}  // namespace si

extern "C" {

size_t si_indexer_topk_noalloc_max_ws_bytes(void) { return si::kNoAllocScratchBytes; }

int si_indexer_topk_noalloc(const void* q, const void* k, const void* w, int w_is_bf16, int ab_fp16, int B, int S,
                            int T, int H, int D, int top_k, int causal_ratio, const uint8_t* causal_mask,
                            int64_t* out_idx, float* out_scores, cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("indexer_topk_noalloc: top_k must be in [1, 2048] (got %d)", top_k);
  if (!out_idx || !out_scores) return si::fail("indexer_topk_noalloc: null output pointer");
  if (H != 16 && H != 32 && H != 64 && H != 128)
    return si::fail("indexer_topk_noalloc: H_I must be 16, 32, 64 or 128 (got %d)", H);
  const size_t need = si::indexer_ws_bytes(B < 1 ? 1 : B, S < 1 ? 1 : S, H, top_k);
  if (need > si::kNoAllocScratchBytes)
    return si::fail(
        "indexer_topk_noalloc: needs %zu bytes of scratch, above the built-in maximum of %zu bytes "
        "(smaller H_I*top_k per SM fits; otherwise use si_indexer_topk with a caller workspace)",
        need, si::kNoAllocScratchBytes);
  int rc = 0;
  void* ws = si::noalloc_scratch_ptr(&rc);
  if (!ws) return rc;
  // run_indexer zeroes the status word on `stream`; the candidate buffers need
  // no clearing (per-query counts start at zero in shared memory).
  const int mode = causal_ratio > 0 ? si::kModeTopk : (causal_mask ? si::kModeTopkMask : si::kModeTopk);
  return si::run_indexer(q, k, w, w_is_bf16, ab_fp16, B, S, T, H, D, top_k, causal_ratio > 0 ? causal_ratio : 0,
                         causal_mask, mode, out_idx, out_scores, ws, si::kNoAllocScratchBytes, stream);
}

int si_indexer_topk_noalloc_read_status(int* status_out, cudaStream_t stream) {
  if (!status_out) return si::fail("indexer_topk_noalloc_read_status: null pointer");
  int rc = 0;
  void* ws = si::noalloc_scratch_ptr(&rc);
  if (!ws) return rc;
  return si_read_status(ws, status_out, stream);
}

}  // extern "C"

// ==================================================================== top-k over a score matrix
// Top-k of materialised scores [B,S,T] (the non-streaming branch of the CSA
// index build, flash_sparse/csa.py:55-69): one warp per row streams the row's
// legal prefix t < limit(s) through the same threshold + candidate-buffer +
// exact radix-select scheme as the fused kernel, then writes unsorted keys for
// the row sort.
namespace si {

constexpr int kRowWarps = 8;

__global__ void __launch_bounds__(32 * kRowWarps)
    scores_topk_kernel(const float* __restrict__ scores, int B, int S, int T, int ksel, int ratio, int cap,
                       const uint8_t* __restrict__ mask, unsigned long long* cand, unsigned long long* out_keys) {
  __shared__ uint32_t hist[kRowWarps][256];
  const int wl = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const uint32_t lt = (1u << lane) - 1u;
  const long long nwarps = (long long)gridDim.x * kRowWarps;
  const long long rows = (long long)B * S;
  unsigned long long* buf = cand + ((long long)blockIdx.x * kRowWarps + wl) * cap;
  for (long long row = (long long)blockIdx.x * kRowWarps + wl; row < rows; row += nwarps) {
    const int s = (int)(row % S);
    int lim = T;
    if (ratio > 0) {
      const long long l = ((long long)s + 1) / ratio;
      lim = l < T ? (int)l : T;
    }
    const float* sr = scores + row * (long long)T;
    unsigned long long thr = 0ull;
    int cnt = 0;
    for (int t0 = 0; t0 < lim; t0 += 32) {
      if (cnt > cap - 32) {
        thr = warp_select_topk(buf, cnt, ksel, hist[wl]);
        cnt = ksel;
      }
      const int t = t0 + (int)lane;
      const bool legal = t < lim && (!mask || mask[row * (long long)T + t] != 0);
      const unsigned long long key = legal ? make_key(sr[t], t) : 0ull;
      const bool pass = legal && key > thr;
      const uint32_t bal = __ballot_sync(0xffffffffu, pass);
      if (pass) buf[cnt + __popc(bal & lt)] = key;
      cnt += __popc(bal);
      __syncwarp();
    }
    if (cnt > ksel) {
      warp_select_topk(buf, cnt, ksel, hist[wl]);
      cnt = ksel;
    }
    unsigned long long* dst = out_keys + row * ksel;
    for (int x = (int)lane; x < ksel; x += 32) dst[x] = x < cnt ? buf[x] : 0ull;
    __syncwarp();
  }
}

static int scores_topk_grid(long long rows) {
  const long long want = (rows + kRowWarps - 1) / kRowWarps;
  const long long maxg = (long long)device_sm_count() * 8;
  return (int)(want < maxg ? (want > 0 ? want : 1) : maxg);
}

}  // namespace si

extern "C" {

size_t si_scores_topk_ws_bytes(int B, int S, int top_k) {
  const long long rows = (long long)(B > 0 ? B : 1) * (S > 0 ? S : 1);
  return si::kStatusBytes + (size_t)si::scores_topk_grid(rows) * si::kRowWarps * si::pick_cap(top_k > 0 ? top_k : 1) *
                                sizeof(unsigned long long);
}

int si_scores_topk_mask(const float* scores, int B, int S, int T, int top_k, int causal_ratio,
                        const uint8_t* causal_mask, int64_t* out_idx, float* out_scores, void* ws, size_t ws_bytes,
                        cudaStream_t stream) {
  if (top_k < 1 || top_k > 2048) return si::fail("scores_topk: top_k must be in [1, 2048] (got %d)", top_k);
  if (B < 1 || S < 0 || T < 0) return si::fail("scores_topk: bad sizes");
  if ((S > 0 && T > 0 && !scores) || !out_idx || !out_scores || !ws) return si::fail("scores_topk: null pointer");
  const size_t need = si_scores_topk_ws_bytes(B, S, top_k);
  if (ws_bytes < need) return si::fail("scores_topk: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  const long long rows = (long long)B * S;
  if (rows == 0) return 0;
  if (T == 0) {
    cudaError_t e = si::launch_fill_pad(out_idx, out_scores, rows * top_k, stream);
    return e == cudaSuccess ? 0 : si::fail_cuda("scores_topk: pad", e);
  }
  const int grid = si::scores_topk_grid(rows);
  auto* keys = reinterpret_cast<unsigned long long*>(out_idx);
  si::scores_topk_kernel<<<grid, 32 * si::kRowWarps, 0, stream>>>(
      scores, B, S, T, top_k, causal_ratio > 0 ? causal_ratio : 0, si::pick_cap(top_k), causal_mask,
      reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(ws) + si::kStatusBytes), keys);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return si::fail_cuda("scores_topk: launch", e);
  e = si::launch_row_sort(keys, out_scores, rows, top_k, stream);
  return e == cudaSuccess ? 0 : si::fail_cuda("scores_topk: row sort", e);
}

int si_scores_topk(const float* scores, int B, int S, int T, int top_k, int causal_ratio, int64_t* out_idx,
                   float* out_scores, void* ws, size_t ws_bytes, cudaStream_t stream) {
  return si_scores_topk_mask(scores, B, S, T, top_k, causal_ratio, nullptr, out_idx, out_scores, ws, ws_bytes,
                             stream);
}

}  // extern "C"
