// Sparse MQA attention forward with attention sink, for sm_100a.
//
// Math (flash_sparse/reference.py:93-129; LSE as flash_sparse/triton/sparse_attn_fwd.py:175):
//   for query (b,s) and head h, over the selected KV rows j = idx[b,s,:] (-1 = masked):
//     p_j = exp(scale * q[b,s,h,:] . kv[b,j,:]),  l = sum_j p_j + exp(sink[h])
//     o[b,s,h,:] = sum_j p_j * kv[b,j,dv_off:dv_off+Dv] / l,   lse = log(l)
//   (computed with a running shift for stability; the sink enters the
//   denominator only).
//
// Mapping.  One persistent CTA per SM walks work items (b, s, 64-head group).
// The item's selected KV rows (1152 bytes per index at D=576) are gathered NK at
// a time into 128-byte-swizzled shared-memory stages that serve both GEMMs:
//   MMA1  S[64 x NK]  = Q . KV^T           (M=64, K=D; Q from TMEM, KV K-major)
//   MMA2  O[64 x Dv] += P . V              (M=64, K=NK, P K-major, V MN-major)
// With M=64 an accumulator occupies 16 lanes of each 32-lane TMEM quarter.  O
// lives in lanes 0-15 (columns [0,Dv)); lanes 16-31 hold the two S buffers
// (columns [0,2*NK)) and Q, the A operand of MMA1, which must sit on the same
// lanes as S: its 64-column atoms fill a ring of 32-column slots after the S
// buffers, so the next item's first atoms go in while the current item runs.
//
// Softmax warps (4, one per lane quarter = 16 heads): threads i and 16+i of a
// warp share head row i, each taking 16 of the tile's 32 scores (16x32bx2 TMEM
// load from the S lanes) and half of the row's O columns; row max and sum are
// combined with one shuffle.  The running shift is only raised when the tile max
// exceeds it by more than 8 (log2 units), so O is rescaled (ld/scale/st with
// the 16x32bx2 TMEM shape, which touches lanes 0-15 only) rarely; P = exp2(s -
// shift) <= 256 stays well inside the bf16 range.  P goes to shared memory (bf16) as
// the A operand of MMA2.
//
// Warp roles (672 threads): warp 0 TMA for Q atoms into a staging ring (and an
// L2 prefetch of the next item's Q), warp 1 TMEM alloc + Q.K^T issue, warp 16
// P.V issue, warps 2-5 softmax / O correction / output, warps 6-13 kv row
// gathers with 16-byte cp.async (completion signalled on the stage barrier with
// cp.async.mbarrier.arrive.noinc), warp 14 TMA gather4 for the first atoms of
// each row (single kv tensor only) and the per-stage valid-slot mask, warp 15
// the index ring (it reads the selected indices several tiles ahead into shared
// memory, so no gather thread waits on a global load of an index), warps 17-20
// move the staged Q atoms into TMEM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "capi_common.h"
#include "ptx.cuh"
#include "../../include/streamindex_b200.h"

namespace si {
namespace attn {

constexpr int kHeads = 64;    // UMMA M (heads per work item)
constexpr int kThreads = 672;   // + warp 14: TMA row gathers, 15: index ring, 16: P.V issue, 17-20: Q to TMEM
constexpr int kIdxSlots = 8;    // index-ring slots (one tile of NK indices each)
constexpr int kGatherWarps = 8;   // warps 6-13
constexpr int kSmemMax = 232448;
constexpr int kMaxAtoms = 16;  // D <= 1024
constexpr int kQStage = 4;     // Q staging atoms (64 rows x 128 B) in shared memory
constexpr int kQCol = 64;      // first TMEM column of Q (lanes 16-31 of each quarter), after the two S buffers
constexpr int kQSlots = (512 - kQCol) / 32;  // 32-column Q atom slots in TMEM (14)
// Full-width value output in one pass (the reference's default D_v = D = 576 of
// the 576/512 MLA layout): O's first 512 columns stay in lanes 0-15, the extra
// kXV value columns take the last kXV TMEM columns of lanes 16-31 (after S and
// a Q ring shortened to kQSlotsXV slots, so D <= 768 there).
constexpr int kXV = 64;
constexpr int kQSlotsXV = (512 - kQCol - kXV) / 32;  // 12
// Element modes (compile-time, so the bf16 path carries no per-element
// branches): q / kv / o bf16, all fp16, or bf16 q / o over FP8 KV rows.
enum AttnMode : int { kBf16 = 0, kF16 = 1, kFp8Rows = 2 };

template <int XV>
struct QRing {
  static constexpr int kSlots = XV ? kQSlotsXV : kQSlots;
};

// Q lives in tensor memory as the A operand of Q.K^T.  Its atoms fill a ring
// of kQSlots 32-column slots: item j's atom a (CTA-local numbering) goes to
// slot (j*NA + a) % kQSlots, so while item j-1 runs, the first kQSlots-NA
// atoms of item j can already be written into slots item j-1 does not use.
__host__ __device__ inline bool q_fits_tmem(int NA) { return NA <= kQSlots; }
__host__ __device__ inline int q_smem_bytes(int) { return kQStage * kHeads * 128; }

struct Params {
  int B, S, H, D;      // D: qk head dim (multiple of 8)
  int NA;              // ceil(D/64) swizzle atoms per row
  int Nkv;             // kv rows per batch (Nkv1 + Nkv2)
  int Nkv1;            // rows of the first kv tensor; indices >= Nkv1 read kv2
  int K;               // indices per query
  int Dv, dv_off;      // value columns [dv_off, dv_off+Dv) of kv (multiples of 64)
  int o_ld, o_off;     // output row stride (elements) and column offset
  float scale_log2;    // softmax_scale * log2(e)
  const int* idx;      // [B,S,K] (explicit index list), or null with comp set
  // CSA index list built in the index ring instead of read from idx (the
  // concatenation of flash_sparse/csa.py:176-179 with the window of
  // flash_sparse/reference.py:460-475): slot kk < nwin is the window position
  // s_glob - nwin + 1 + kk (-1 if negative), slot nwin + j the compressed pick
  // comp[b, s, j] offset by Nkv1 (-1 kept).  K = nwin + comp_k.
  const long long* comp;  // [B,S,comp_k] int64 or null
  int comp_k, nwin;
  long long s_off;      // global position of local query 0
  const __nv_bfloat16* kv;   // [B,Nkv1,D]
  const __nv_bfloat16* kv2;  // [B,Nkv-Nkv1,D] or null
  const float* sink;   // [H]
  __nv_bfloat16* o;    // [B,S,H,o_ld]
  float* lse;          // [B,S,H] or null
  int* status;
  int hgroups;         // ceil(H/64)
  int na_tma;          // leading atoms of each kv row gathered by TMA (warp 14); the rest by cp.async
  int o_v8;            // o rows are 32-byte aligned: 256-bit output stores
  // FP8 KV rows (fp8 != 0): kv / kv2 hold rows of row_bytes bytes:
  //   [n_nope e4m3 | n_nope/64 fp32 block scales | pad to 16 B | n_rope bf16 (at rope_off) | pad to 16 B]
  // dequantised by the gather warps into the same bf16 stage layout:
  //   value = bf16(float(e4m3) * scale[block])
  int fp8, n_nope, row_bytes, rope_off;
  int f16;             // q / kv / o are fp16 (else bf16); P is packed in the same type
  unsigned long long* trace;  // debug builds (SI_ATTN_TRACE) only: per-role timestamps of CTA 0
};

#ifdef SI_ATTN_TRACE
// trace layout: [role 0..2][item < 4][tile < 16][point < 8] globaltimer ns
#define SI_TRACE(role, item, tile, pt)                                                                  \
  do {                                                                                                  \
    if (p.trace && blockIdx.x == 0 && (item) < 4 && (tile) < 16)                                        \
      p.trace[(((role) * 4 + (item)) * 16 + (tile)) * 8 + (pt)] = globaltimer();                         \
  } while (0)
#define SI_TRACE_IF(cond, role, item, tile, pt) \
  do {                                          \
    if (cond) SI_TRACE(role, item, tile, pt);   \
  } while (0)
#else
#define SI_TRACE_IF(cond, role, item, tile, pt) \
  do {                                          \
  } while (0)
#define SI_TRACE(role, item, tile, pt) \
  do {                                 \
  } while (0)
#endif

struct __align__(8) Misc {
  uint64_t kv_full[8], kv_empty[8];
  uint64_t idx_full[kIdxSlots], idx_empty[kIdxSlots];
  uint32_t kvmask[8];             // valid-slot mask of the tile in each kv stage
  int idx_ring[kIdxSlots][32];    // selected kv rows of upcoming tiles (-1 = masked)
  uint64_t q_full[2], q_empty;  // q_full[j & 1]: item j's Q is in TMEM; q_empty: an item's Q.K^T completed
  uint64_t qs_full[kQStage], qs_empty[kQStage];  // Q staging ring
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done[2], o_free;  // pv_done[b]: MMA2 that read P buffer b completed
  uint32_t tmem_base;
  int abort_flag;
};

template <int NK>
__host__ __device__ inline int stage_bytes(int NA) { return NA * NK * 128; }

template <int NK>
__host__ __device__ inline int num_stages(int NA) {
  const int fixed = 1024 + q_smem_bytes(NA) + 2 * NK * 128 + (int)sizeof(Misc) + 64;
  int n = (kSmemMax - fixed) / stage_bytes<NK>(NA);
  return n > 8 ? 8 : n;
}

template <int NK>
__host__ __device__ inline size_t smem_bytes(int NA) {
  return 1024 + (size_t)q_smem_bytes(NA) + (size_t)num_stages<NK>(NA) * stage_bytes<NK>(NA) + 2 * NK * 128 +
         sizeof(Misc);
}

}  // namespace attn
}  // namespace si

namespace si {
namespace attn {

// Address of kv row v of batch b in the (possibly split) kv storage.
__device__ __forceinline__ const __nv_bfloat16* kv_row_ptr(const Params& p, int b, int v) {
  if (v < p.Nkv1) return p.kv + ((size_t)b * p.Nkv1 + v) * p.D;
  return p.kv2 + ((size_t)b * (p.Nkv - p.Nkv1) + (v - p.Nkv1)) * p.D;
}
__device__ __forceinline__ const uint8_t* kv_row_ptr_fp8(const Params& p, int b, int v) {
  if (v < p.Nkv1) return reinterpret_cast<const uint8_t*>(p.kv) + ((size_t)b * p.Nkv1 + v) * p.row_bytes;
  return reinterpret_cast<const uint8_t*>(p.kv2) + ((size_t)b * (p.Nkv - p.Nkv1) + (v - p.Nkv1)) * p.row_bytes;
}

// 16 e4m3 values -> 16 bf16 = bf16(float(e) * scale), two 16-byte stage chunks.
__device__ __forceinline__ void dequant16_e4m3(const uint4& x, float scale, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t h01, h23;  // f16x2 (exact: every e4m3 value is an f16 value)
    asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(h01), "=r"(h23) : "r"(w[i]));
    const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
    const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
    out[2 * i] = pack_bf16x2(f01.x * scale, f01.y * scale);
    out[2 * i + 1] = pack_bf16x2(f23.x * scale, f23.y * scale);
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

// 128-byte-swizzled stage offset of 16-byte chunk ch of row r in atom a.
template <int NK>
__device__ __forceinline__ uint32_t stage_off(int a, int r, int ch) {
  return (uint32_t)(a * NK * 128 + r * 128) + ((uint32_t)(ch ^ (r & 7)) << 4);
}

template <int NK, int DVH, int XV, int MODE>
__device__ __forceinline__ void attn_softmax(const Params& p, Misc* ms, uint8_t* sP, uint32_t tmem, int warp,
                                             uint32_t lane, int nitems, int ntiles) {
  constexpr float kLn2 = 0.6931471805599453f;
  constexpr float kLog2e = 1.4426950408889634f;
  const int qd = warp & 3;
  const int r = (int)(lane & 15);          // row within the quarter
  const int half = (int)(lane >> 4);       // which 16 of the tile's 32 keys / which half of O's columns
  const int hrow = 16 * qd + r;            // row within the 64-head group
  const uint32_t tq = tmem + ((uint32_t)(32 * qd) << 16);
  volatile int* abort_flag = &ms->abort_flag;
  uint32_t sf[2] = {0, 0};
  // kv stage of the current tile (same ring walk as the gather and MMA roles):
  // its valid-slot mask is published before the stage's kv_full arrival
  const uint32_t nst = (uint32_t)num_stages<NK>(p.NA);
  uint32_t kst = 0, kph = 0;
  // MMA2 of tile j signals pv_done[j & 1]; waited[b] counts completions of
  // barrier b already consumed, so "MMA2 of tile j is done" is a wait for
  // completion number (j >> 1) of barrier j & 1 (skipped if already seen).
  uint32_t waited[2] = {0, 0}, issued_base[2] = {0, 0};
  auto wait_pv = [&](int j) -> bool {
    const int bb = j & 1;
    const uint32_t need = issued_base[bb] + (uint32_t)(j >> 1) + 1;
    while (waited[bb] < need) {
      if (!mbar_wait(&ms->pv_done[bb], waited[bb] & 1, &ms->abort_flag, p.status, kErrWaitAccFull)) return false;
      ++waited[bb];
    }
    return true;
  };

  for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int hg = it % p.hgroups;
    const int bs = it / p.hgroups;
    const int head = hg * kHeads + hrow;
#ifdef SI_ATTN_TRACE
    const int ii = (it - (int)blockIdx.x) / (int)gridDim.x;
    const bool tr = (warp == 2 && lane == 0);
#endif
    const float sink2 = head < p.H ? p.sink[head] * kLog2e : 0.f;
    // m_used / l are kept identically by both half-warp threads of a row
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      SI_TRACE_IF(tr, 2, ii, t, 0);
      if (!mbar_wait(&ms->s_full[t & 1], sf[t & 1], abort_flag, p.status, kErrWaitAccFull)) {
        ok = false;
        break;
      }
      sf[t & 1] ^= 1;
      // S of this tile is complete, so its kv stage has long been filled; the
      // wait only acquires the mask written before the stage's arrival
      if (!mbar_wait(&ms->kv_full[kst], kph, abort_flag, p.status, kErrWaitTmaFull)) {
        ok = false;
        break;
      }
      const uint32_t vmask = *reinterpret_cast<volatile uint32_t*>(&ms->kvmask[kst]) >> (half * 16);
      if (++kst == nst) {
        kst = 0;
        kph ^= 1;
      }
      tc_fence_after();
      SI_TRACE_IF(tr, 2, ii, t, 1);
      float sv[16];
      tmem_ld16x32bx2_x16_sync<16>(tq + (16u << 16) + (t & 1) * NK, sv);
      SI_TRACE_IF(tr, 2, ii, t, 2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms->s_free[t & 1]);

      // The max is taken on the raw scores and the scale is folded into the
      // exponent's FMA (a positive scale keeps the order; any other scale is
      // applied up front).  Masked slots become -inf, and a fully valid half
      // tile (the common case) skips the per-slot test.
      float sc = p.scale_log2;
      if (!(sc > 0.f)) {
#pragma unroll
        for (int j = 0; j < 16; ++j) sv[j] *= sc;
        sc = 1.f;
      }
      if ((vmask & 0xffffu) != 0xffffu) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (!((vmask >> j) & 1u)) sv[j] = -INFINITY;
      }
      float mx[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int j = 4; j < 16; ++j) mx[j & 3] = fmaxf(mx[j & 3], sv[j]);
      float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16)) * sc;
      bool rescale = false;
      float alpha = 1.f;
      if (mt > -INFINITY) {
        if (m_used == -INFINITY) {
          m_used = mt;  // nothing accumulated yet for this row: O row is zero
        } else if (mt > m_used + 8.f) {
          alpha = exp2f(m_used - mt);
          m_used = mt;
          l *= alpha;
          rescale = true;
        }
      }
      // m_used = -inf only while no valid key has been seen; then every p is 0
      const float shift = (m_used == -INFINITY) ? INFINITY : m_used;
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        sv[j] = ex2_approx(fmaf(sv[j], sc, -shift));
        ps[j & 3] += sv[j];
      }
      float psum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
      psum += __shfl_xor_sync(0xffffffffu, psum, 16);
      l += psum;
      SI_TRACE_IF(tr, 2, ii, t, 5);

      // P buffer t&1 was last read by MMA2 of tile t-2; a rescale of O also
      // needs MMA2 of tile t-1 to be complete.
      const bool any_rescale = __any_sync(0xffffffffu, rescale);
      if (t >= 2 && !wait_pv(t - 2)) {
        ok = false;
        break;
      }
      if (any_rescale && t >= 1 && !wait_pv(t - 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      SI_TRACE_IF(tr, 2, ii, t, 3);
      if (any_rescale) {
#pragma unroll 1
        for (int c = 0; c < DVH / 32; ++c) {
          float v[32];
          tmem_ld16x32bx2_x32_sync<DVH>(tq + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= alpha;
          tmem_st16x32bx2_x32<DVH>(tq + c * 32, v);
        }
        if (XV) {  // extra value columns in lanes 16-31: this thread's 32 of them
          float v[32];
          tmem_ld16x32bx2_x32_sync<XV / 2>(tq + (16u << 16) + (512 - XV), v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= alpha;
          tmem_st16x32bx2_x32<XV / 2>(tq + (16u << 16) + (512 - XV), v);
        }
        tmem_st_wait();
      }
      {
        // P row hrow, keys [16*half, 16*half+16): two 8-key core-matrix chunks
        uint8_t* prow = sP + (t & 1) * NK * 128 + (hrow >> 3) * 128 + (hrow & 7) * 16 + half * 2048;
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
          uint4 u;
          u.x = pack_x2(sv[kc * 8 + 0], sv[kc * 8 + 1], MODE == kF16);
          u.y = pack_x2(sv[kc * 8 + 2], sv[kc * 8 + 3], MODE == kF16);
          u.z = pack_x2(sv[kc * 8 + 4], sv[kc * 8 + 5], MODE == kF16);
          u.w = pack_x2(sv[kc * 8 + 6], sv[kc * 8 + 7], MODE == kF16);
          *reinterpret_cast<uint4*>(prow + kc * 1024) = u;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ms->p_full[t & 1]);
      SI_TRACE_IF(tr, 2, ii, t, 4);
    }
    if (!ok) break;
    if ((ntiles >= 2 && !wait_pv(ntiles - 2)) || !wait_pv(ntiles - 1)) break;
    tc_fence_after();
    issued_base[0] += (uint32_t)((ntiles + 1) >> 1);  // MMA2s per buffer in this item
    issued_base[1] += (uint32_t)(ntiles >> 1);

    // ---- epilogue: sink in the denominator, normalise, write O and LSE
    // The shift becomes max(m, sink) (sparse_attn_fwd.py:152-156), so a sink far
    // above every score cannot overflow the denominator.
    if (m_used == -INFINITY) m_used = sink2;  // no valid key: O = 0, l = exp(sink - sink)
    const float m_fin = fmaxf(m_used, sink2);
    const float o_scale = exp2f(m_used - m_fin);
    const float l_tot = l * o_scale + exp2f(sink2 - m_fin);
    const float inv = l_tot > 0.f ? o_scale / l_tot : 0.f;
    if (half == 0 && head < p.H && p.lse)
      p.lse[(size_t)bs * p.H + head] = l_tot > 0.f ? (m_fin + log2f(l_tot)) * kLn2 : -1.0e30f;
    __nv_bfloat16* orow = p.o + ((size_t)bs * p.H + head) * p.o_ld + p.o_off + half * DVH;
    constexpr int NC = DVH / 32 + (XV ? 1 : 0);
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      float v[32];
      __nv_bfloat16* dst = orow + c * 32;
      if (XV && c == DVH / 32) {  // the extra value columns (lanes 16-31)
        tmem_ld16x32bx2_x32_sync<XV / 2>(tq + (16u << 16) + (512 - XV), v);
        dst = orow - half * DVH + 2 * DVH + half * (XV / 2);
      } else {
        tmem_ld16x32bx2_x32_sync<DVH>(tq + c * 32, v);
      }
      if (head < p.H) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = pack_x2(v[2 * j] * inv, v[2 * j + 1] * inv, MODE == kF16);
        if (p.o_v8) {  // two 32-byte stores: half the store transactions of 16-byte ones
#pragma unroll
          for (int j = 0; j < 16; j += 8)
            asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst + 2 * j), "r"(w[j]),
                         "r"(w[j + 1]), "r"(w[j + 2]), "r"(w[j + 3]), "r"(w[j + 4]), "r"(w[j + 5]), "r"(w[j + 6]),
                         "r"(w[j + 7])
                         : "memory");
        } else {
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(w[j], w[j + 1], w[j + 2], w[j + 3]);
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&ms->o_free);
  }
}

template <int NK, int DVH, int XV, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_attn_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_kv,
                           Params p) {
  static_assert(NK == 32, "one index per lane per tile");
  constexpr int DV = 2 * DVH;
  constexpr int NMMA = DV < 256 ? DV : 256;  // UMMA N of the PV product
  constexpr int NCH = DV / NMMA;
  constexpr int QSL = QRing<XV>::kSlots;  // Q atom slots in TMEM
  static_assert(XV == 0 || DV == 512, "extra value columns only beside a full 512-column O");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NA = p.NA;
  const int NST = num_stages<NK>(NA);
  const int SB = stage_bytes<NK>(NA);
  uint8_t* sQ = smem;  // [kQStage][64 rows][128 B], 128B swizzle: Q staging ring
  uint8_t* sKV = sQ + q_smem_bytes(NA);                 // [NST][NA][NK rows][128 B], 128B swizzle
  uint8_t* sP = sKV + (size_t)NST * SB;                 // [2][NK/8][8 row groups][8 rows][16 B]
  Misc* ms = reinterpret_cast<Misc*>(sP + 2 * NK * 128);

  const int warp = threadIdx.x / 32;
  const uint32_t lane = lane_id();
  const int nitems = p.B * p.S * p.hgroups;
  const int ntiles = p.K > 0 ? (p.K + NK - 1) / NK : 1;
  volatile int* abort_flag = &ms->abort_flag;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NST; ++i) {
      // one cp.async completion arrival per gather thread + the TMA warp's
      // arrival (with its byte count when it gathers atoms)
      mbar_init(&ms->kv_full[i], kGatherWarps * 32 + 1);
      mbar_init(&ms->kv_empty[i], 1);
    }
    for (int i = 0; i < kIdxSlots; ++i) {
      mbar_init(&ms->idx_full[i], 32);                // every lane of the index warp
      mbar_init(&ms->idx_empty[i], kGatherWarps + 1);  // gather warps + TMA warp
    }
    mbar_init(&ms->q_full[0], 4);  // one arrival per loader warp
    mbar_init(&ms->q_full[1], 4);
    mbar_init(&ms->q_empty, 1);
    for (int i = 0; i < kQStage; ++i) {
      mbar_init(&ms->qs_full[i], 1);
      mbar_init(&ms->qs_empty[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ms->s_full[i], 1);
      mbar_init(&ms->s_free[i], 4);
      mbar_init(&ms->p_full[i], 4);
    }
    mbar_init(&ms->pv_done[0], 1);
    mbar_init(&ms->pv_done[1], 1);
    mbar_init(&ms->o_free, 4);
    ms->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map_q);
    prefetch_tmap(&map_kv);
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
    // ------------------------------------------------------------ producer: Q tile (TMA)
    uint32_t qslot = 0, qsph = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
      const int hg = it % p.hgroups;
      const int bs = it / p.hgroups;
      const int nx = it + (int)gridDim.x;
      if (nx < nitems && lane < NA) {  // next item's Q into L2 while this one runs
        const int nbs = nx / p.hgroups;
        tma_prefetch_l2_4d(&map_q, (int)lane * 64, (nx % p.hgroups) * kHeads, nbs % p.S, nbs / p.S);
      }
      const int qs = bs % p.S, qb = bs / p.S;
      // Q atoms through the staging ring; the loader warps move them to TMEM
      bool ok = true;
      for (int a = 0; a < NA; ++a) {
        if (!mbar_wait(&ms->qs_empty[qslot], qsph ^ 1, abort_flag, p.status, kErrWaitQ)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_expect_tx(&ms->qs_full[qslot], (uint32_t)kHeads * 128);
          tma_load_4d(sQ + qslot * kHeads * 128, &map_q, &ms->qs_full[qslot], a * 64, hg * kHeads, qs, qb);
        }
        __syncwarp();
        if (++qslot == (uint32_t)kQStage) {
          qslot = 0;
          qsph ^= 1;
        }
      }
      if (!ok) break;
    }
  } else if (warp >= 9 + kGatherWarps) {
    // ------------------------------------------------------------ Q loaders
    // Warp w owns TMEM lane quarter w % 4: rows 16*(w%4) .. +15 of the 64-head
    // group at lanes 16-31, beside S (the A operand of an M=64 MMA sits on the
    // same lanes as its D).  Each staged atom (64 Q columns) goes in with one
    // 16x32bx2 store per warp: thread i writes row i's columns [0,32) of the
    // atom, thread 16+i columns [32,64) (two bf16 per 32-bit TMEM column).  An
    // atom slot is rewritten only after the Q.K^T of the item that last used it
    // completed (q_empty completions are counted in item order).
    {
      const int qd = warp & 3;
      const int hrow = 16 * qd + (int)(lane & 15);
      const uint32_t half = lane >> 4;
      const uint32_t tq = tmem + ((uint32_t)(32 * qd + 16) << 16) + kQCol;
      uint32_t qslot = 0, qsph = 0, done_items = 0;
      bool ok = true;
      auto wait_items_done = [&](int n) -> bool {  // Q.K^T of CTA-local items 0..n-1 complete
        while ((int)done_items < n) {
          if (!mbar_wait(&ms->q_empty, done_items & 1, abort_flag, p.status, kErrWaitQ)) return false;
          ++done_items;
        }
        return true;
      };
      int jj = 0;
      for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x, ++jj) {
        for (int a = 0; a < NA; ++a) {
          const int g = jj * NA + a;
          const int prev = g - QSL;  // atom that last used this slot
          if (prev >= 0 && !wait_items_done(prev / NA + 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (!mbar_wait(&ms->qs_full[qslot], qsph, abort_flag, p.status, kErrWaitQ)) {
            ok = false;
            break;
          }
          const uint8_t* rowp = sQ + qslot * kHeads * 128 + hrow * 128;
          uint32_t v[16];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t c = 4 * half + (uint32_t)k;
            const uint4 x = *reinterpret_cast<const uint4*>(rowp + ((c ^ (uint32_t)(hrow & 7)) << 4));
            v[4 * k + 0] = x.x;
            v[4 * k + 1] = x.y;
            v[4 * k + 2] = x.z;
            v[4 * k + 3] = x.w;
          }
          tmem_st16x32bx2_x16<16>(tq + (uint32_t)(g % QSL) * 32, v);
          __syncwarp();
          if (lane == 0) mbar_arrive(&ms->qs_empty[qslot]);
          if (++qslot == (uint32_t)kQStage) {
            qslot = 0;
            qsph ^= 1;
          }
        }
        // q_full[jj & 1] was last consumed for item jj-2, whose Q.K^T began
        // before item jj-2's completed
        if (!ok || (jj >= 2 && !wait_items_done(jj - 1))) break;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms->q_full[jj & 1]);
      }
    }
  } else if (warp == 6 + kGatherWarps) {
    // ------------------------------------------------------------ TMA row gathers (gather4) of atoms [0, na_tma)
    // and the valid-slot mask of every tile (published before this warp's kv_full arrival)
    uint32_t st = 0, kph = 0, islot = 0, iph = 0;
    const int g4 = (int)lane & 7;
    const int a = (int)lane >> 3;
    bool ok = true;
    for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
      const int bs = it / p.hgroups;
      const int b = bs / p.S;
      for (int t = 0; t < ntiles; ++t) {
        if (!mbar_wait(&ms->idx_full[islot], iph, abort_flag, p.status, kErrWaitTmaFull)) {
          ok = false;
          break;
        }
        const int v = ms->idx_ring[islot][lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms->idx_empty[islot]);
        if (++islot == (uint32_t)kIdxSlots) {
          islot = 0;
          iph ^= 1;
        }
        const uint32_t vm = __ballot_sync(0xffffffffu, v >= 0);
        const int row = v >= 0 ? b * p.Nkv + v : p.B * p.Nkv;  // out of range: zero fill
        if (!mbar_wait(&ms->kv_empty[st], kph ^ 1, abort_flag, p.status, kErrWaitTmaEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          ms->kvmask[st] = vm;
          if (p.na_tma > 0)
            mbar_expect_tx(&ms->kv_full[st], (uint32_t)(p.na_tma * NK * 128));
          else
            mbar_arrive(&ms->kv_full[st]);
        }
        __syncwarp();
        if (p.na_tma > 0) {
          const int r0 = __shfl_sync(0xffffffffu, row, 4 * g4 + 0);
          const int r1 = __shfl_sync(0xffffffffu, row, 4 * g4 + 1);
          const int r2 = __shfl_sync(0xffffffffu, row, 4 * g4 + 2);
          const int r3 = __shfl_sync(0xffffffffu, row, 4 * g4 + 3);
          if (a < p.na_tma)
            tma_gather4(sKV + (size_t)st * SB + a * NK * 128 + g4 * 4 * 128, &map_kv, &ms->kv_full[st], a * 64, r0,
                        r1, r2, r3);
          __syncwarp();
        }
        if (++st == (uint32_t)NST) {
          st = 0;
          kph ^= 1;
        }
      }
    }
  } else if (warp == 7 + kGatherWarps) {
    // ------------------------------------------------------------ index ring producer
    // Reads the selected indices of 8 tiles at a time (independent loads in
    // flight together), then publishes them one tile per slot as slots free up.
    uint32_t islot = 0, iph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
      const int bs = it / p.hgroups;
      const int b = bs / p.S, s = bs % p.S;
      const int* src = p.idx + ((size_t)b * p.S + s) * p.K;
      const long long* csrc = p.comp + ((size_t)b * p.S + s) * p.comp_k;
      const long long s_glob = p.s_off + s;
      for (int t0 = 0; t0 < ntiles && ok; t0 += 8) {
        // (the explicit-list loads stay a branch-free unrolled batch: a branch
        // per element here slowed the whole kernel by ~4%)
        int v[8];
        if (p.comp == nullptr) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int kk = (t0 + j) * NK + (int)lane;
            v[j] = kk < p.K ? src[kk] : -1;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int kk = (t0 + j) * NK + (int)lane;
            if (kk < p.nwin) {
              const long long pos = s_glob - p.nwin + 1 + kk;
              v[j] = pos >= 0 ? (int)pos : -1;
            } else if (kk < p.K) {
              const long long c = csrc[kk - p.nwin];
              v[j] = c >= 0 ? (int)(c + p.Nkv1) : -1;
            } else {
              v[j] = -1;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (t0 + j >= ntiles) break;
          if (!mbar_wait(&ms->idx_empty[islot], iph ^ 1, abort_flag, p.status, kErrWaitTmaEmpty)) {
            ok = false;
            break;
          }
          ms->idx_ring[islot][lane] = (v[j] >= 0 && v[j] < p.Nkv) ? v[j] : -1;
          mbar_arrive(&ms->idx_full[islot]);
          if (++islot == (uint32_t)kIdxSlots) {
            islot = 0;
            iph ^= 1;
          }
        }
      }
    }
  } else if (warp >= 6 && warp < 6 + kGatherWarps) {
    // ------------------------------------------------------------ KV row gathers (cp.async)
    // A tile is NK rows x NA 128-byte atoms.  Gather warp gw owns rows
    // 4*gw .. 4*gw+3 of every tile: 8 lanes per row, lane & 7 = 16-byte chunk of
    // an atom, so one warp instruction copies 4 rows x 128 bytes and each thread
    // computes its row address once per tile and then issues its atoms back to
    // back.  The destination applies the 128-byte swizzle (16-byte chunk c of row
    // r goes to chunk c ^ (r & 7)), the layout the UMMA descriptors expect.
    static_assert(kGatherWarps * 4 == NK, "one gather-warp row quad per 4 tile rows");
    const int gw = warp - 6;
    const int r = 4 * gw + (int)(lane >> 3);
    const uint32_t c = lane & 7;
    const uint32_t dst_off = (uint32_t)r * 128 + ((c ^ (uint32_t)(r & 7)) << 4);
    uint32_t st = 0, kph = 0, islot = 0, iph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
      const int bs = it / p.hgroups;
      const int b = bs / p.S;
#ifdef SI_ATTN_TRACE
      const int ii = (it - (int)blockIdx.x) / (int)gridDim.x;
      const bool tr = (gw == 0 && lane == 0);
#endif
      for (int t = 0; t < ntiles; ++t) {
        SI_TRACE_IF(tr, 0, ii, t, 0);
        if (!mbar_wait(&ms->idx_full[islot], iph, abort_flag, p.status, kErrWaitTmaFull)) {
          ok = false;
          break;
        }
        const int row = ms->idx_ring[islot][r];
        const bool vld = row >= 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ms->idx_empty[islot]);
        if (++islot == (uint32_t)kIdxSlots) {
          islot = 0;
          iph ^= 1;
        }
        if (!mbar_wait(&ms->kv_empty[st], kph ^ 1, abort_flag, p.status, kErrWaitTmaEmpty)) {
          ok = false;
          break;
        }
        SI_TRACE_IF(tr, 0, ii, t, 1);
        if (MODE == kFp8Rows) {
          // FP8 rows: this thread loads 16-byte chunks q = c + 8i of the row's
          // e4m3 part (64-dim block q/4 = atom q/4), the row's block scales and
          // rope chunk c, then writes the dequantised bf16 chunks into the stage.
          uint4 x[4] = {}, rp = make_uint4(0u, 0u, 0u, 0u);
          float4 sc0 = make_float4(0.f, 0.f, 0.f, 0.f), sc1 = sc0;
          const int nq = p.n_nope >> 4;
          if (vld) {
            const uint8_t* rowp = kv_row_ptr_fp8(p, b, row);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int qc = (int)c + 8 * i;
              if (qc < nq) x[i] = __ldg(reinterpret_cast<const uint4*>(rowp) + qc);
            }
            sc0 = __ldg(reinterpret_cast<const float4*>(rowp + p.n_nope));
            if (p.n_nope > 256) sc1 = __ldg(reinterpret_cast<const float4*>(rowp + p.n_nope) + 1);
            if ((int)c * 8 < p.D - p.n_nope) rp = __ldg(reinterpret_cast<const uint4*>(rowp + p.rope_off) + c);
          }
          uint8_t* stg = sKV + (size_t)st * SB;
          const float scs[8] = {sc0.x, sc0.y, sc0.z, sc0.w, sc1.x, sc1.y, sc1.z, sc1.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int qc = (int)c + 8 * i;
            if (qc < nq) {
              uint4 lo, hi;
              // block qc/4 = 2i + (c >= 4): static indices, no local-memory array
              dequant16_e4m3(x[i], (c >= 4) ? scs[2 * i + 1] : scs[2 * i], lo, hi);
              const int a = qc >> 2, ch = 2 * (qc & 3);
              *reinterpret_cast<uint4*>(stg + stage_off<NK>(a, r, ch)) = lo;
              *reinterpret_cast<uint4*>(stg + stage_off<NK>(a, r, ch + 1)) = hi;
            }
          }
          *reinterpret_cast<uint4*>(stg + stage_off<NK>(p.n_nope >> 6, r, (int)c)) = rp;
          fence_proxy_async_smem();
          mbar_arrive(&ms->kv_full[st]);
          if (++st == (uint32_t)NST) {
            st = 0;
            kph ^= 1;
          }
          continue;
        }
        const uint32_t base = smem_u32(sKV + (size_t)st * SB) + dst_off;
        const __nv_bfloat16* src = (vld ? kv_row_ptr(p, b, row) : p.kv) + c * 8;
#pragma unroll
        for (int a = 0; a < kMaxAtoms; ++a) {
          if (a >= NA) break;
          if (a < p.na_tma) continue;
          const bool in = vld && a * 64 + (int)c * 8 < p.D;
          cp_async_16(base + a * NK * 128, in ? src + a * 64 : p.kv, in ? 16u : 0u);
        }
        cp_async_arrive_noinc(&ms->kv_full[st]);
        SI_TRACE_IF(tr, 0, ii, t, 2);
        if (++st == (uint32_t)NST) {
          st = 0;
          kph ^= 1;
        }
      }
    }
    cp_async_wait<0>();
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer: S = Q.K^T
    // P.V is issued by warp 16, so a P.V never waits behind a Q.K^T whose rows
    // are still in flight, and (a tcgen05.commit tracks only the issuing
    // thread's MMAs) an S completion never waits for a P.V.
    if (lane == 0) {
      const uint32_t idesc1 = umma_idesc_f16(kHeads, NK, MODE == kF16 ? 0 : 1);
      uint32_t st = 0, kph = 0;
      uint32_t sfr[2] = {0, 0};
      bool ok = true;
      int jj = 0;
      for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x, ++jj) {
#ifdef SI_ATTN_TRACE
        const int ii = (it - (int)blockIdx.x) / (int)gridDim.x;
#endif
        if (!mbar_wait(&ms->q_full[jj & 1], (uint32_t)(jj >> 1) & 1, abort_flag, p.status, kErrWaitQ)) break;
        tc_fence_after();
        for (int t = 0; t < ntiles; ++t) {
          SI_TRACE(1, ii, t, 0);
          if (!mbar_wait(&ms->kv_full[st], kph, abort_flag, p.status, kErrWaitTmaFull) ||
              !mbar_wait(&ms->s_free[t & 1], sfr[t & 1] ^ 1, abort_flag, p.status, kErrWaitAccEmpty)) {
            ok = false;
            break;
          }
          sfr[t & 1] ^= 1;
          // the KV tile was written by cp.async (generic proxy); order it
          // before the tensor core's (async proxy) reads
          fence_proxy_async_smem();
          tc_fence_after();
          const uint32_t kvbase = smem_u32(sKV + (size_t)st * SB);
          const uint32_t d_s = tmem + (16u << 16) + (t & 1) * NK;
          const uint32_t a_q = tmem + (16u << 16) + kQCol;
          for (int a = 0; a < NA; ++a) {
            const uint32_t a_col = a_q + (uint32_t)((jj * NA + a) % QSL) * 32;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              umma_f16_tmem_a(d_s, a_col + kk * 8, umma_desc_sw128(kvbase + a * NK * 128 + kk * 32), idesc1,
                              (a | kk) != 0);
            }
          }
          umma_commit(&ms->s_full[t & 1]);
          SI_TRACE(1, ii, t, 3);
          if (t == ntiles - 1) umma_commit(&ms->q_empty);
          if (++st == (uint32_t)NST) {
            st = 0;
            kph ^= 1;
          }
        }
      }
    }
  } else if (warp == 8 + kGatherWarps) {
    // ------------------------------------------------------------ UMMA issuer: O += P.V
    // Tile j's kv stage is released here: its Q.K^T completed before the
    // softmax published P, so this commit covers every read of the stage.
    if (lane == 0) {
      const uint32_t idesc2 = umma_idesc_f16(kHeads, NMMA, MODE == kF16 ? 0 : 1) | (1u << 16);  // B (V) MN-major
      const uint32_t idesc2x = umma_idesc_f16(kHeads, XV ? XV : 64, MODE == kF16 ? 0 : 1) | (1u << 16);
      uint32_t st = 0, pf[2] = {0, 0}, ofr = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
#ifdef SI_ATTN_TRACE
        const int ii = (it - (int)blockIdx.x) / (int)gridDim.x;
#endif
        for (int j = 0; j < ntiles; ++j) {
          if (!mbar_wait(&ms->p_full[j & 1], pf[j & 1], abort_flag, p.status, kErrWaitAccFull)) {
            ok = false;
            break;
          }
          pf[j & 1] ^= 1;
          SI_TRACE(1, ii, j, 4);
          if (j == 0) {
            if (!mbar_wait(&ms->o_free, ofr ^ 1, abort_flag, p.status, kErrWaitAccEmpty)) {
              ok = false;
              break;
            }
            ofr ^= 1;
          }
          tc_fence_after();
          const uint32_t pbase = smem_u32(sP + (j & 1) * NK * 128);
          const uint32_t vbase = smem_u32(sKV + (size_t)st * SB) + (p.dv_off / 64) * NK * 128;
#pragma unroll
          for (int kk = 0; kk < NK / 16; ++kk) {
            const uint64_t adesc = umma_desc(pbase + kk * 2048, 1024, 128, 0);
#pragma unroll
            for (int nh = 0; nh < NCH; ++nh) {
              const uint64_t bdesc = umma_desc(vbase + nh * (NMMA / 64) * NK * 128 + kk * 2048, NK * 128, 1024, 2);
              umma_f16(tmem + nh * NMMA, adesc, bdesc, idesc2, (j > 0 || kk > 0) ? 1u : 0u);
            }
            if (XV) {  // value columns [DV, DV+XV) into lanes 16-31
              const uint64_t bdesc = umma_desc(vbase + (DV / 64) * NK * 128 + kk * 2048, NK * 128, 1024, 2);
              umma_f16(tmem + (16u << 16) + (512 - XV), adesc, bdesc, idesc2x, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&ms->pv_done[j & 1]);
          umma_commit(&ms->kv_empty[st]);
          SI_TRACE(1, ii, j, 5);
          if (++st == (uint32_t)NST) st = 0;
        }
      }
    }
  } else {
    attn_softmax<NK, DVH, XV, MODE>(p, ms, sP, tmem, warp, lane, nitems, ntiles);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn
}  // namespace si

// ==================================================================== host side
namespace si {
namespace attn {

template <int DVH, int XV, int MODE>
static cudaError_t launch_t(const CUtensorMap& mq, const CUtensorMap& mkv, const Params& p, int grid,
                            cudaStream_t stream) {
  constexpr int NK = 32;
  static unsigned long long configured = 0;  // devices on which the attribute is set
  cudaError_t e = set_smem_attr_once(reinterpret_cast<const void*>(sparse_attn_fwd_kernel<NK, DVH, XV, MODE>), kSmemMax,
                                     &configured);
  if (e != cudaSuccess) return e;
  sparse_attn_fwd_kernel<NK, DVH, XV, MODE><<<grid, kThreads, smem_bytes<NK>(p.NA), stream>>>(mq, mkv, p);
  return cudaGetLastError();
}

template <int MODE>
static cudaError_t launch_m(const CUtensorMap& mq, const CUtensorMap& mkv, const Params& p, int grid,
                            cudaStream_t stream) {
  switch (p.Dv) {
    case 64: return launch_t<32, 0, MODE>(mq, mkv, p, grid, stream);
    case 128: return launch_t<64, 0, MODE>(mq, mkv, p, grid, stream);
    case 256: return launch_t<128, 0, MODE>(mq, mkv, p, grid, stream);
    case 512: return launch_t<256, 0, MODE>(mq, mkv, p, grid, stream);
    case 512 + kXV: return launch_t<256, kXV, MODE>(mq, mkv, p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

static cudaError_t launch(const CUtensorMap& mq, const CUtensorMap& mkv, const Params& p, int grid,
                          cudaStream_t stream) {
  if (p.fp8) return launch_m<kFp8Rows>(mq, mkv, p, grid, stream);
  if (p.f16) return launch_m<kF16>(mq, mkv, p, grid, stream);
  return launch_m<kBf16>(mq, mkv, p, grid, stream);
}

}  // namespace attn
}  // namespace si

#ifdef SI_ATTN_TRACE
static unsigned long long* g_attn_trace = nullptr;
extern "C" SI_API void si_debug_set_attn_trace(unsigned long long* t) { g_attn_trace = t; }
#endif

extern "C" {

}  // extern "C"

namespace si {
// Byte layout of one FP8 KV row (see Params::fp8).
struct Fp8RowLayout {
  int n_nope, rope_off, row_bytes;
};
static inline Fp8RowLayout fp8_row_layout(int D, int n_nope) {
  Fp8RowLayout l;
  l.n_nope = n_nope;
  l.rope_off = ((n_nope + 4 * (n_nope / 64)) + 15) / 16 * 16;
  l.row_bytes = ((l.rope_off + 2 * (D - n_nope)) + 15) / 16 * 16;
  return l;
}

static int run_sparse_attn(const void* q, const void* kv, int Nkv, const void* kv2, int Nkv2, const float* attn_sink,
                           const int32_t* topk_idxs, const int64_t* comp, int comp_k, int nwin, long long s_off,
                           int B, int S, int H, int D, int K, int Dv, float softmax_scale, void* o, float* lse,
                           void* ws, size_t ws_bytes, cudaStream_t stream, int fp8_n_nope = 0, int f16 = 0,
                           const long long* q_strides = nullptr) {
  if (Nkv2 < 0 || (Nkv2 > 0 && !kv2)) return fail("sparse_attn_fwd: bad second kv tensor");
  if (Nkv2 > 0 && (((uintptr_t)kv2) & 15)) return fail("sparse_attn_fwd: 16-byte alignment of kv2");
  const int Nkv1 = Nkv;
  Nkv = Nkv1 + Nkv2;
  if (!q || (Nkv1 > 0 && !kv) || !attn_sink || !o || !ws) return fail("sparse_attn_fwd: null pointer");
  if (K > 0 && !topk_idxs && !comp) return fail("sparse_attn_fwd: null topk_idxs");
  if (B < 1 || S < 0 || H < 1 || Nkv < 0 || K < 0) return fail("sparse_attn_fwd: bad sizes");
  if (D < 8 || D % 8 || D > attn::kQSlots * 64)
    return fail("sparse_attn_fwd: D must be a multiple of 8 in [8,%d] (got %d)", attn::kQSlots * 64, D);
  if (Dv < 64 || Dv % 64 || Dv > ((D + 63) / 64) * 64 || Dv > D)
    return fail("sparse_attn_fwd: Dv must be a multiple of 64 with Dv <= D (got Dv=%d, D=%d)", Dv, D);
  if ((((uintptr_t)q) | ((uintptr_t)kv) | ((uintptr_t)o)) & 15) return fail("sparse_attn_fwd: 16-byte alignment");
  if (ws_bytes < kStatusBytes) return fail("sparse_attn_fwd: workspace must hold at least 256 bytes");
  if ((long long)B * S * H + 64 >= (1ll << 31) || (long long)B * Nkv + 1 >= (1ll << 31))
    return fail("sparse_attn_fwd: sizes exceed the 2^31 TMA coordinate range");
  const int NA = (D + 63) / 64;
  if (!attn::q_fits_tmem(NA) || attn::num_stages<32>(NA) < 2)
    return fail("sparse_attn_fwd: D=%d too large (Q must fit in tensor memory: D <= %d)", D, attn::kQSlots * 64);
  int* status = reinterpret_cast<int*>(ws);
  if (cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream)) return fail_cuda("sparse_attn_fwd: status", e);
  if (S == 0) return 0;
  // No kv rows: every slot is masked (an index must be < Nkv), so the result is
  // the all-masked one (O = 0, LSE = sink) and nothing may be gathered.  The kv
  // tensor map then points at q, which the kernel never reads through it.
  if (Nkv == 0) K = 0;

  CUtensorMap mq, mkv;
  if (f16 && fp8_n_nope) return fail("sparse_attn_fwd: FP8 KV rows dequantise to bf16; q must be bf16");
  {
    // q as a 4-D [B,S,H,D] map (element strides q_strides = {b, s, h}, or contiguous)
    long long sb = (long long)S * H * D, ss = (long long)H * D, sh = D;
    if (q_strides) {
      sb = q_strides[0];
      ss = q_strides[1];
      sh = q_strides[2];
      if (sb < 0 || ss < 0 || sh < 0 || (sb | ss | sh) % 8)
        return fail("sparse_attn_fwd: q strides must be non-negative multiples of 8 elements");
    }
    const uint64_t qd[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)S, (uint64_t)B};
    const uint64_t qst[3] = {(uint64_t)sh * 2, (uint64_t)ss * 2, (uint64_t)sb * 2};
    const uint32_t qbx[4] = {64, (uint32_t)attn::kHeads, 1, 1};
    if (int rc = make_tmap_nd_16b(&mq, q, 4, qd, qst, qbx, f16 ? 1 : 0)) return rc;
  }
  if (fp8_n_nope) {
    if (fp8_n_nope % 64 || fp8_n_nope > 512 || D - fp8_n_nope <= 0 || D - fp8_n_nope > 64 || D % 8)
      return fail("sparse_attn_fwd_fp8kv: need n_nope a multiple of 64 in [64,512] and 0 < D - n_nope <= 64, "
                  "D %% 8 == 0 (got D=%d, n_nope=%d)", D, fp8_n_nope);
  }
  // FP8 rows are not bf16 tensors: the kv map (used only by TMA row gathers,
  // which are off for FP8 rows) then points at q like the empty-kv case.
  const void* kv_map_base = fp8_n_nope ? q : (Nkv1 > 0 ? kv : (Nkv2 > 0 ? kv2 : q));
  if (int rc = make_tmap_2d_16b(&mkv, kv_map_base, D,
                                (uint64_t)(fp8_n_nope ? 1 : B * (Nkv1 > 0 ? Nkv1 : (Nkv2 > 0 ? Nkv2 : 1))), 64, 1,
                                f16 ? 1 : 0))
    return rc;

  attn::Params p{};
  p.B = B; p.S = S; p.H = H; p.D = D; p.NA = NA; p.Nkv = Nkv; p.K = K;
  p.o_ld = Dv;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.idx = topk_idxs;
  p.f16 = f16;
  p.comp = K > 0 ? reinterpret_cast<const long long*>(comp) : nullptr;
  p.comp_k = comp_k;
  p.nwin = nwin;
  p.s_off = s_off;
  p.kv = reinterpret_cast<const __nv_bfloat16*>(kv);
  p.kv2 = reinterpret_cast<const __nv_bfloat16*>(kv2);
  // two atoms per row go through TMA gathers when kv is one tensor (measured best at D=576)
  p.na_tma = (Nkv2 > 0 || Nkv == 0 || fp8_n_nope) ? 0 : (NA >= 6 ? 2 : 0);
  if (fp8_n_nope) {
    const Fp8RowLayout l = fp8_row_layout(D, fp8_n_nope);
    p.fp8 = 1;
    p.n_nope = l.n_nope;
    p.rope_off = l.rope_off;
    p.row_bytes = l.row_bytes;
  }
  p.Nkv1 = Nkv1;
  p.sink = attn_sink;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_v8 = (((uintptr_t)o) & 31) == 0 && (Dv * 2) % 32 == 0;  // row stride Dv, column offsets multiples of 64
  p.status = status;
  p.hgroups = (H + attn::kHeads - 1) / attn::kHeads;
#ifdef SI_ATTN_TRACE
  p.trace = g_attn_trace;
#endif
  const long long items = (long long)B * S * p.hgroups;
  const int sms = device_sm_count();
  const int grid = (int)(items < sms ? items : sms);
  if (Dv == 512 + attn::kXV && NA <= attn::kQSlotsXV) {
    // full 576-wide output in one pass: O = 512 columns in lanes 0-15 + 64 in lanes 16-31
    p.Dv = Dv;
    p.dv_off = 0;
    p.o_off = 0;
    p.lse = lse;
    cudaError_t e = attn::launch(mq, mkv, p, grid, stream);
    if (e != cudaSuccess) return fail_cuda("sparse_attn_fwd: kernel launch", e);
    return 0;
  }
  // other widths: value columns in passes of 512 / 256 / 128 / 64 (TMEM holds at most 512 fp32 columns)
  int done = 0;
  while (done < Dv) {
    int pass = 512;
    while (pass > Dv - done) pass >>= 1;
    p.Dv = pass;
    p.dv_off = done;
    p.o_off = done;
    p.lse = done == 0 ? lse : nullptr;
    cudaError_t e = attn::launch(mq, mkv, p, grid, stream);
    if (e != cudaSuccess) return fail_cuda("sparse_attn_fwd: kernel launch", e);
    done += pass;
  }
  return 0;
}

}  // namespace si

extern "C" {

int si_sparse_attn_fwd_kv2(const void* q, const void* kv, int Nkv, const void* kv2, int Nkv2, const float* attn_sink,
                           const int32_t* topk_idxs, int B, int S, int H, int D, int K, int Dv, float softmax_scale,
                           void* o, float* lse, void* ws, size_t ws_bytes, cudaStream_t stream) {
  return si::run_sparse_attn(q, kv, Nkv, kv2, Nkv2, attn_sink, topk_idxs, nullptr, 0, 0, 0, B, S, H, D, K, Dv,
                             softmax_scale, o, lse, ws, ws_bytes, stream);
}

int si_csa_sparse_attn_fwd(const void* q, const void* kv, int S_total, const void* kv_comp, int T,
                           const float* attn_sink, const int64_t* comp_idx, int top_k, int n_win, long long s_offset,
                           int B, int S, int H, int D, int Dv, float softmax_scale, void* o, float* lse, void* ws,
                           size_t ws_bytes, cudaStream_t stream) {
  using namespace si;
  if (n_win < 0 || top_k < 0) return fail("csa_sparse_attn_fwd: n_win and top_k must be >= 0");
  if (top_k > 0 && !comp_idx) return fail("csa_sparse_attn_fwd: null comp_idx");
  if (s_offset < 0 || s_offset + S > S_total)
    return fail("csa_sparse_attn_fwd: query slice [%lld, %lld) outside the sequence of %d tokens", s_offset,
                s_offset + S, S_total);
  if ((long long)n_win + top_k >= (1ll << 30)) return fail("csa_sparse_attn_fwd: n_win + top_k too large");
  return run_sparse_attn(q, kv, S_total, kv_comp, T, attn_sink, nullptr, comp_idx, top_k, n_win, s_offset, B, S, H,
                         D, n_win + top_k, Dv, softmax_scale, o, lse, ws, ws_bytes, stream);
}

int si_fp8_kv_row_bytes(int D, int n_nope) {
  if (n_nope <= 0 || n_nope % 64 || D <= n_nope) return -1;
  return si::fp8_row_layout(D, n_nope).row_bytes;
}

int si_sparse_attn_fwd_fp8kv(const void* q, const void* kv_rows, int Nkv, const void* kv2_rows, int Nkv2, int n_nope,
                             const float* attn_sink, const int32_t* topk_idxs, int B, int S, int H, int D, int K,
                             int Dv, float softmax_scale, void* o, float* lse, void* ws, size_t ws_bytes,
                             cudaStream_t stream) {
  if (n_nope <= 0) return si::fail("sparse_attn_fwd_fp8kv: n_nope must be > 0");
  return si::run_sparse_attn(q, kv_rows, Nkv, kv2_rows, Nkv2, attn_sink, topk_idxs, nullptr, 0, 0, 0, B, S, H, D, K,
                             Dv, softmax_scale, o, lse, ws, ws_bytes, stream, n_nope);
}

int si_sparse_attn_fwd_ex(const void* q, const void* kv, int Nkv, const void* kv2, int Nkv2, const float* attn_sink,
                          const int32_t* topk_idxs, int B, int S, int H, int D, int K, int Dv, float softmax_scale,
                          int dtype, void* o, float* lse, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (dtype != 0 && dtype != 1) return si::fail("sparse_attn_fwd: dtype must be 0 (bf16) or 1 (fp16), got %d", dtype);
  return si::run_sparse_attn(q, kv, Nkv, kv2, Nkv2, attn_sink, topk_idxs, nullptr, 0, 0, 0, B, S, H, D, K, Dv,
                             softmax_scale, o, lse, ws, ws_bytes, stream, 0, dtype);
}

int si_sparse_attn_fwd_strided(const void* q, const long long* q_strides, const void* kv, int Nkv, const void* kv2,
                               int Nkv2, const float* attn_sink, const int32_t* topk_idxs, int B, int S, int H, int D,
                               int K, int Dv, float softmax_scale, int dtype, void* o, float* lse, void* ws,
                               size_t ws_bytes, cudaStream_t stream) {
  if (dtype != 0 && dtype != 1) return si::fail("sparse_attn_fwd: dtype must be 0 (bf16) or 1 (fp16), got %d", dtype);
  return si::run_sparse_attn(q, kv, Nkv, kv2, Nkv2, attn_sink, topk_idxs, nullptr, 0, 0, 0, B, S, H, D, K, Dv,
                             softmax_scale, o, lse, ws, ws_bytes, stream, 0, dtype, q_strides);
}

int si_sparse_attn_fwd(const void* q, const void* kv, const float* attn_sink, const int32_t* topk_idxs, int B, int S,
                       int H, int D, int Nkv, int K, int Dv, float softmax_scale, void* o, float* lse, void* ws,
                       size_t ws_bytes, cudaStream_t stream) {
  return si_sparse_attn_fwd_kv2(q, kv, Nkv, nullptr, 0, attn_sink, topk_idxs, B, S, H, D, K, Dv, softmax_scale, o, lse,
                                ws, ws_bytes, stream);
}

}  // extern "C"
