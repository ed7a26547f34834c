// Sparse MQA attention backward with attention sink.
//
// Math (flash_sparse/triton/sparse_attn_bwd.py:1-30, the sink-augmented
// softmax of flash_sparse/reference.py:44-130; K and V share the kv rows):
//   p[h,j]   = exp(scale * q[h].kv[j] - lse[h])            (lse from the forward)
//   delta[h] = sum_d o[h,d] * do[h,d]
//   dp[h,j]  = p[h,j] * (do[h] . kv[j,:Dv] - delta[h]) * scale
//   dq[h]    = sum_j dp[h,j] * kv[j]
//   dkv[j]  += sum_{queries, h} dp[h,j] * q[h]  +  p[h,j] * do[h]   (value part: first Dv dims)
//   dsink[h] = -sum_queries exp(sink[h] - lse[h]) * delta[h]
// As in the reference, p and dp enter the products rounded to the operand type.
//
// Mapping.  A work item is one query (b, s) and a group of 64 heads (four
// m16 tiles of the warp-level bf16 MMA, mma.sync m16n8k16), so every selected
// kv row is gathered once per query and its dkv contribution is summed over
// all 64 heads before it reaches global memory.  16 warps; the rows of tile
// t+1 are gathered (cp.async, masked slots zero-filled) while tile t computes:
//   1. S and dO.V^T: warp w owns heads 16*(w%4).. and keys 8*(w/4)..; p and dp
//      in registers, written to shared memory in bf16;
//   2. dq[64 x D] += dp . kv: warp w owns 16 heads x D/4 columns,
//      accumulated in registers across all tiles of the item;
//   3. dkv[32 x D] = dp^T . q + p^T . do (contraction over the 64 heads):
//      warp w owns 16 keys x D/8 columns; each value is added to the fp32 dkv
//      buffer with a 16-byte vector reduction (red.global.add.v4.f32: lane
//      pairs swap half rows so each lane holds four consecutive columns of one
//      row; the buffer is L2-resident at the benchmark sizes).
// The backward runs on the warp-level MMA path; the forward is the tcgen05
// kernel.
#include <cuda_bf16.h>

#include "capi_common.h"
#include "ptx.cuh"
#include "../../include/streamindex_b200.h"

namespace si {
namespace attn_bwd {

constexpr int kHeads = 64;   // heads per work item (4 m16 tiles)
constexpr int kKeys = 32;    // keys per tile
constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxSmem = 232448;

struct Params {
  int B, S, H, D, Dv, Nkv, K;
  float scale;
  const __nv_bfloat16 *q, *kv, *o, *dout;
  const float *lse, *sink;
  const int* idx;
  __nv_bfloat16* dq;
  float* dkv;    // [B,Nkv,D] fp32, zeroed by the caller
  float* dsink;  // [H] fp32, zeroed by the caller
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
// C[16x8] += A[16x16] . B[16x8], bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// 32 TMEM lanes x 8 fp32 columns (thread i: lane base + i), load + wait in one asm.
__device__ __forceinline__ void tmem_ld8_sync(uint32_t taddr, float (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

__host__ __device__ inline int row_elems(int n) { return n + 8; }  // +16 B per row: conflict-free ldmatrix

__host__ __device__ inline size_t smem_bytes(int D, int Dv, int nst) {
  return (size_t)2 * (kHeads * row_elems(D) + kHeads * row_elems(Dv) + (size_t)nst * kKeys * row_elems(D) +
                      2 * kHeads * row_elems(kKeys)) +
         sizeof(float) * 2 * kHeads + sizeof(int) * 2 * kKeys + 64 + 16;
}
// Two kv stages (the next tile's gather overlaps this tile's math) when they fit.
__host__ __device__ inline int kv_stages(int D, int Dv) { return smem_bytes(D, Dv, 2) <= (size_t)kMaxSmem ? 2 : 1; }

// NT = D / 32: n8 tiles of a warp's dq columns (D/4); D/64 of its dkv columns (D/8).
template <int NT>
__global__ void __launch_bounds__(kThreads, 1) sparse_attn_bwd_kernel(Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int NTK = NT / 2;
  const int D = p.D, Dv = p.Dv;
  const int LQ = row_elems(D), LO = row_elems(Dv), LP = row_elems(kKeys);
  const int nst = kv_stages(D, Dv);
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sDO = sQ + kHeads * LQ;
  __nv_bfloat16* sKV = sDO + kHeads * LO;
  __nv_bfloat16* sP = sKV + nst * kKeys * LQ;
  __nv_bfloat16* sDS = sP + kHeads * LP;
  float* sLse = reinterpret_cast<float*>(sDS + kHeads * LP);
  float* sDelta = sLse + kHeads;
  int* sIdx = reinterpret_cast<int*>(sDelta + kHeads);  // [2][kKeys]
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sIdx + 2 * kKeys);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int hm = warp & 3;   // head tile of phases 1 and 2
  const int hgroups = (p.H + kHeads - 1) / kHeads;
  const long long nitems = (long long)p.B * p.S * hgroups;
  const int ntiles = (p.K + kKeys - 1) / kKeys;
  const int chunks = D / 8;  // 16-byte chunks per kv / q row
  // dq lives in tensor memory between tiles (72 fp32 per thread at D=576 would
  // otherwise pin registers the three products need): warp w owns lanes
  // 32*(w%4).., columns (w/4)*4*NT.., one column per fp32 value of its
  // m16n8 fragments (tile j at columns 4j..4j+3).
  // The C warps (8..15) park their dkv tile there too, columns 16*NT + ((w-8)/4)*4*NT.
  constexpr uint32_t kTmemCols = NT * 24 <= 32 ? 32 : NT * 24 <= 64 ? 64 : NT * 24 <= 128 ? 128 : NT * 24 <= 256 ? 256 : 512;
  if (warp == 0) {
    tmem_alloc(sTmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tdq = *sTmem + ((uint32_t)(32 * hm) << 16) + (uint32_t)((warp >> 2) * 4 * NT);
  const uint32_t tkv = *sTmem + ((uint32_t)(32 * hm) << 16) + (uint32_t)(16 * NT + (((warp - 8) >> 2) & 1) * 4 * NT);

  // cp.async of one tile's kv rows into a stage, indices read from global memory
  auto gather = [&](const int* irow, int b, int t, __nv_bfloat16* stage, int* sidx) {
    if (tid < kKeys) {
      const int kk = t * kKeys + tid;
      const int v = kk < p.K ? irow[kk] : -1;
      sidx[tid] = (v >= 0 && v < p.Nkv) ? v : -1;
    }
    for (int i = tid; i < kKeys * chunks; i += kThreads) {
      const int r = i / chunks, c = i % chunks;
      const int kk = t * kKeys + r;
      int v = kk < p.K ? __ldg(irow + kk) : -1;
      v = (v >= 0 && v < p.Nkv) ? v : -1;
      const __nv_bfloat16* src = v >= 0 ? p.kv + ((size_t)b * p.Nkv + v) * D + c * 8 : p.kv;
      cp_async_16(smem_u32(stage + r * LQ + c * 8), src, v >= 0 ? 16u : 0u);
    }
  };

  for (long long it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int hg = (int)(it % hgroups);
    const long long bs = it / hgroups;
    const int b = (int)(bs / p.S);
    const int h0 = hg * kHeads;
    const int* irow = p.idx + (size_t)bs * p.K;
    __syncthreads();  // the previous item is done with every shared tile
    // ---- q, do rows of the 64 heads (zero rows past H)
    for (int i = tid; i < kHeads * chunks; i += kThreads) {
      const int r = i / chunks, c = i % chunks;
      const bool ok = h0 + r < p.H;
      cp_async_16(smem_u32(sQ + r * LQ + c * 8), ok ? p.q + ((size_t)bs * p.H + h0 + r) * D + c * 8 : p.q, ok ? 16u : 0u);
    }
    for (int i = tid; i < kHeads * (Dv / 8); i += kThreads) {
      const int r = i / (Dv / 8), c = i % (Dv / 8);
      const bool ok = h0 + r < p.H;
      cp_async_16(smem_u32(sDO + r * LO + c * 8), ok ? p.dout + ((size_t)bs * p.H + h0 + r) * Dv + c * 8 : p.dout,
                  ok ? 16u : 0u);
    }
    cp_async_commit();
    if (nst == 2) gather(irow, b, 0, sKV, sIdx);
    cp_async_commit();
    // ---- delta = o . do, lse and dsink: four heads per warp (o read from global memory)
#pragma unroll 1
    for (int r = warp; r < kHeads; r += kWarps) {
      const int h = h0 + r;
      float acc = 0.f;
      if (h < p.H) {
        const __nv_bfloat16* orow = p.o + ((size_t)bs * p.H + h) * Dv;
        const __nv_bfloat16* drow = p.dout + ((size_t)bs * p.H + h) * Dv;
        for (int d = lane * 8; d < Dv; d += 256) {
          const uint4 ov = *reinterpret_cast<const uint4*>(orow + d);
          const uint4 dv = *reinterpret_cast<const uint4*>(drow + d);
          const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
          const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 a = __bfloat1622float2(o2[e]), c = __bfloat1622float2(d2[e]);
            acc += a.x * c.x + a.y * c.y;
          }
        }
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
      if (lane == 0) {
        const float lse = h < p.H ? p.lse[(size_t)bs * p.H + h] : 0.f;
        sDelta[r] = acc;
        sLse[r] = lse;
        if (h < p.H) atomicAdd(p.dsink + h, -expf(p.sink[h] - lse) * acc);
      }
    }

    // dkv of the previous tile, parked in tensor memory by the C warps (8..15)
    // until the next tile's phase 1 runs, so its global reductions overlap that phase
    float* cdst = nullptr;
    bool pending = false;
    const bool codd = t4 & 1;
    // even lanes (t4 = 0, 2) add row k0, columns 2*t4 .. 2*t4+3; odd lanes add
    // row k0+8, columns 2*(t4-1) .. +3 (each lane takes its partner's half)
    auto flush_dkv = [&]() {
      if (!pending) return;
      pending = false;
#pragma unroll 3
      for (int j2 = 0; j2 < NT; j2 += 2) {
        float v[8];
        tmem_ld8_sync(tkv + 4 * j2, v);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float* c = v + 4 * h;
          const float s0 = codd ? c[0] : c[2], s1 = codd ? c[1] : c[3];
          const float r0 = __shfl_xor_sync(0xffffffffu, s0, 1), r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
          if (cdst) {
            if (codd)
              red_add_v4(cdst + (j2 + h) * 8, r0, r1, c[2], c[3]);
            else
              red_add_v4(cdst + (j2 + h) * 8, c[0], c[1], r0, r1);
          }
        }
      }
    };

#pragma unroll 1
    for (int t = 0; t < ntiles; ++t) {
      __nv_bfloat16* stage = sKV + (nst == 2 ? (t & 1) : 0) * kKeys * LQ;
      const int* sid = sIdx + (nst == 2 ? (t & 1) : 0) * kKeys;
      if (nst == 2) {
        if (t + 1 < ntiles) gather(irow, b, t + 1, sKV + ((t + 1) & 1) * kKeys * LQ, sIdx + ((t + 1) & 1) * kKeys);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        gather(irow, b, t, stage, sIdx);
        cp_async_commit();
        cp_async_wait<0>();
      }
      __syncthreads();  // tile t (and, at t = 0, q / do / delta) visible to all warps

      if (warp < 8) {
        // ---- 1. S and dO.V^T for heads 16*hm.., keys 16*(warp/4).. (two n8 tiles);
        // S over D and dO.V^T over Dv share the kv fragments of each k step
        const int kq = warp >> 2;
        float s[2][4], dp[2][4];
#pragma unroll
        for (int e = 0; e < 4; ++e) s[0][e] = s[1][e] = dp[0][e] = dp[1][e] = 0.f;
        const uint32_t a_q = smem_u32(sQ + (hm * 16 + (lane & 15)) * LQ + (lane >> 4) * 8);
        const uint32_t a_o = smem_u32(sDO + (hm * 16 + (lane & 15)) * LO + (lane >> 4) * 8);
        const uint32_t b_kv = smem_u32(stage + (kq * 16 + (lane & 7) + (lane >> 4) * 8) * LQ + ((lane >> 3) & 1) * 8);
#pragma unroll 4
        for (int k = 0; k < Dv / 16; ++k) {
          uint32_t a[4], c[4], bb[4];
          ldsm_x4(b_kv + k * 32, bb);
          ldsm_x4(a_q + k * 32, a);
          ldsm_x4(a_o + k * 32, c);
          mma16816(s[0], a, bb[0], bb[1]);
          mma16816(s[1], a, bb[2], bb[3]);
          mma16816(dp[0], c, bb[0], bb[1]);
          mma16816(dp[1], c, bb[2], bb[3]);
        }
#pragma unroll 4
        for (int k = Dv / 16; k < D / 16; ++k) {  // the q.k dims past Dv
          uint32_t a[4], bb[4];
          ldsm_x4(b_kv + k * 32, bb);
          ldsm_x4(a_q + k * 32, a);
          mma16816(s[0], a, bb[0], bb[1]);
          mma16816(s[1], a, bb[2], bb[3]);
        }
        // thread values: heads 16*hm + g (+8); keys 16*kq + 8*nt + 2*t4 (+1)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int c0 = kq * 16 + nt * 8 + 2 * t4;
          const bool v0 = sid[c0] >= 0, v1 = sid[c0 + 1] >= 0;
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int r = hm * 16 + g + 8 * hr;
            const bool hv = h0 + r < p.H;
            const float lse = sLse[r], dl = sDelta[r];
            const float p0 = (hv && v0) ? expf(s[nt][2 * hr] * p.scale - lse) : 0.f;
            const float p1 = (hv && v1) ? expf(s[nt][2 * hr + 1] * p.scale - lse) : 0.f;
            const float d0 = p0 * (dp[nt][2 * hr] - dl) * p.scale;
            const float d1 = p1 * (dp[nt][2 * hr + 1] - dl) * p.scale;
            *reinterpret_cast<uint32_t*>(sP + r * LP + c0) = pack_bf16x2(p0, p1);
            *reinterpret_cast<uint32_t*>(sDS + r * LP + c0) = pack_bf16x2(d0, d1);
          }
        }
      } else {
        flush_dkv();  // the previous tile's dkv reductions
      }
      __syncthreads();

      // ---- 2. dq += dS . kv  (A = dS [16 heads x 32 keys], B = kv [32 keys x D/4] via trans loads),
      // two n8 tiles at a time through tensor memory
      {
        const int col0 = (warp >> 2) * (D / 4);
        uint32_t a0[4], a1[4];
        ldsm_x4(smem_u32(sDS + (hm * 16 + (lane & 15)) * LP + (lane >> 4) * 8), a0);
        ldsm_x4(smem_u32(sDS + (hm * 16 + (lane & 15)) * LP + 16 + (lane >> 4) * 8), a1);
        const uint32_t b0 = smem_u32(stage + (lane & 15) * LQ + col0 + (lane >> 4) * 8);
        const uint32_t b1 = b0 + 16 * LQ * 2;
#pragma unroll 3
        for (int j = 0; j < NT; j += 2) {
          float v[8];
          if (t == 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = 0.f;
          } else {
            tmem_ld8_sync(tdq + 4 * j, v);
          }
          float(&c0)[4] = *reinterpret_cast<float(*)[4]>(v);
          float(&c1)[4] = *reinterpret_cast<float(*)[4]>(v + 4);
          uint32_t bb[4], bc[4];
          ldsm_x4_t(b0 + j * 16, bb);
          ldsm_x4_t(b1 + j * 16, bc);
          mma16816(c0, a0, bb[0], bb[1]);
          mma16816(c1, a0, bb[2], bb[3]);
          mma16816(c0, a1, bc[0], bc[1]);
          mma16816(c1, a1, bc[2], bc[3]);
          tmem_st8(tdq + 4 * j, v);
        }
        tmem_st_wait();
      }
      if (warp >= 8) {
        // ---- 3. dkv[16 keys x D/4] = dS^T . q + P^T . do, contraction over the 64 heads
        const int c = warp - 8, km = c & 1, colc = (c >> 1) * (D / 4);
        const int arow = (lane >> 4) * 8 + (lane & 7), acol = km * 16 + ((lane >> 3) & 1) * 8;
        float cacc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) cacc[j][0] = cacc[j][1] = cacc[j][2] = cacc[j][3] = 0.f;
#pragma unroll
        for (int kh = 0; kh < kHeads / 16; ++kh) {
          // A = X^T with X [16 heads x 16 keys]: transposed 8x8 blocks
          uint32_t ads[4], ap[4];
          ldsm_x4_t(smem_u32(sDS + (kh * 16 + arow) * LP + acol), ads);
          ldsm_x4_t(smem_u32(sP + (kh * 16 + arow) * LP + acol), ap);
          const uint32_t bq = smem_u32(sQ + (kh * 16 + (lane & 15)) * LQ + colc + (lane >> 4) * 8);
          const uint32_t bo = smem_u32(sDO + (kh * 16 + (lane & 15)) * LO + colc + (lane >> 4) * 8);
#pragma unroll
          for (int j = 0; j < NT; j += 2) {
            uint32_t bb[4];
            ldsm_x4_t(bq + j * 16, bb);
            mma16816(cacc[j], ads, bb[0], bb[1]);
            mma16816(cacc[j + 1], ads, bb[2], bb[3]);
            if (colc + j * 8 < Dv) {
              ldsm_x4_t(bo + j * 16, bb);
              mma16816(cacc[j], ap, bb[0], bb[1]);
              mma16816(cacc[j + 1], ap, bb[2], bb[3]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < NT; j += 2) tmem_st8(tkv + 4 * j, *reinterpret_cast<float(*)[8]>(&cacc[j][0]));
        tmem_st_wait();
        const int v = sid[km * 16 + g + (codd ? 8 : 0)];
        cdst = v >= 0 ? p.dkv + ((size_t)b * p.Nkv + v) * D + colc + 2 * (t4 & ~1) : nullptr;
        pending = true;
      }
      __syncthreads();  // stage t and sP / sDS free for the next tile
    }
    if (warp >= 8) flush_dkv();
    // ---- dq out (heads 16*hm + g (+8); columns col0 + 8j + 2*t4)
    const int col0 = (warp >> 2) * (D / 4);
#pragma unroll 1
    for (int j = 0; j < NT; j += 2) {
      float v[8];
      if (ntiles > 0) {
        tmem_ld8_sync(tdq + 4 * j, v);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int h = h0 + hm * 16 + g + 8 * hr;
        if (h >= p.H) continue;
        __nv_bfloat16* drow = p.dq + ((size_t)bs * p.H + h) * D + col0 + 2 * t4;
        *reinterpret_cast<uint32_t*>(drow + j * 8) = pack_bf16x2(v[2 * hr], v[2 * hr + 1]);
        *reinterpret_cast<uint32_t*>(drow + j * 8 + 8) = pack_bf16x2(v[4 + 2 * hr], v[4 + 2 * hr + 1]);
      }
    }
  }
  cp_async_wait<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*sTmem, kTmemCols);
  }
}

template <int NT>
static cudaError_t launch_nt(const Params& p, int grid, cudaStream_t stream) {
  const size_t smem = smem_bytes(p.D, p.Dv, kv_stages(p.D, p.Dv));
  static unsigned long long configured = 0;
  cudaError_t e = set_smem_attr_once(reinterpret_cast<const void*>(sparse_attn_bwd_kernel<NT>), (int)smem, &configured);
  if (e != cudaSuccess) return e;
  sparse_attn_bwd_kernel<NT><<<grid, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace attn_bwd
}  // namespace si

extern "C" {

int si_sparse_attn_bwd(const void* q, const void* kv, const float* attn_sink, const int32_t* topk_idxs, const void* o,
                       const float* lse, const void* dout, int B, int S, int H, int D, int Nkv, int K, int Dv,
                       float softmax_scale, void* dq, float* dkv_f32, float* dsink, cudaStream_t stream) {
  using namespace si;
  if (!q || !kv || !attn_sink || !o || !lse || !dout || !dq || !dkv_f32 || !dsink)
    return fail("sparse_attn_bwd: null pointer");
  if (K > 0 && !topk_idxs) return fail("sparse_attn_bwd: null topk_idxs");
  if (B < 1 || S < 0 || H < 1 || Nkv < 0 || K < 0) return fail("sparse_attn_bwd: bad sizes");
  if (Dv < 32 || Dv % 32 || Dv > D) return fail("sparse_attn_bwd: Dv must be a multiple of 32 with Dv <= D (got %d)", Dv);
  if ((((uintptr_t)q) | ((uintptr_t)kv) | ((uintptr_t)o) | ((uintptr_t)dout) | ((uintptr_t)dq) | ((uintptr_t)dkv_f32)) &
      15)
    return fail("sparse_attn_bwd: 16-byte alignment");
  if (S == 0 || K == 0) return 0;  // dq = 0 must be set by the caller when K == 0
  attn_bwd::Params p{};
  p.B = B; p.S = S; p.H = H; p.D = D; p.Dv = Dv; p.Nkv = Nkv; p.K = K;
  p.scale = softmax_scale;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.kv = reinterpret_cast<const __nv_bfloat16*>(kv);
  p.o = reinterpret_cast<const __nv_bfloat16*>(o);
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout);
  p.lse = lse;
  p.sink = attn_sink;
  p.idx = topk_idxs;
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq);
  p.dkv = dkv_f32;
  p.dsink = dsink;
  const long long items = (long long)B * S * ((H + attn_bwd::kHeads - 1) / attn_bwd::kHeads);
  const long long cap = (long long)device_sm_count();
  const int grid = (int)(items < cap ? items : cap);
  cudaError_t e;
  switch (D) {
    case 64: e = attn_bwd::launch_nt<2>(p, grid, stream); break;
    case 128: e = attn_bwd::launch_nt<4>(p, grid, stream); break;
    case 256: e = attn_bwd::launch_nt<8>(p, grid, stream); break;
    case 512: e = attn_bwd::launch_nt<16>(p, grid, stream); break;
    case 576: e = attn_bwd::launch_nt<18>(p, grid, stream); break;
    default: return fail("sparse_attn_bwd: D must be 64, 128, 256, 512 or 576 (got %d)", D);
  }
  return e == cudaSuccess ? 0 : fail_cuda("sparse_attn_bwd: launch", e);
}

}  // extern "C"
