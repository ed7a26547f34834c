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
// Mapping.  A work item is one query (b, s) and a group of 16 heads (the M of
// the warp-level bf16 MMA, mma.sync m16n8k16).  Four warps; per 32-key tile:
//   1. the tile's kv rows are gathered into shared memory (cp.async; masked
//      slots zero-filled);
//   2. warp w computes S and dO.V^T for keys [8w, 8w+8) (K = D and Dv), then
//      p and dp in registers, written to shared memory in bf16;
//   3. dq[16 x D] += dp . kv: warp w owns D/4 columns, accumulated in registers
//      across all tiles of the item;
//   4. dkv[32 x D] = dp^T . q + p^T . do: warp w owns D/4 columns; each value
//      is added to the fp32 dkv buffer with a 16-byte vector reduction
//      (red.global.add.v4.f32: lane pairs swap half rows so each lane holds
//      four consecutive columns of one row; the buffer is L2-resident at the
//      benchmark sizes).
// This is a correctness-first kernel on the warp-level MMA path (the reference
// backward is forward-only territory for the north star); the forward is the
// tcgen05 kernel.
#include <cuda_bf16.h>

#include "capi_common.h"
#include "ptx.cuh"
#include "../../include/streamindex_b200.h"

namespace si {
namespace attn_bwd {

constexpr int kHeads = 16;   // MMA M
constexpr int kKeys = 32;    // keys per tile
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;

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
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__host__ __device__ inline int row_elems(int n) { return n + 8; }  // +16 B per row: conflict-free ldmatrix

__host__ __device__ inline size_t smem_bytes(int D, int Dv) {
  return (size_t)2 * (kHeads * row_elems(D) + kHeads * row_elems(Dv) + kKeys * row_elems(D) +
                      2 * kHeads * row_elems(kKeys)) +
         sizeof(float) * 2 * kHeads + sizeof(int) * kKeys + 64;
}

// NT = D / 32: n8 tiles per warp over its quarter of the D columns.
template <int NT>
__global__ void __launch_bounds__(kThreads) sparse_attn_bwd_kernel(Params p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int D = p.D, Dv = p.Dv;
  const int LQ = row_elems(D), LO = row_elems(Dv), LP = row_elems(kKeys);
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sDO = sQ + kHeads * LQ;
  __nv_bfloat16* sKV = sDO + kHeads * LO;
  __nv_bfloat16* sP = sKV + kKeys * LQ;
  __nv_bfloat16* sDS = sP + kHeads * LP;
  float* sLse = reinterpret_cast<float*>(sDS + kHeads * LP);
  float* sDelta = sLse + kHeads;
  int* sIdx = reinterpret_cast<int*>(sDelta + kHeads);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int hgroups = (p.H + kHeads - 1) / kHeads;
  const long long nitems = (long long)p.B * p.S * hgroups;
  const int ntiles = (p.K + kKeys - 1) / kKeys;
  const int CW = D / 4;  // columns per warp (NT n8 tiles)

  for (long long it = blockIdx.x; it < nitems; it += gridDim.x) {
    const int hg = (int)(it % hgroups);
    const long long bs = it / hgroups;
    const int b = (int)(bs / p.S);
    const int h0 = hg * kHeads;
    // ---- q, do rows of the 16 heads (zero rows past H), lse, delta, dsink
    for (int i = tid; i < kHeads * (D / 8); i += kThreads) {
      const int r = i / (D / 8), c = i % (D / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (h0 + r < p.H) v = *reinterpret_cast<const uint4*>(p.q + ((size_t)bs * p.H + h0 + r) * D + c * 8);
      *reinterpret_cast<uint4*>(sQ + r * LQ + c * 8) = v;
    }
    for (int i = tid; i < kHeads * (Dv / 8); i += kThreads) {
      const int r = i / (Dv / 8), c = i % (Dv / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (h0 + r < p.H) v = *reinterpret_cast<const uint4*>(p.dout + ((size_t)bs * p.H + h0 + r) * Dv + c * 8);
      *reinterpret_cast<uint4*>(sDO + r * LO + c * 8) = v;
    }
#pragma unroll 1
    for (int r = warp; r < kHeads; r += kWarps) {  // delta: one warp per head row
      const int h = h0 + r;
      float acc = 0.f;
      if (h < p.H) {
        const __nv_bfloat16* orow = p.o + ((size_t)bs * p.H + h) * Dv;
        const __nv_bfloat16* drow = p.dout + ((size_t)bs * p.H + h) * Dv;
        for (int d = lane; d < Dv; d += 32) acc += __bfloat162float(orow[d]) * __bfloat162float(drow[d]);
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

    float dq[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) dq[j][0] = dq[j][1] = dq[j][2] = dq[j][3] = 0.f;

    const int* irow = p.idx + (size_t)bs * p.K;
#pragma unroll 1
    for (int t = 0; t < ntiles; ++t) {
      __syncthreads();  // previous tile's shared tiles are free; q/do/lse/delta visible
      if (tid < kKeys) {
        const int kk = t * kKeys + tid;
        const int v = kk < p.K ? irow[kk] : -1;
        sIdx[tid] = (v >= 0 && v < p.Nkv) ? v : -1;
      }
      __syncthreads();
      for (int i = tid; i < kKeys * (D / 8); i += kThreads) {
        const int r = i / (D / 8), c = i % (D / 8);
        const int v = sIdx[r];
        const __nv_bfloat16* src = v >= 0 ? p.kv + ((size_t)b * p.Nkv + v) * D + c * 8 : p.kv;
        cp_async_16(smem_u32(sKV + r * LQ + c * 8), src, v >= 0 ? 16u : 0u);
      }
      cp_async_commit();
      cp_async_wait<0>();
      __syncthreads();

      // ---- S and dO.V^T for keys [8w, 8w+8)
      {
        float s[4] = {0.f, 0.f, 0.f, 0.f}, dpv[4] = {0.f, 0.f, 0.f, 0.f};
        const int n0 = 8 * warp;
        const uint32_t a_q = smem_u32(sQ + (lane & 15) * LQ + (lane >> 4) * 8);
        const uint32_t a_o = smem_u32(sDO + (lane & 15) * LO + (lane >> 4) * 8);
        const uint32_t b_kv = smem_u32(sKV + (n0 + (lane & 7)) * LQ + ((lane >> 3) & 1) * 8);
#pragma unroll 4
        for (int k = 0; k < D / 16; ++k) {
          uint32_t a[4], bb[2];
          ldsm_x4(a_q + k * 32, a);
          ldsm_x2(b_kv + k * 32, bb);
          mma16816(s, a, bb);
        }
#pragma unroll 4
        for (int k = 0; k < Dv / 16; ++k) {
          uint32_t a[4], bb[2];
          ldsm_x4(a_o + k * 32, a);
          ldsm_x2(b_kv + k * 32, bb);
          mma16816(dpv, a, bb);
        }
        // thread values: heads g, g+8; keys n0 + 2*t4, +1
        const int c0 = n0 + 2 * t4;
        const bool v0 = sIdx[c0] >= 0, v1 = sIdx[c0 + 1] >= 0;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int r = g + 8 * hr;
          const bool hv = h0 + r < p.H;
          const float lse = sLse[r], dl = sDelta[r];
          const float p0 = (hv && v0) ? expf(s[2 * hr] * p.scale - lse) : 0.f;
          const float p1 = (hv && v1) ? expf(s[2 * hr + 1] * p.scale - lse) : 0.f;
          const float d0 = p0 * (dpv[2 * hr] - dl) * p.scale;
          const float d1 = p1 * (dpv[2 * hr + 1] - dl) * p.scale;
          *reinterpret_cast<uint32_t*>(sP + r * LP + c0) = pack_bf16x2(p0, p1);
          *reinterpret_cast<uint32_t*>(sDS + r * LP + c0) = pack_bf16x2(d0, d1);
        }
      }
      __syncthreads();

      const int col0 = warp * CW;
      // ---- dq += dS . kv   (A = dS [16 x 32], B = kv [32 keys x D] row-major -> trans loads)
#pragma unroll
      for (int ks = 0; ks < kKeys / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(smem_u32(sDS + (lane & 15) * LP + ks * 16 + (lane >> 4) * 8), a);
        const uint32_t b_base = smem_u32(sKV + (ks * 16 + (lane & 15)) * LQ + col0);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          uint32_t bb[2];
          ldsm_x2_t(b_base + j * 16, bb);
          mma16816(dq[j], a, bb);
        }
      }
      // ---- dkv[32 x D] = dS^T . q + P^T . do, one 16-key half at a time
#pragma unroll 1
      for (int mt = 0; mt < kKeys / 16; ++mt) {
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        // A = X^T with X [16 heads x 32 keys]: transposed 8x8 blocks
        const int arow = (lane >> 4) * 8 + (lane & 7), acol = mt * 16 + ((lane >> 3) & 1) * 8;
        uint32_t ads[4], ap[4];
        ldsm_x4_t(smem_u32(sDS + arow * LP + acol), ads);
        ldsm_x4_t(smem_u32(sP + arow * LP + acol), ap);
        const uint32_t bq = smem_u32(sQ + (lane & 15) * LQ + col0);
        const uint32_t bo = smem_u32(sDO + (lane & 15) * LO + col0);
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          uint32_t bb[2];
          ldsm_x2_t(bq + j * 16, bb);
          mma16816(acc[j], ads, bb);
          if (col0 + j * 8 < Dv) {
            ldsm_x2_t(bo + j * 16, bb);
            mma16816(acc[j], ap, bb);
          }
        }
        // even lanes (t4 = 0, 2) add row k0, columns 2*t4 .. 2*t4+3; odd lanes add
        // row k0+8, columns 2*(t4-1) .. +3 (each lane takes its partner's half)
        const bool odd = t4 & 1;
        const int kr = mt * 16 + g + (odd ? 8 : 0);
        const int v = sIdx[kr];
        float* dst = v >= 0 ? p.dkv + ((size_t)b * p.Nkv + v) * D + col0 + 2 * (t4 & ~1) : nullptr;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const float s0 = odd ? acc[j][0] : acc[j][2], s1 = odd ? acc[j][1] : acc[j][3];
          const float r0 = __shfl_xor_sync(0xffffffffu, s0, 1), r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
          if (dst) {
            if (odd)
              red_add_v4(dst + j * 8, r0, r1, acc[j][2], acc[j][3]);
            else
              red_add_v4(dst + j * 8, acc[j][0], acc[j][1], r0, r1);
          }
        }
      }
    }
    // ---- dq out (rows g, g+8; columns col0 + 8j + 2*t4)
    const int col0 = warp * CW;
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int h = h0 + g + 8 * hr;
      if (h >= p.H) continue;
      __nv_bfloat16* drow = p.dq + ((size_t)bs * p.H + h) * D + col0 + 2 * t4;
#pragma unroll
      for (int j = 0; j < NT; ++j)
        *reinterpret_cast<uint32_t*>(drow + j * 8) = pack_bf16x2(dq[j][2 * hr], dq[j][2 * hr + 1]);
    }
    __syncthreads();
  }
}

template <int NT>
static cudaError_t launch_nt(const Params& p, int grid, cudaStream_t stream) {
  const size_t smem = smem_bytes(p.D, p.Dv);
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
  const long long cap = (long long)device_sm_count() * 2;
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
