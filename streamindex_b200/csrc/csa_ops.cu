// CSA glue kernels: sliding-window + compressed index build and the mean-pool
// compressor.  Both are HBM-bound elementwise passes (grid-stride, coalesced,
// grid sized to a multiple of the SM count).
#include <cuda_bf16.h>

#include "capi_common.h"
#include "../../include/streamindex_b200.h"

namespace si {

// out[b,s,:] = [ window(s) | comp[b,s,j] + S (or -1) ], int32.
// window(s)_w = s - n_win + 1 + w if that position is in [0, s], else -1
// (flash_sparse/reference.py:470-475); compressed indices are offset by S
// because the attention reads cat[kv; kv_compressed] (flash_sparse/csa.py:177-179).
__global__ void csa_build_idx_kernel(const int64_t* __restrict__ comp, int B, int S, int top_k, int n_win,
                                     long long s_offset, int S_total, int32_t* __restrict__ out) {
  const int W = n_win + top_k;
  const long long total = (long long)B * S * W;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int col = (int)(i % W);
    const long long bs = i / W;
    const long long s = s_offset + bs % S;  // global query position
    int v;
    if (col < n_win) {
      const long long pos = s - n_win + 1 + col;
      v = (pos >= 0 && pos <= s) ? (int)pos : -1;
    } else {
      const long long c = comp[bs * top_k + (col - n_win)];
      v = c >= 0 ? (int)(c + S_total) : -1;
    }
    out[i] = v;
  }
}

// Mean over each block of m tokens: [B,S,C] -> [B,S/m,C] (fp32 math, bf16 out);
// the non-overlapping compressor with uniform softmax weights
// (reference_token_compressor(overlap=False), flash_sparse/reference.py:234-240).
__global__ void mean_pool_kernel(const __nv_bfloat16* __restrict__ x, int B, int S, int C, int m,
                                 __nv_bfloat16* __restrict__ out) {
  const int nb = S / m;
  const int C2 = C / 2;
  const long long total = (long long)B * nb * C2;
  const float inv = 1.f / (float)m;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c2 = (int)(i % C2);
    const long long bn = i / C2;
    const int n = (int)(bn % nb);
    const int b = (int)(bn / nb);
    const __nv_bfloat162* src = reinterpret_cast<const __nv_bfloat162*>(x + ((long long)b * S + (long long)n * m) * C) + c2;
    float sx = 0.f, sy = 0.f;
    for (int j = 0; j < m; ++j) {
      const float2 f = __bfloat1622float2(src[(long long)j * C2]);
      sx += f.x * inv;
      sy += f.y * inv;
    }
    reinterpret_cast<__nv_bfloat162*>(out)[i] = __floats2bfloat162_rn(sx, sy);
  }
}

static int elementwise_grid(long long n) {
  const long long blocks = (n + 255) / 256;
  const long long cap = (long long)device_sm_count() * 16;
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace si

extern "C" {

int si_csa_build_idx_ex(const int64_t* comp_idx, int B, int S, long long s_offset, int S_total, int top_k, int n_win,
                        int32_t* out, cudaStream_t stream) {
  if (B < 1 || S < 0 || top_k < 0 || n_win < 0 || s_offset < 0 || s_offset + S > S_total)
    return si::fail("csa_build_idx: bad sizes (S=%d, s_offset=%lld, S_total=%d)", S, s_offset, S_total);
  if ((long long)S_total * 2 + 1 >= (1ll << 31)) return si::fail("csa_build_idx: S too large for int32 indices");
  const long long n = (long long)B * S * (n_win + top_k);
  if (n == 0) return 0;
  if (!out || (top_k > 0 && !comp_idx)) return si::fail("csa_build_idx: null pointer");
  si::csa_build_idx_kernel<<<si::elementwise_grid(n), 256, 0, stream>>>(comp_idx, B, S, top_k, n_win, s_offset,
                                                                          S_total, out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("csa_build_idx: launch", e);
}

int si_csa_build_idx(const int64_t* comp_idx, int B, int S, int top_k, int n_win, int32_t* out, cudaStream_t stream) {
  return si_csa_build_idx_ex(comp_idx, B, S, 0, S, top_k, n_win, out, stream);
}

int si_mean_pool(const void* x, int B, int S, int C, int m, void* out, cudaStream_t stream) {
  if (B < 1 || S < 0 || C < 2 || (C & 1) || m < 1) return si::fail("mean_pool: bad sizes (C must be even)");
  if (((uintptr_t)x | (uintptr_t)out) & 3) return si::fail("mean_pool: 4-byte alignment");
  const long long n = (long long)B * (S / m) * (C / 2);
  if (n == 0) return 0;
  si::mean_pool_kernel<<<si::elementwise_grid(n), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), B, S, C, m, reinterpret_cast<__nv_bfloat16*>(out));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("mean_pool: launch", e);
}

}  // extern "C"

namespace si {

// HCA index list [B,S,n_win+n_comp]: the sliding window, then every compressed
// block i legal for query s ((i+1)*m' - 1 <= s), offset by S, else -1
// (flash_sparse/hca.py:24-51).
__global__ void hca_build_idx_kernel(int B, int S, int n_win, int n_comp, int m_prime, int32_t* __restrict__ out) {
  const int W = n_win + n_comp;
  const long long total = (long long)B * S * W;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int col = (int)(i % W);
    const int s = (int)((i / W) % S);
    int v;
    if (col < n_win) {
      const int pos = s - n_win + 1 + col;
      v = (pos >= 0 && pos <= s) ? pos : -1;
    } else {
      const int c = col - n_win;
      v = ((long long)(c + 1) * m_prime - 1 <= s) ? c + S : -1;
    }
    out[i] = v;
  }
}

}  // namespace si

extern "C" {

int si_hca_build_idx(int B, int S, int n_win, int n_comp, int m_prime, int32_t* out, cudaStream_t stream) {
  if (B < 1 || S < 0 || n_win < 0 || n_comp < 0 || m_prime < 1) return si::fail("hca_build_idx: bad sizes");
  if ((long long)S + n_comp >= (1ll << 31)) return si::fail("hca_build_idx: indices exceed int32");
  const long long n = (long long)B * S * (n_win + n_comp);
  if (n == 0) return 0;
  if (!out) return si::fail("hca_build_idx: null output");
  si::hca_build_idx_kernel<<<si::elementwise_grid(n), 256, 0, stream>>>(B, S, n_win, n_comp, m_prime, out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("hca_build_idx: launch", e);
}

}  // extern "C"

namespace si {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Softmax-gated token compressor (flash_sparse/reference.py:176-272), one
// thread per (b, block, channel), fp32 math.  Non-overlapping: weights =
// softmax over the block's m tokens of z_a + b_a.  Overlapping: a joint 2m-way
// softmax over the block's a-stream (z_a + b_a, values c_a) and the previous
// block's b-stream (z_b + b_b, values c_b; absent for block 0).
template <typename T>
__global__ void token_compressor_kernel(const T* __restrict__ ca, const T* __restrict__ za,
                                        const T* __restrict__ ba, const T* __restrict__ cb,
                                        const T* __restrict__ zb, const T* __restrict__ bb, int B, int S, int C,
                                        int m, int overlap, T* __restrict__ out) {
  const int nb = S / m;
  const long long total = (long long)B * nb * C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const long long bn = i / C;
    const int n = (int)(bn % nb);
    const int b = (int)(bn / nb);
    const long long row0 = (long long)b * S + (long long)n * m;  // first token of block n
    const bool use_b = overlap && n > 0;
    float mx = -INFINITY;
    for (int j = 0; j < m; ++j) mx = fmaxf(mx, to_f(za[(row0 + j) * C + c]) + to_f(ba[j * C + c]));
    if (use_b)
      for (int j = 0; j < m; ++j) mx = fmaxf(mx, to_f(zb[(row0 - m + j) * C + c]) + to_f(bb[j * C + c]));
    float den = 0.f, num = 0.f;
    for (int j = 0; j < m; ++j) {
      const float e = __expf(to_f(za[(row0 + j) * C + c]) + to_f(ba[j * C + c]) - mx);
      den += e;
      num += e * to_f(ca[(row0 + j) * C + c]);
    }
    if (use_b)
      for (int j = 0; j < m; ++j) {
        const float e = __expf(to_f(zb[(row0 - m + j) * C + c]) + to_f(bb[j * C + c]) - mx);
        den += e;
        num += e * to_f(cb[(row0 - m + j) * C + c]);
      }
    out[i] = from_f<T>(num / den);
  }
}

}  // namespace si

extern "C" {

int si_token_compressor(const void* c_a, const void* z_a, const void* b_a, const void* c_b, const void* z_b,
                        const void* b_b, int B, int S, int C, int m, int overlap, int is_bf16, void* out,
                        cudaStream_t stream) {
  if (B < 1 || S < 0 || C < 1 || m < 1) return si::fail("token_compressor: bad sizes");
  if (!c_a || !z_a || !b_a || !out) return si::fail("token_compressor: null pointer");
  if (overlap && (!c_b || !z_b || !b_b)) return si::fail("token_compressor: overlap needs c_b, z_b, b_b");
  const long long n = (long long)B * (S / m) * C;
  if (n == 0) return 0;
  const int grid = si::elementwise_grid(n);
  if (is_bf16) {
    using T = __nv_bfloat16;
    si::token_compressor_kernel<T><<<grid, 256, 0, stream>>>(
        (const T*)c_a, (const T*)z_a, (const T*)b_a, (const T*)c_b, (const T*)z_b, (const T*)b_b, B, S, C, m,
        overlap, (T*)out);
  } else {
    si::token_compressor_kernel<float><<<grid, 256, 0, stream>>>(
        (const float*)c_a, (const float*)z_a, (const float*)b_a, (const float*)c_b, (const float*)z_b,
        (const float*)b_b, B, S, C, m, overlap, (float*)out);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("token_compressor: launch", e);
}

}  // extern "C"
