// FP8 KV row quantiser: bf16 kv rows [rows, D] -> the FP8 row format read by
// si_sparse_attn_fwd_fp8kv.
//
// Row layout (the V4 production KV row: FP8 e4m3 NoPE dims with one fp32 scale
// per 64-dim block, RoPE dims kept in bf16; docs/ir_analysis.md:45-55 of the
// reference, scale block 64 as model.py's act_quant(kv[..., :-rd], 64) there):
//   bytes [0, n_nope)                    e4m3 of dims [0, n_nope)
//   bytes [n_nope, n_nope + 4*nblk)      fp32 scale of each 64-dim block
//   bytes [rope_off, rope_off + 2*n_rope) bf16 dims [n_nope, D)
//   rope_off = n_nope + 4*nblk rounded up to 16, row_bytes = end rounded up to 16
// (pads are zero).  At D = 576 / n_nope = 512 a row is 672 bytes; at the V4-Pro
// 512 / 448 split it is 608 bytes (the 604-byte payload, 16-byte aligned so the
// gather loads stay 16-byte loads).
//
// Per block the arithmetic is the reference's quant-dequant simulation
// act_quant_simulate (flash_sparse/utils/quantization.py:19-36) on bf16 input,
// step for step in the input dtype:
//   amax  = max(max|x|, 1e-4)            (bf16)
//   scale = bf16(amax / 448)
//   q     = e4m3_rn(clamp(bf16(x / scale), -448, 448))
// and the stored scale is float(scale), so float(q) * scale rounded to bf16 is
// exactly the simulation's dequantised value.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "capi_common.h"
#include "../../include/streamindex_b200.h"

namespace si {

__global__ void kv_quant_fp8_kernel(const __nv_bfloat16* __restrict__ kv, long long rows, int D, int n_nope,
                                    int rope_off, int row_bytes, uint8_t* __restrict__ out) {
  const int nblk = n_nope / 64;
  const int items_per_row = nblk + 1;  // one warp per 64-dim block, plus one for the rope dims and pads
  const long long total = rows * items_per_row;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); it < total; it += warps) {
    const long long row = it / items_per_row;
    const int blk = (int)(it - row * items_per_row);
    const __nv_bfloat16* x = kv + row * D;
    uint8_t* o = out + row * row_bytes;
    if (blk < nblk) {
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(x + blk * 64)[lane];
      const float x0 = __bfloat162float(v.x), x1 = __bfloat162float(v.y);
      float a = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, m));
      a = fmaxf(a, __bfloat162float(__float2bfloat16_rn(1e-4f)));
      const float scale = __bfloat162float(__float2bfloat16_rn(a / 448.0f));
      const float q0 = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn(x0 / scale)), -448.f), 448.f);
      const float q1 = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn(x1 / scale)), -448.f), 448.f);
      const __nv_fp8x2_storage_t q2 =
          __nv_cvt_float2_to_fp8x2(make_float2(q0, q1), __NV_SATFINITE, __NV_E4M3);
      reinterpret_cast<__nv_fp8x2_storage_t*>(o + blk * 64)[lane] = q2;
      if (lane == 0) reinterpret_cast<float*>(o + n_nope)[blk] = scale;
    } else {
      // rope dims as bf16 at rope_off; zero the pad between the scales and the
      // rope dims and after the rope dims
      const int n_rope = D - n_nope;
      for (int j = lane; j < n_rope; j += 32)
        reinterpret_cast<__nv_bfloat16*>(o + rope_off)[j] = x[n_nope + j];
      for (int j = n_nope + 4 * nblk + lane; j < rope_off; j += 32) o[j] = 0;
      for (int j = rope_off + 2 * n_rope + lane; j < row_bytes; j += 32) o[j] = 0;
    }
  }
}

}  // namespace si

extern "C" {

int si_kv_quant_fp8(const void* kv, long long rows, int D, int n_nope, void* out, cudaStream_t stream) {
  if (!kv || !out) return si::fail("kv_quant_fp8: null pointer");
  if (rows < 0) return si::fail("kv_quant_fp8: rows must be >= 0");
  const int row_bytes = si_fp8_kv_row_bytes(D, n_nope);
  if (row_bytes < 0 || n_nope > 512 || D - n_nope > 64 || D % 8)
    return si::fail("kv_quant_fp8: need n_nope a multiple of 64 in [64,512] and 0 < D - n_nope <= 64, D %% 8 == 0 "
                    "(got D=%d, n_nope=%d)", D, n_nope);
  if (((uintptr_t)kv | (uintptr_t)out) & 15) return si::fail("kv_quant_fp8: 16-byte alignment");
  if (rows == 0) return 0;
  const int rope_off = ((n_nope + 4 * (n_nope / 64)) + 15) / 16 * 16;
  const long long warps = rows * (n_nope / 64 + 1);
  long long blocks = (warps + 7) / 8;
  const long long cap = (long long)si::device_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  si::kv_quant_fp8_kernel<<<(int)blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(kv), rows, D,
                                                            n_nope, rope_off, row_bytes,
                                                            reinterpret_cast<uint8_t*>(out));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("kv_quant_fp8: launch", e);
}

}  // extern "C"
