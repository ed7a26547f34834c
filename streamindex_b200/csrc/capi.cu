// Common C-ABI plumbing: error reporting, tensor maps, device status readback.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "capi_common.h"
#include "ptx.cuh"
#include "../../include/streamindex_b200.h"

namespace si {

static thread_local char g_err[512] = "";

int fail(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return -1;
}

int fail_cuda(const char* what, cudaError_t e) {
  return fail("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int device_sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d_16b(CUtensorMap* map, const void* base, int cols, uint64_t rows, int box_cols, int box_rows,
                     int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled is unavailable from the driver");
  if ((((uintptr_t)base) & 15) || ((cols * 2) % 16)) return fail("tensor map: base/row stride not 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)(rows > 0 ? rows : 1)};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return 0;
}

int make_tmap_nd_16b(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* byte_strides, const uint32_t* box, int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled is unavailable from the driver");
  if (rank < 2 || rank > 5) return fail("tensor map: rank %d outside [2,5]", rank);
  if (((uintptr_t)base) & 15) return fail("tensor map: base not 16-byte aligned");
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i] > 0 ? dims[i] : 1;
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    if (byte_strides[i] % 16) return fail("tensor map: stride %d (%llu bytes) not a multiple of 16", i + 1,
                                          (unsigned long long)byte_strides[i]);
    st[i] = byte_strides[i];
  }
  CUresult r = fn(map, dtype ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank,
                  const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled (rank %d) failed (CUresult %d)", rank, (int)r);
  return 0;
}

cudaError_t set_smem_attr_once(const void* func, int bytes, unsigned long long* seen) {
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  std::lock_guard<std::mutex> lock(mu);
  if (*seen & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) *seen |= bit;
  return e;
}

__global__ void fill_pad_kernel(int64_t* idx, float* scores, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    idx[i] = -1;
    scores[i] = -INFINITY;
  }
}

cudaError_t launch_fill_pad(int64_t* idx, float* scores, long long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 4 * 148 * 8) blocks = 4 * 148 * 8;
  fill_pad_kernel<<<(unsigned)blocks, 256, 0, stream>>>(idx, scores, n);
  return cudaGetLastError();
}

// Self-test of the bounded-wait machinery: one CTA waits on an mbarrier that
// nothing ever arrives on.  The wait must give up after `limit_ns`, record
// kErrWaitTmaFull in the status word and let the kernel return normally.
__global__ void wait_timeout_selftest_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait_ns(&bar, 0, &abort_flag, status, kErrWaitTmaFull, limit_ns);
  __syncthreads();
}

}  // namespace si

extern "C" {

int si_selftest_wait_timeout(void* ws, unsigned long long limit_ns, cudaStream_t stream) {
  if (!ws) return si::fail("selftest_wait_timeout: null workspace");
  if (limit_ns > 2000000000ull) return si::fail("selftest_wait_timeout: limit above 2 s");
  int* status = reinterpret_cast<int*>(ws);
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream);
  if (e != cudaSuccess) return si::fail_cuda("selftest_wait_timeout: status reset", e);
  si::wait_timeout_selftest_kernel<<<1, 64, 0, stream>>>(status, limit_ns);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : si::fail_cuda("selftest_wait_timeout: launch", e);
}


const char* si_last_error(void) { return si::g_err; }

int si_abi_version(void) { return SI_ABI_VERSION; }

int si_read_status(const void* ws, int* status_out, cudaStream_t stream) {
  if (!ws || !status_out) return si::fail("si_read_status: null pointer");
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return si::fail_cuda("si_read_status", e);
  *status_out = v;
  return 0;
}

}  // extern "C"
