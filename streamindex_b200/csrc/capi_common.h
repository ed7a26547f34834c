// Host-side helpers shared by the C-ABI entry points: thread-local error
// string, TMA tensor-map encoding, device queries.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace si {

constexpr size_t kStatusBytes = 256;  // status word at the head of every workspace

int fail(const char* fmt, ...);                      // records the message, returns -1
int fail_cuda(const char* what, cudaError_t e);      // records "<what>: <cuda error>", returns -1
int device_sm_count();
// 2-D row-major tensor of 16-bit elements [rows, cols] (cols contiguous), box
// [box_rows, box_cols] with the 128-byte swizzle.  dtype: 0 bf16, 1 fp16.
int make_tmap_2d_16b(CUtensorMap* map, const void* base, int cols, uint64_t rows, int box_cols, int box_rows,
                     int dtype);
// Sets a kernel's max dynamic shared memory once per (kernel, device); thread safe.
// `seen` is a per-kernel bitmask of devices already configured.
// N-D (rank 2..5) tensor of 16-bit elements, dims[0] innermost and contiguous;
// byte_strides[i] is the stride of dimension i+1 (multiples of 16 bytes), box
// per dimension, the 128-byte swizzle.  dtype: 0 bf16, 1 fp16.
int make_tmap_nd_16b(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* byte_strides, const uint32_t* box, int dtype);
cudaError_t set_smem_attr_once(const void* func, int bytes, unsigned long long* seen);
cudaError_t launch_fill_pad(int64_t* idx, float* scores, long long n, cudaStream_t stream);

}  // namespace si
