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
// Q [64 heads x D] stays in shared memory for the item; the item's selected
// KV rows are gathered NK at a time with TMA row gathers (tile::gather4, one
// 1152-byte row per index at D=576) into 128-byte-swizzled tiles that serve
// both GEMMs:
//   MMA1  S[64 x NK]  = Q . KV^T           (M=64, K=D, A and B K-major)
//   MMA2  O[64 x Dv] += P . V              (M=64, K=NK, P K-major, V MN-major)
// With M=64 an accumulator occupies TMEM lanes 0-15 of each 32-lane quarter;
// O lives there (lanes 0-15, columns [0,Dv)) and the two S buffers live in
// lanes 16-31 (columns [0,2*NK)), so the whole TMEM is used without overlap.
//
// Softmax warps (4, one per lane quarter = 16 heads): thread 16+i of a warp
// owns head row i of S and computes the online softmax for it; thread i owns
// the same head's O row.  The running shift is only raised when the tile max
// exceeds it by more than 8 (log2 units), so O is rescaled (ld/scale/st with
// the 16x32bx2 TMEM shape, which touches lanes 0-15 only) rarely; P = exp2(s -
// shift) <= 256 stays exact in bf16 range.  P goes to shared memory (bf16) as
// the A operand of MMA2.
//
// Warp roles (192 threads): warp 0 TMA (Q + gathers), warp 1 TMEM alloc +
// UMMA issue, warps 2-5 softmax / correction / output.
#include <cuda_bf16.h>

#include "capi_common.h"
#include "ptx.cuh"
#include "../../include/streamindex_b200.h"

namespace si {
namespace attn {

constexpr int kHeads = 64;    // UMMA M (heads per work item)
constexpr int kThreads = 192;
constexpr int kSmemMax = 232448;

struct Params {
  int B, S, H, D;      // D: qk head dim (multiple of 8)
  int NA;              // ceil(D/64) swizzle atoms per row
  int Nkv;             // kv rows per batch
  int K;               // indices per query
  int Dv, dv_off;      // value columns [dv_off, dv_off+Dv) of kv (multiples of 64)
  int o_ld, o_off;     // output row stride (elements) and column offset
  float scale_log2;    // softmax_scale * log2(e)
  const int* idx;      // [B,S,K]
  const float* sink;   // [H]
  __nv_bfloat16* o;    // [B,S,H,o_ld]
  float* lse;          // [B,S,H] or null
  int* status;
  int hgroups;         // ceil(H/64)
};

struct __align__(8) Misc {
  uint64_t kv_full[8], kv_empty[8];
  uint64_t q_full, q_empty;
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done, o_free;
  uint32_t tmem_base;
  int abort_flag;
};

template <int NK>
__host__ __device__ inline int stage_bytes(int NA) { return NA * NK * 128; }

template <int NK>
__host__ __device__ inline int num_stages(int NA) {
  const int fixed = 1024 + NA * kHeads * 128 + 2 * NK * 128 + (int)sizeof(Misc) + 64;
  int n = (kSmemMax - fixed) / stage_bytes<NK>(NA);
  return n > 8 ? 8 : n;
}

template <int NK>
__host__ __device__ inline size_t smem_bytes(int NA) {
  return 1024 + (size_t)NA * kHeads * 128 + (size_t)num_stages<NK>(NA) * stage_bytes<NK>(NA) + 2 * NK * 128 +
         sizeof(Misc);
}

}  // namespace attn
}  // namespace si
