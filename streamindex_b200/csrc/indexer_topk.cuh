// Fused lightning-indexer score + streaming top-k for sm_100a.
//
// Math (flash_sparse/reference.py:163-168, eq. 16 of the V4 report):
//   I[b,s,t] = sum_h w[b,s,h] * relu(q[b,s,h,:] . k[b,t,:])
// followed by the causal mask t < (s+1)//ratio (flash_sparse/triton/chunked_indexer.py:137)
// and a per-query top-k in the order (score desc, index asc)
// (docs/streaming_topk.md:48-66).  The [B,S,T] score tensor is never written
// (except in the explicit materialise mode used by indexer_score).
//
// Mapping.  One persistent CTA per SM owns a "query block" of QC = 512/H
// consecutive queries at a time.  Their Q rows ([QC*H, D] bf16, 128-byte
// swizzled) stay resident in shared memory.  Keys stream through in tiles of
// 128 rows (TMA), and the tensor core computes, per tile and per query group
// g (two groups of 256 (query, head) columns):
//     C_g[t, (s,h)] = k[t] . q[s,h]      M = 128 keys, N = 256, K = D
// into TMEM columns [256g, 256g+256).  Keys on M means each epilogue thread
// owns one key row, so ReLU, the fp32 w multiply and the sum over heads run
// inside the thread with no cross-thread reduction.  The two groups form a
// double buffer: the epilogue of group 0 overlaps the MMAs of group 1.
//
// Warp roles (576 threads for H_I <= 64, 320 for H_I = 128):
//   warp 0      TMA producer (Q block, K tiles; q and k are 2-D [rows, D] tensor
//               maps when their rows are evenly spaced, else 4-D [B,S,H,D] /
//               3-D [B,T,D] maps, so any strides with a contiguous last dim are
//               read in place)
//   warp 1      TMEM allocator + single-thread UMMA issuer
//   warps 2..   epilogue: scores + streaming top-k.  Warp w reads TMEM lanes
//               32*(w%4)..+32 (its "quadrant"); the epilogue warps are cut into
//               slices of four (one per quadrant) that own the same queries:
//               64-column slices for H_I <= 64 (16 warps), 128-column slices
//               for H_I = 128 (8 warps) — see EpiCfg.
//
// Streaming top-k.  Each query keeps, in a global workspace slab (L2
// resident), a candidate buffer of CAP 64-bit keys
//   key = ord(score) << 32 | (2^32-1 - t)
// (larger key = better under the reference's order).  A key enters the buffer
// iff it beats the query's threshold key (the smallest key kept at the last
// flush, 0 before; cached in registers).  Every kSyncTiles key tiles the
// slice's four warps meet; a buffer that could not absorb kSyncTiles more
// tiles of inserts is flushed: the four warps load it into registers, run an
// exact radix select (8-bit digits over the 64-bit key, below the keys' common
// prefix), compact it to the top K and raise the threshold.  Selection is
// exact, so the result is the exact top-K under the total order whatever the
// tiling.  At the end of a query block the kept keys are written unsorted into
// the idx output; a row-sort kernel turns them into (idx int64, score fp32)
// sorted descending, padded with -1 / -inf.
#pragma once
#include "ptx.cuh"

namespace si {

constexpr int kKeysPerTile = 128;   // UMMA M
constexpr int kGroupCols = 256;     // UMMA N per group
constexpr int kQRows = 512;         // (query, head) rows resident per block
constexpr int kEpiWarps = 16;      // maximum epilogue warps (hist scratch sizing)

// Epilogue shape per head count: NS column slices of each 256-column group,
// one warp per (TMEM lane quadrant, slice).  H_I <= 64 uses 16 warps (four per
// SM sub-partition, one 64-column slice = one H_I=64 query each) so the
// epilogue hides TMEM / shared-memory latency; H_I = 128 uses 8 warps with
// 128-column slices so a query never straddles two warps.
template <int H>
struct EpiCfg {
  static constexpr int NS = (H == 128) ? 2 : 4;
  static constexpr int CW = kGroupCols / NS;   // columns per warp
  static constexpr int NQW = CW / H;           // queries per warp
  static constexpr int WARPS = 4 * NS;
  static constexpr int THREADS = 32 * (2 + WARPS);
};
constexpr int kMaxQC = 32;          // H >= 16
constexpr int kSyncTiles = 4;
constexpr int kSelRegs = 12;        // keys per thread held in registers by the cooperative select       // top-k capacity checks / flushes every kSyncTiles key tiles

enum IndexerMode : int { kModeTopk = 0, kModeTopkMask = 1, kModeScore = 2 };

struct IndexerParams {
  int B, S, T, H, D;          // D is the padded head dim (multiple of 64, <= 128)
  int ratio;                  // > 0: causal t < (s+1)//ratio ; 0: none
  int ksel;                   // top-k width (selection size)
  int cap;                    // candidate buffer capacity per query (multiple of 32, >= ksel + 128)
  int w_is_bf16;
  const void* w;              // [B,S,H] fp32 or bf16, contiguous
  const uint8_t* mask;        // [B,S,T] bool (mode 1), contiguous
  unsigned long long* out_keys;  // [B,S,ksel] (aliases the int64 idx output) — topk modes
  float* out_scores;          // [B,S,T] — score mode
  unsigned long long* cand;   // workspace: gridDim.x * QC * cap keys
  int* status;                // device status word
  int nblk_per_batch;         // ceil(S / QC)
  long long s_offset;         // global position of local query 0 (causal mask uses s_offset + s)
  unsigned long long* trace;  // debug builds (SI_IDX_TRACE) only
};

#ifdef SI_IDX_TRACE
// [role 0..2][tile < 512][point < 8], first block of CTA 0 only
#define SI_ITRACE(role, r, tile, pt)                                                        \
  do {                                                                                      \
    if (p.trace && blockIdx.x == 0 && (r) == 0 && (tile) < 512)                             \
      p.trace[((role) * 512 + (tile)) * 8 + (pt)] = globaltimer();                          \
  } while (0)
#else
#define SI_ITRACE(role, r, tile, pt) \
  do {                               \
  } while (0)
#endif

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Order-preserving map of an fp32 score to uint32 (larger float -> larger uint).
__device__ __forceinline__ uint32_t ord_f32(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
__device__ __forceinline__ unsigned long long make_key(float score, int t) {
  return ((unsigned long long)ord_f32(score) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)t);
}

}  // namespace si
