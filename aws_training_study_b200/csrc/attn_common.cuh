// Shared definitions of the history-attention kernel (attn_pair.cuh): tile
// shape, TMEM map, thread roles, error codes and launch parameters.
//
// Every (KV head, 256-row Q tile, key split) work unit computes
// softmax(Q K^T * scale) V over a contiguous range of 128-key tiles of a
// dense, compacted bf16 K/V buffer, on a cluster of two CTAs (one per SM)
// that share each tcgen05 MMA (cta_group::2).
//
// Replaces the NKI kernel body of the reference (pcp_attention/kernel.py:
// 84-554).  Stage map, reference -> here:
//   resident Q load + pre-scale (kernel.py:141-173) -> TMA load of the CTA's
//       128 bf16 Q rows into 128B-swizzled smem once; scale applied in fp32.
//   K/V resident load (kernel.py:295-339) -> TMA producer warp streaming each
//       CTA's half of every K tile ([64 keys, D]) and V tile ([128 keys, D/2])
//       through a smem ring holding 2.5 tiles.
//   QK^T into PSUM (kernel.py:383-394) -> tcgen05.mma kind::f16, M=256 over the
//       pair, N=128 keys, fp32 accumulator S in TMEM (two buffers).
//   mask + max + fused exp/sum (kernel.py:396-437) -> two softmax warpgroups
//       per CTA, one thread per row (TMEM lane) and 64 keys per warpgroup;
//       exp2 (MUFU) with an fp32 running reference max and sums; keys past
//       the valid count in the final tile are -inf.
//   P transpose (kernel.py:439-462) -> none: P is written back to TMEM as bf16
//       (over S) and used as the A operand of the PV MMA.
//   PV + rescale (kernel.py:464-511) -> tcgen05.mma A=P (TMEM), B=V (smem,
//       MN-major), O accumulates in TMEM across all tiles; O is rescaled in
//       TMEM only when the running max grows by more than 2^8 (lazy rescale).
//   finalise/store (kernel.py:516-553) -> O/l in fp32, bf16 via swizzled smem
//       + TMA store, or fp32 partial + log2-sum-exp for the split combine.
//
// Thread roles (320 threads per CTA, 1 CTA per SM):
//   warps 0-7 softmax / correction / epilogue in two warpgroups: warpgroup w
//     owns key columns [64w, 64w+64) of every S tile and head-dim columns
//     [w*D/2, (w+1)*D/2) of O,
//   warp 8 TMA producer, warp 9 TMEM allocator and (leader CTA) the single
//     thread that issues every MMA of the pair.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include "ptx.cuh"

namespace pcp {

constexpr int kTileM = 128;       // query rows per CTA (TMEM lanes)
constexpr int kTileN = 128;       // keys per tile
constexpr int kBoxCols = 64;      // bf16 columns per 128B-swizzled TMA box
constexpr int kBoxBytes = 128 * 128;  // one box of 128 rows x 128 B
constexpr int kTmemCols = 512;
constexpr int kTmemS0 = 256;      // S/P buffers at columns 256 and 384; O at 0
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kSoftmaxWarpgroups = 2;
constexpr int kSoftmaxThreads = 128 * kSoftmaxWarpgroups;
constexpr int kThreads = kSoftmaxThreads + 64;  // + TMA warp + MMA warp
constexpr int kProducerWarp = kSoftmaxThreads / 32;
constexpr int kMmaWarp = kProducerWarp + 1;

enum : int {
  kErrWaitQ = 101,
  kErrWaitKvEmpty = 102,
  kErrWaitKvFull = 103,
  kErrWaitPFull = 104,
  kErrWaitSFull = 105,
  kErrWaitODone = 106,
  kErrSmemAlign = 107,
  kErrWaitRed = 108,
  kErrBlockTable = 109,  // a block-table entry outside the pool (nothing written or read there)
  kErrBucket = 110,      // a device valid length above its bucket's bound (clamped to the bound)
  kErrSchedule = 111,    // a segment's partial slot beyond the launch's slot count (not written)
};

struct AttnParams {
  int rows_per_head;     // R: query rows sharing one KV head (q_heads_per_kv * Qloc)
  int m_tiles_per_head;  // ceil(R / 128)
  int num_kv_heads;
  int num_keys;          // valid keys in the compacted K/V buffer
  int tiles_per_split;   // key tiles per split
  int split_base;        // first split index of this launch in the partial buffers
  int total_rows;        // num_kv_heads * R
  float scale_log2;      // softmax_scale * log2(e)
  int write_final;       // static schedule: 1 bf16 O, 0 fp32 partial O + lse
  __nv_bfloat16* out;    // bf16 O [total_rows][D]
  float* part_o;         // [splits][total_rows][D]
  float* part_lse;       // [splits][total_rows]
  int* err;              // device error word
  // Causal current-token mode (causal != 0): the keys are the current
  // (prefill) tokens of every rank in global order, key index = global
  // position.  Query row i of this rank's striped shard sits at global
  // position (i / I) * (P * I) + rank * I + i % I and sees keys <= it; each
  // pair tile stops after the key tile holding its last query's position.
  // Launched with one split.
  int causal;
  int q_local_len;       // Qloc
  int stripe_ranks;      // P
  int stripe_width;      // I
  int stripe_rank;       // rank of the query shard
  // Device-length mode: the valid keys are *num_keys_dev (written by the
  // unpack of this part; at most num_keys, the bucket's bound).  Splits past
  // them are empty: they store lse = -inf so the combine ignores them.
  const int* num_keys_dev;
  // Stream-K instantiation: partial slots [split_base, split_base +
  // max_segs) per unit; a unit that one segment covers is written as bf16 O
  // when final_ok.  (Static: unit = pair, split = blockIdx.y, bf16 O when
  // write_final.)
  int max_segs;
  int final_ok;
};

// Stream-K partition of T (unit, key tile) steps over G pairs: pair g owns
// steps [T g / G, T (g + 1) / G).  At least two steps per pair, so a unit of a
// launch with U units is cut into at most ceil(2G/U) + 1 segments.
__host__ __device__ __forceinline__ long long stream_k_pairs(long long steps, int grid_pairs) {
  const long long half = steps / 2;
  const long long g = grid_pairs < half ? grid_pairs : half;
  return g > 1 ? g : 1;
}
// The pair whose range holds step x.
__host__ __device__ __forceinline__ long long stream_k_pair_of(long long x, long long steps, long long pairs) {
  return ((x + 1) * pairs + steps - 1) / steps - 1;
}

// Global position of local query/key index i of `rank`'s striped shard
// (pcp_attention/layout.py:19-31).
__host__ __device__ __forceinline__ int striped_position(int i, int ranks, int width, int rank) {
  return (i / width) * (ranks * width) + rank * width + i % width;
}

}  // namespace pcp
