// Per-row pieces of the softmax warpgroups, shared by the CTA-pair attention
// kernels (attn_pair.cuh, attn_pair_sk.cuh, attn_pair2.cuh, attn_kv.cuh).
//
// A softmax thread owns one TMEM lane, i.e. one query row of its CTA's 128:
// a contiguous run of S columns per key tile and a contiguous run of O
// columns.  Every function here is warp-collective (tcgen05.ld / st /
// wait are .sync.aligned) and must be reached by all 32 lanes of the warp
// under warp-uniform control flow.  All are force-inlined, so each kernel
// compiles to what it did with the code written out in place.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace pcp {

// This lane's kKeys scores of a tile: TMEM columns [t_col, t_col + kKeys).
// Keys at or past `valid` (counted from the first of them) become -inf.
template <int kKeys>
__device__ __forceinline__ void load_scores(uint32_t t_col, int valid, float (&s)[kKeys]) {
  static_assert(kKeys % 32 == 0, "scores are loaded 32 columns at a time");
#pragma unroll
  for (int c = 0; c < kKeys / 32; ++c) tmem_ld32(t_col + 32 * c, s + 32 * c);
  tmem_wait_ld();
  if (valid < kKeys) {
#pragma unroll
    for (int i = 0; i < kKeys; ++i)
      if (i >= valid) s[i] = -INFINITY;
  }
}

// Maximum of kKeys scores (four independent chains).
template <int kKeys>
__device__ __forceinline__ float row_max(const float (&s)[kKeys]) {
  float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
  for (int i = 4; i < kKeys; i += 4) {
    mx0 = fmaxf(mx0, s[i]);
    mx1 = fmaxf(mx1, s[i + 1]);
    mx2 = fmaxf(mx2, s[i + 2]);
    mx3 = fmaxf(mx3, s[i + 3]);
  }
  return fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
}

// P = 2^((s - m) * sl2) of kKeys keys (ex2.approx on the MUFU), packed in
// pairs -- bf16, or f16 with kF16 (the PV MMA's A and B share one type) --
// into TMEM columns [t_col, t_col + kKeys / 2) of this lane: the first half
// of the columns the scores came from, whose values this lane already holds,
// so no other lane's unread scores are overwritten.  The stores are complete
// on return; returns the fp32 sum of the unrounded P.
template <int kKeys, bool kF16 = false>
__device__ __forceinline__ float store_probs(const float* s, float m, float sl2, uint32_t t_col) {
  const float neg = -m * sl2;
  float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
  for (int c2 = 0; c2 < kKeys / 32; ++c2) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float p0 = ex2_approx(fmaf(s[c2 * 32 + 2 * i], sl2, neg));
      const float p1 = ex2_approx(fmaf(s[c2 * 32 + 2 * i + 1], sl2, neg));
      sum0 += p0;
      sum1 += p1;
      pk[i] = kF16 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
    }
    tmem_st16(t_col + c2 * 16, pk);
  }
  tmem_wait_st();
  return sum0 + sum1;
}

// O *= alpha over kCols fp32 TMEM columns from t_o (the running-max rescale;
// the PV MMAs that write these columns must be complete).
template <int kCols>
__device__ __forceinline__ void rescale_o(uint32_t t_o, float alpha) {
#pragma unroll 1
  for (int c = 0; c < kCols / 32; ++c) {
    float o[32];
    tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] *= alpha;
    tmem_st32(t_o + c * 32, o);
  }
  tmem_wait_st();
}

// O * inv_l of kCols TMEM columns from t_o as fp32 to dst (a split partial
// row); rows past the end (`live` false) load but write nothing.
template <int kCols>
__device__ __forceinline__ void store_o_partial(uint32_t t_o, float inv_l, float* dst, bool live) {
#pragma unroll 1
  for (int c = 0; c < kCols / 32; ++c) {
    float o[32];
    tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
    if (live) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + c * 32 + i) =
            make_float4(o[i] * inv_l, o[i + 1] * inv_l, o[i + 2] * inv_l, o[i + 3] * inv_l);
    }
  }
}

// O * inv_l of kCols TMEM columns from t_o as bf16 straight to global dst.
template <int kCols>
__device__ __forceinline__ void store_o_bf16(uint32_t t_o, float inv_l, __nv_bfloat16* dst, bool live) {
#pragma unroll 1
  for (int c = 0; c < kCols / 32; ++c) {
    float o[32];
    tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(o[2 * i] * inv_l, o[2 * i + 1] * inv_l);
    if (live) {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4)
        *reinterpret_cast<uint4*>(dst + c * 32 + q4 * 8) =
            make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
    }
  }
}

// O * inv_l of kCols TMEM columns from t_o as bf16 into row `row`, columns
// [col0, col0 + kCols), of a 128-row shared-memory tile laid out like the Q
// tiles the TMA loads: boxes of 64 columns (128 rows x 128 B each, `box_bytes`
// apart), 16-byte chunks XOR-swizzled by row % 8 (the 128B swizzle).  A TMA
// store of the boxes then writes the rows out.
template <int kCols>
__device__ __forceinline__ void stage_o_sw128(uint32_t t_o, float inv_l, uint8_t* tile, int box_bytes, int col0,
                                              int row) {
#pragma unroll 1
  for (int c = 0; c < kCols / 32; ++c) {
    float o[32];
    const int col = col0 + c * 32;
    tmem_ld32(t_o + c * 32, o);
    tmem_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(o[2 * i] * inv_l, o[2 * i + 1] * inv_l);
    uint8_t* rowp = tile + (col / 64) * box_bytes + row * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int chunk = ((col % 64) / 8) + q;
      const int phys = chunk ^ (row & 7);
      *reinterpret_cast<uint4*>(rowp + phys * 16) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
  }
}

}  // namespace pcp
