// Memory-bound helper kernels around the attention kernel.
//
// kv_unpack_kernel: paged ring payload -> dense compacted bf16 K and V.
//   Input per source rank: blocks in the reference's packed ring-payload
//   format (pcp_attention/kernel.py:17-29), block b = [2][Hkv][bs][D] with all
//   K before all V, e4m3fn (dequantised at unit scale exactly as `.float()` in
//   pcp_attention/reference.py:29-31,70-71; every e4m3 value is exact in bf16)
//   or bf16.  Only the first valid_len tokens of a source are kept (the
//   reference masks the rest with an additive -9984 bias, run_poc.py:137-153),
//   so fully masked blocks are neither read nor computed.
//   Output: K, V as [Hkv][key_stride][D] bf16 with source s's tokens at keys
//   [dst_offset[s], dst_offset[s] + valid_len[s]).
//
// combine_kernel: merges split-KV partials (normalised O, log2-sum-exp) into
//   the bf16 output [Hq][Qloc][D].  One warp per output row.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "ptx.cuh"

namespace pcp {

constexpr int kMaxSources = 64;

struct UnpackSource {
  const uint8_t* base;  // first block of this source's packed payload
  int valid;            // valid tokens of this source
  int dst_offset;       // first key slot in the dense output
};

struct UnpackParams {
  UnpackSource src[kMaxSources];
  int num_sources;
  int num_kv_heads;
  int block_size;
  int head_dim;
  int kv_is_bf16;
  int key_stride;            // keys per head in the dense output
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
};

__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint16_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  return pack_bf16x2(f.x, f.y);
}

// grid: (x = chunks of one source's live payload, y = source).  Each thread
// converts 16 consecutive head-dim elements of one token of one head.
__global__ void __launch_bounds__(256) kv_unpack_kernel(const UnpackParams p) {
  const int s = blockIdx.y;
  const UnpackSource src = p.src[s];
  const int chunks_per_row = p.head_dim / 16;
  const int live_blocks = (src.valid + p.block_size - 1) / p.block_size;
  const long long per_block = 2LL * p.num_kv_heads * p.block_size * chunks_per_row;
  const long long total = per_block * live_blocks;
  const int elt = p.kv_is_bf16 ? 2 : 1;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    long long r = e;
    const int chunk = static_cast<int>(r % chunks_per_row);
    r /= chunks_per_row;
    const int tok = static_cast<int>(r % p.block_size);
    r /= p.block_size;
    const int h = static_cast<int>(r % p.num_kv_heads);
    r /= p.num_kv_heads;
    const int kv = static_cast<int>(r % 2);
    const int blk = static_cast<int>(r / 2);
    const int local = blk * p.block_size + tok;
    if (local >= src.valid) continue;
    const uint8_t* in = src.base + e * 16 * elt;
    __nv_bfloat16* out = (kv ? p.v_out : p.k_out) +
                         (static_cast<size_t>(h) * p.key_stride + src.dst_offset + local) * p.head_dim + chunk * 16;
    if (p.kv_is_bf16) {
      const uint4 a = *reinterpret_cast<const uint4*>(in);
      const uint4 b = *reinterpret_cast<const uint4*>(in + 16);
      reinterpret_cast<uint4*>(out)[0] = a;
      reinterpret_cast<uint4*>(out)[1] = b;
    } else {
      const uint4 a = *reinterpret_cast<const uint4*>(in);
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[2 * i] = e4m3x2_to_bf16x2(static_cast<uint16_t>(w[i] & 0xFFFFu));
        o[2 * i + 1] = e4m3x2_to_bf16x2(static_cast<uint16_t>(w[i] >> 16));
      }
      reinterpret_cast<uint4*>(out)[0] = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4*>(out)[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
}

struct CombineParams {
  const float* part_o;    // [splits][rows][D]
  const float* part_lse;  // [splits][rows]
  __nv_bfloat16* out;     // [rows][D]
  int num_splits;         // <= 32
  int rows;
};

template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
  const int warps_per_block = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps_per_block + (threadIdx.x >> 5); row < p.rows;
       row += gridDim.x * warps_per_block) {
    const float lse = lane < p.num_splits ? p.part_lse[static_cast<size_t>(lane) * p.rows + row] : -INFINITY;
    float m = lse;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float w = lane < p.num_splits ? ex2_approx(lse - m) : 0.f;
    float wsum = w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
    const float inv = 1.f / wsum;
    // Each lane owns D/32 consecutive elements (4 or 8).
    constexpr int per_lane = D / 32;
    float acc[per_lane];
#pragma unroll
    for (int i = 0; i < per_lane; ++i) acc[i] = 0.f;
    for (int s = 0; s < p.num_splits; ++s) {
      const float ws = __shfl_sync(0xffffffffu, w, s);
      const float* src = p.part_o + (static_cast<size_t>(s) * p.rows + row) * D + lane * per_lane;
#pragma unroll
      for (int i = 0; i < per_lane; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + i);
        acc[i] += ws * v.x;
        acc[i + 1] += ws * v.y;
        acc[i + 2] += ws * v.z;
        acc[i + 3] += ws * v.w;
      }
    }
    __nv_bfloat16* dst = p.out + static_cast<size_t>(row) * D + lane * per_lane;
#pragma unroll
    for (int i = 0; i < per_lane; i += 4) {
      uint2 pk;
      pk.x = pack_bf16x2(acc[i] * inv, acc[i + 1] * inv);
      pk.y = pack_bf16x2(acc[i + 2] * inv, acc[i + 3] * inv);
      *reinterpret_cast<uint2*>(dst + i) = pk;
    }
  }
}

}  // namespace pcp
