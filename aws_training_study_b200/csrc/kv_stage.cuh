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

#include "attn_common.cuh"
#include "ptx.cuh"

namespace pcp {

constexpr int kMaxSources = 64;

struct UnpackSource {
  const uint8_t* base;   // first block of this source's packed payload (or the block pool)
  const int32_t* table;  // NULL: blocks are contiguous; else logical block -> pool block (device)
  long long pool_blocks; // blocks the pool holds (checked when `table` is set)
  int valid;             // valid tokens of this source (device-length mode: the bucket's upper bound)
  int dst_offset;        // first key slot in the dense output (device-length mode: the part's first key)
  int dev_index;         // device-length mode: index of this source in UnpackParams::valid_dev
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
  int* err;                  // set to kErrBlockTable on an entry outside the pool
  // Device-length mode (valid_dev != NULL, bucketed graphs): the valid count
  // of source s is valid_dev[src[s].dev_index], clamped to src[s].valid (a
  // larger one records kErrBucket); sources are compacted in order from
  // their common dst_offset, and block (0, 0) stores the part's total keys
  // in *part_keys for the attention launch that follows.
  const int32_t* valid_dev;
  int* part_keys;
};

__device__ __forceinline__ int device_valid(const UnpackParams& p, int s) {
  const int v = p.valid_dev[p.src[s].dev_index];
  return min(max(v, 0), p.src[s].valid);
}

__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint16_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  return pack_bf16x2(f.x, f.y);
}

// grid: (x = chunks of one source's live payload, y = source).  Each thread
// converts 16 consecutive head-dim elements of one token of one head.
__global__ void __launch_bounds__(256) kv_unpack_kernel(const UnpackParams p) {
  const int s = blockIdx.y;
  UnpackSource src = p.src[s];
  if (p.valid_dev) {
    const int v = p.valid_dev[src.dev_index];
    if ((v < 0 || v > src.valid) && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(p.err, 0, kErrBucket);
    for (int i = 0; i < s; ++i) src.dst_offset += device_valid(p, i);
    src.valid = device_valid(p, s);
    if (blockIdx.x == 0 && s == 0 && threadIdx.x == 0) {
      int total = 0;
      for (int i = 0; i < p.num_sources; ++i) total += device_valid(p, i);
      *p.part_keys = total;
    }
  }
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
    long long pblk = blk;
    if (src.table) {
      pblk = src.table[blk];
      if (pblk < 0 || pblk >= src.pool_blocks) {
        atomicCAS(p.err, 0, kErrBlockTable);
        continue;
      }
    }
    const uint8_t* in = src.base + (pblk * per_block + (e - blk * per_block)) * 16 * elt;
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

// current_scatter_kernel: the current (prefill) tokens' K and V of every rank,
//   each a striped shard [Hkv][Qloc][D] bf16 laid out like the Q shards
//   (pcp_attention/layout.py:34-51), source s at s * Hkv * Qloc * D -> dense
//   K, V [Hkv][key_stride][D] with local token i of source s at key
//   key_off + its global position, so the causal attention launch sees the
//   keys in sequence order.
struct ScatterParams {
  const __nv_bfloat16* k_src;  // [P][Hkv][Qloc][D]
  const __nv_bfloat16* v_src;
  int num_sources;             // P
  int num_kv_heads;
  int local_len;               // Qloc
  int head_dim;
  int stripe_width;            // I
  int key_stride;
  int key_off;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
};

// grid-stride over 16-byte chunks of [2][P][Hkv][Qloc][D]; consecutive
// threads copy consecutive chunks of one token row.
__global__ void __launch_bounds__(256) current_scatter_kernel(const ScatterParams p) {
  const int chunks_per_row = p.head_dim / 8;
  const long long per_kv = static_cast<long long>(p.num_sources) * p.num_kv_heads * p.local_len * chunks_per_row;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < 2 * per_kv;
       e += (long long)gridDim.x * blockDim.x) {
    const int kv = e >= per_kv;
    long long r = kv ? e - per_kv : e;
    const int chunk = static_cast<int>(r % chunks_per_row);
    r /= chunks_per_row;
    const int i = static_cast<int>(r % p.local_len);
    r /= p.local_len;
    const int h = static_cast<int>(r % p.num_kv_heads);
    const int s = static_cast<int>(r / p.num_kv_heads);
    const uint4 val = reinterpret_cast<const uint4*>(kv ? p.v_src : p.k_src)[kv ? e - per_kv : e];
    const int g = striped_position(i, p.num_sources, p.stripe_width, s);
    __nv_bfloat16* out = (kv ? p.v_out : p.k_out) +
                         (static_cast<size_t>(h) * p.key_stride + p.key_off + g) * p.head_dim + chunk * 8;
    *reinterpret_cast<uint4*>(out) = val;
  }
}

// cache_write_kernel: the paged-cache producer.  New tokens' K/V in sequence
//   order ([Hkv][T][D] bf16, token t at absolute position first + t) are
//   written, quantised to the cache dtype, into the owner rank's paged cache:
//   position p belongs to rank (p / I) % P at local slot
//   (p / (P I)) * I + p % I (pcp_attention/layout.py:10-16, 54-98), i.e.
//   logical block slot / bs, row slot % bs, and the logical block lives at
//   pool block table[logical] in the packed payload format
//   ([2][Hkv][bs][D] per block, pcp_attention/kernel.py:17-29).  This rank
//   writes only the tokens it owns; they map to one contiguous local range.
//   e4m3fn rounding: nearest-even, magnitudes above 464 and non-finite values
//   -> NaN (the behaviour of tensor.to(torch.float8_e4m3fn)).
struct CacheWriteParams {
  const __nv_bfloat16* k_src;  // [Hkv][T][D]
  const __nv_bfloat16* v_src;
  int num_tokens;              // T
  long long first;             // absolute position of token 0
  long long local0;            // first local slot this rank owns in [first, first + T)
  int owned;                   // tokens this rank owns in [first, first + T)
  int ranks, width, rank;      // P, I, this rank
  int num_kv_heads, block_size, head_dim, kv_is_bf16;
  const int32_t* table;        // logical block -> pool block (device)
  int table_len;
  long long pool_blocks;
  uint8_t* pool;               // [pool_blocks][payload]
  int* err;                    // kErrBlockTable on a missing / out-of-pool entry
};

__device__ __forceinline__ uint16_t e4m3x2_from_floats(float a, float b) {
  uint16_t c = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  // Beyond the rounding range of the largest finite value (448), and NaN/Inf:
  // the NaN code with the input's sign.
  if (!(fabsf(a) <= 464.f)) c = static_cast<uint16_t>((c & 0xFF00u) | 0x7Fu | ((__float_as_uint(a) >> 24) & 0x80u));
  if (!(fabsf(b) <= 464.f))
    c = static_cast<uint16_t>((c & 0x00FFu) | ((0x7Fu | ((__float_as_uint(b) >> 24) & 0x80u)) << 8));
  return c;
}

// grid-stride over 8-element chunks of [2][Hkv][owned][D].
__global__ void __launch_bounds__(256) cache_write_kernel(const CacheWriteParams p) {
  const int chunks_per_row = p.head_dim / 8;
  const long long per_kv = static_cast<long long>(p.num_kv_heads) * p.owned * chunks_per_row;
  const long long stride_pi = static_cast<long long>(p.ranks) * p.width;
  const int elt = p.kv_is_bf16 ? 2 : 1;
  const long long payload = 2LL * p.num_kv_heads * p.block_size * p.head_dim * elt;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < 2 * per_kv;
       e += (long long)gridDim.x * blockDim.x) {
    const int kv = e >= per_kv;
    long long r = kv ? e - per_kv : e;
    const int chunk = static_cast<int>(r % chunks_per_row);
    r /= chunks_per_row;
    const long long local = p.local0 + r % p.owned;
    const int h = static_cast<int>(r / p.owned);
    const long long pos = (local / p.width) * stride_pi + static_cast<long long>(p.rank) * p.width + local % p.width;
    const long long t = pos - p.first;
    const long long lblk = local / p.block_size;
    const int slot = static_cast<int>(local % p.block_size);
    const long long pblk = lblk < p.table_len ? p.table[lblk] : -1;
    if (t < 0 || t >= p.num_tokens || pblk < 0 || pblk >= p.pool_blocks) {
      atomicCAS(p.err, 0, kErrBlockTable);
      continue;
    }
    const uint4 in = *reinterpret_cast<const uint4*>((kv ? p.v_src : p.k_src) +
                                                      (static_cast<size_t>(h) * p.num_tokens + t) * p.head_dim + chunk * 8);
    uint8_t* dst = p.pool + pblk * payload +
                   ((static_cast<long long>(kv) * p.num_kv_heads + h) * p.block_size + slot) * p.head_dim * elt +
                   chunk * 8 * elt;
    if (p.kv_is_bf16) {
      *reinterpret_cast<uint4*>(dst) = in;
    } else {
      const uint32_t w[4] = {in.x, in.y, in.z, in.w};
      uint16_t c[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        c[i] = e4m3x2_from_floats(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
      *reinterpret_cast<uint2*>(dst) = make_uint2(c[0] | (static_cast<uint32_t>(c[1]) << 16),
                                                  c[2] | (static_cast<uint32_t>(c[3]) << 16));
    }
  }
}

// block_gather_kernel: the live blocks of one rank's paged shard, read
//   through its block table, copied into a contiguous packed buffer (the send
//   buffer of the exchange).  16-byte chunks, grid-stride.
struct BlockGatherParams {
  const uint8_t* pool;
  const int32_t* table;
  long long pool_blocks;
  int live_blocks;
  long long payload;  // bytes per block (multiple of 16)
  uint8_t* out;
  int* err;
};

__global__ void __launch_bounds__(256) block_gather_kernel(const BlockGatherParams p) {
  const long long per_block = p.payload / 16;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < per_block * p.live_blocks;
       e += (long long)gridDim.x * blockDim.x) {
    const long long blk = e / per_block;
    const long long pblk = p.table[blk];
    if (pblk < 0 || pblk >= p.pool_blocks) {
      atomicCAS(p.err, 0, kErrBlockTable);
      continue;
    }
    reinterpret_cast<uint4*>(p.out)[e] = reinterpret_cast<const uint4*>(p.pool + pblk * p.payload)[e - blk * per_block];
  }
}

struct CombineParams {
  const float* part_o;    // [splits][rows][D]
  const float* part_lse;  // [splits][rows]
  __nv_bfloat16* out;     // [rows][D]
  int num_splits;         // <= 32
  int rows;
  // Single-part stream-K launch: the attention kernel wrote the rows of every
  // unit that one segment covered as final output; those rows are skipped.
  int skip_single;
  int units, grid_pairs, rows_per_head, m_tiles;
  // The launch's key tiles: `count` (or its bound), `count_dev` the actual
  // number in device-length mode; both count keys (ceil(keys / 128) tiles)
  // when count_is_keys (dense launches), else tiles (in-place launches).
  int count;
  const int* count_dev;
  int count_is_keys;
};

template <int D>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
  const int warps_per_block = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  long long n_kt = 0, steps = 0, pairs = 1;
  if (p.skip_single) {
    const int cnt = p.count_dev ? min(max(*p.count_dev, 0), p.count) : p.count;
    n_kt = p.count_is_keys ? (cnt + kTileN - 1) / kTileN : cnt;
    steps = static_cast<long long>(p.units) * n_kt;
    pairs = stream_k_pairs(steps, p.grid_pairs);
  }
  for (int row = blockIdx.x * warps_per_block + (threadIdx.x >> 5); row < p.rows;
       row += gridDim.x * warps_per_block) {
    if (p.skip_single && steps > 0) {
      const long long unit =
          static_cast<long long>(row / p.rows_per_head) * p.m_tiles + (row % p.rows_per_head) / (2 * kTileM);
      const long long ub = unit * n_kt;
      if (stream_k_pair_of(ub + n_kt - 1, steps, pairs) == stream_k_pair_of(ub, steps, pairs)) continue;
    }
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
      if (ws == 0.f) continue;  // an empty split (lse = -inf): its O was never written
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
