// History attention that reads the FP8 e4m3 KV cache in place.
//
// The same CTA-pair pipeline as attn_fwd_pair_kernel / attn_fwd_pair_sk_kernel
// (attn_pair.cuh, attn_pair_sk.cuh: one thread issues the pair's
// tcgen05 cta_group::2 MMAs, two softmax warpgroups per CTA with lazy
// rescale, accumulators in TMEM), with the K/V operands taken straight from
// the packed cache instead of a dense bf16 copy:
//   * The TMA producer loads each CTA's half of every K tile ([64 keys][D]
//     e4m3) and V tile ([128 keys][D/2] e4m3) from the cache blocks
//     [blocks][2][Hkv][bs][D] (pcp_attention/kernel.py:17-29 payload) through
//     a 5-D tensor map, block index = the source's first block + logical
//     block, or its block-table entry for a paged pool (kernel.py:295-339
//     reads the same blocks from its ring buffer).  Loads land in a raw
//     e4m3 ring (kRawStages) of THIS CTA; no multicast.
//   * Four converter warps per CTA upcast each raw item to f16 (exact:
//     cvt.rn.f16x2.e4m3x2, the unit-scale dequantisation of `.float()` in
//     pcp_attention/reference.py:29-31) into the 128B-swizzled operand layout
//     the MMAs read (kOpStages), writing zeros for keys past the source's
//     valid count, then fence the async proxy and arrive on the leader's
//     op_full barrier.  Q (bf16) is converted to f16 in place once per
//     segment the same way.
//   * Every MMA is kind::f16 with f16 A and B (Q K^T: Q f16, K f16; P V: P
//     f16 from TMEM, V f16): f16 holds every e4m3 and every bf16 Q value of
//     normal magnitude exactly, and P in [0, 2^8] with 3 more mantissa bits
//     than bf16.
// Keys are walked per source: source s contributes ceil(valid_s / 128) key
// tiles, the last one partial (kernel.py's additive mask, run_poc.py:137-153,
// skips nothing the valid count does not).  Fully masked blocks are never
// loaded.  The schedule is the wave-scheduled one (one (unit, split) item
// per pair) or stream-K (equal contiguous tile ranges per persistent pair),
// chosen per launch.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "attn_common.cuh"
#include "attn_pair.cuh"
#include "attn_pair_sk.cuh"
#include "kv_stage.cuh"
#include "ptx.cuh"

namespace pcp {

// Four converter warps, one per SM sub-partition (warps 10..13 -> SMSPs
// 2, 3, 0, 1): the e4m3 -> f16 conversion (~6 issue cycles per warp
// instruction of cvt.rn.f16x2.e4m3x2 per sub-partition, measured) is spread
// over every issue port.
constexpr int kConvWarps = 4;
constexpr int kConvThreads = 32 * kConvWarps;
constexpr int kKvThreads = kThreads + kConvThreads;  // 448: 8 softmax, TMA, MMA, 4 converter warps
constexpr int kConvWarp0 = kMmaWarp + 1;
constexpr int kSchedStatic = 0;
constexpr int kSchedStreamK = 1;

// One history source of a launch: its blocks in the launch's tensor map.
struct KvSource {
  const int32_t* table;  // NULL: logical block b is map block blk0 + b; else map block table[b] (device)
  long long blk0;
  int valid;             // valid tokens (device-length mode: the bucket's upper bound)
  int dev_index;         // device-length mode: index of this source's count in valid_dev
};

struct KvParams {
  AttnParams a;              // shapes, split bookkeeping, outputs (num_keys / causal fields unused)
  KvSource src[kMaxSources];
  int num_sources;
  int block_size;
  long long map_blocks;      // blocks the tensor maps cover (table entries are checked against it)
  const int32_t* valid_dev;  // device-length mode: actual counts, clamped to src[].valid
  int* tiles_out;            // device-length mode: the launch's key-tile count, for the combine
  int sched;                 // kSchedStatic or kSchedStreamK
};

template <int D>
struct KvSmem {
  static constexpr int kQBytes = D * 2 * kTileM;  // own 128 rows, f16 after conversion
  static constexpr int kOpBytes = 128 * D;         // f16 K half [64, D] or V half [128, D/2], swizzled
  static constexpr int kRawBytes = 64 * D;         // e4m3 K half [64][D] or V half [128][D/2]
  static constexpr int kOpStages = (D == 256) ? 3 : 8;
  static constexpr int kRawStages = (D == 256) ? 4 : 7;
  static constexpr int kKBox = 64 * 128;   // f16 K box: 64 rows x 128 B
  static constexpr int kVBox = 128 * 128;  // f16 V box: 128 rows x 128 B
  static constexpr int kQOff = 0;
  static constexpr int kOpOff = kQBytes;
  static constexpr int kRawOff = kOpOff + kOpStages * kOpBytes;
  static constexpr int kBarOff = kRawOff + kRawStages * kRawBytes;
  // q_raw, q_ready, q_empty, raw_full[NR], raw_empty[NR], op_full[NS],
  // op_empty[NS], s_full[2], p_full[2], o_done[2], teardown, red[2]
  static constexpr int kNumBars = 3 + 2 * kRawStages + 2 * kOpStages + 9;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kRedOff = kMiscOff + 16;
  static constexpr int kSrcOff = kRedOff + 2 * kSoftmaxWarpgroups * kTileM * 4;
  // int tile0[kMaxSources + 1], valid[kMaxSources]
  static constexpr int kBytes = kSrcOff + (2 * kMaxSources + 1) * 4;
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 232448, "exceeds the 227 KB of shared memory per CTA");
  static_assert(kOpOff % 1024 == 0 && kOpBytes % 1024 == 0 && kRawOff % 1024 == 0, "operand alignment");
};

// Key tile kt of a launch: its source, first key within the source and the
// source's valid keys in the tile (1..128).
struct TileLoc {
  int src;
  int key0;
  int valid;
};

__device__ __forceinline__ TileLoc locate_tile(const int* tile0, const int* valid, int nsrc, int kt) {
  int s = 0;
  while (s + 1 < nsrc && tile0[s + 1] <= kt) ++s;
  const int key0 = (kt - tile0[s]) * kTileN;
  return {s, key0, min(kTileN, valid[s] - key0)};
}

// Where converter thread ct moves its chunks of one item.  A K half is 64
// raw rows of D bytes, a V half 128 raw rows of D/2 bytes: 4 x `boxes`
// 16-byte chunks per row, stored as `boxes` 128B-swizzled f16 boxes of 64
// columns.  The 16 quarter-warps (8 threads: one 128-bit shared-memory
// wavefront) take tasks (row pair, box): rows 2p and 2p+1 get four
// consecutive chunks each, of boxes b and b ^ 1, so the raw loads (16-byte
// bank group = row * cpr + chunk, mod 8) and the swizzled stores (group =
// (2 * (chunk % 4) [+1]) ^ (row & 7)) both hit 8 distinct groups.  Task
// m of a thread is 32 / boxes rows below its task 0 (same chunk, same
// row & 7), so a thread's m-th chunk is 2048 m raw bytes and
// 4096 / boxes * m operand bytes past its first.
struct ConvGeo {
  uint32_t raw;   // raw byte offset of chunk 0
  uint32_t lo;    // operand byte offsets of its two f16 halves
  uint32_t hi;
  int row;        // row (key) of chunk 0
};

__device__ __forceinline__ ConvGeo conv_geo(int ct, int boxes, uint32_t box_bytes) {
  const int j = ct & 7, q = ct >> 3;
  const int row = 2 * (q / boxes) + (j >> 2);
  const int cbox = boxes > 1 ? ((q % boxes) ^ (j >> 2)) : 0;
  const int c16 = 4 * cbox + (j & 3);
  const int ch = (j & 3) * 2;
  const uint32_t rowp = cbox * box_bytes + row * 128;
  return {static_cast<uint32_t>((row * 4 * boxes + c16) * 16), rowp + ((ch ^ (row & 7)) << 4),
          rowp + (((ch + 1) ^ (row & 7)) << 4), row};
}

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kKvThreads, 1)
    attn_fwd_kv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const KvParams kp) {
  using L = KvSmem<D>;
  constexpr int NS = L::kOpStages;
  constexpr int NR = L::kRawStages;
  const AttnParams& p = kp.a;

  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // identical in both CTAs: neither starts
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, kErrSmemAlign);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t sQ = sbase + L::kQOff;
  const uint32_t sOp = sbase + L::kOpOff;
  const uint32_t sRaw = sbase + L::kRawOff;
  const uint32_t bars = sbase + L::kBarOff;
  const uint32_t bar_q_raw = bars;        // this CTA's Q landed (TMA bytes)
  const uint32_t bar_q_ready = bars + 8;  // leader: Q converted in both CTAs (one arrive per converter warp)
  const uint32_t bar_q_empty = bars + 16; // the segment's last QK^T has read Q (MMA commit, both CTAs)
  auto bar_raw_full = [&](int s) { return bars + 8u * (3 + s); };
  auto bar_raw_empty = [&](int s) { return bars + 8u * (3 + NR + s); };
  auto bar_op_full = [&](int s) { return bars + 8u * (3 + 2 * NR + s); };
  auto bar_op_empty = [&](int s) { return bars + 8u * (3 + 2 * NR + NS + s); };
  constexpr int kB2 = 3 + 2 * NR + 2 * NS;
  auto bar_s_full = [&](int b) { return bars + 8u * (kB2 + b); };
  auto bar_p_full = [&](int b) { return bars + 8u * (kB2 + 2 + b); };
  // o_done[b] completes once per PV of tile J with J % 2 == b (phase J / 2).
  auto bar_o = [&](int b) { return bars + 8u * (kB2 + 4 + b); };
  const uint32_t bar_td = bars + 8u * (kB2 + 6);
  auto bar_red = [&](int b) { return bars + 8u * (kB2 + 7 + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  int* s_tile0 = reinterpret_cast<int*>(smem + L::kSrcOff);
  int* s_valid = s_tile0 + kMaxSources + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;
  const int nsrc = kp.num_sources;

  if (threadIdx.x == 0) {
    // Valid keys and first key tile of every source (device-length mode: the
    // counts on the device, clamped to their bounds).
    int acc = 0;
    for (int s = 0; s < nsrc; ++s) {
      int v = kp.src[s].valid;
      if (kp.valid_dev) {
        const int x = kp.valid_dev[kp.src[s].dev_index];
        if ((x < 0 || x > v) && blockIdx.x == 0 && blockIdx.y == 0) atomicCAS(p.err, 0, kErrBucket);
        v = min(max(x, 0), v);
      }
      s_valid[s] = v;
      s_tile0[s] = acc;
      acc += (v + kTileN - 1) / kTileN;
    }
    s_tile0[nsrc] = acc;
    if (kp.tiles_out && blockIdx.x == 0 && blockIdx.y == 0) *kp.tiles_out = acc;
  }
  if (warp == kProducerWarp && lane == 0) {
    mbar_init(bar_q_raw, 1);
    mbar_init(bar_q_ready, 2 * kConvWarps);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < NR; ++s) {
      mbar_init(bar_raw_full(s), 1);
      mbar_init(bar_raw_empty(s), kConvWarps);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_op_full(s), 2 * kConvWarps);
      mbar_init(bar_op_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), 2 * kSoftmaxWarps);  // one arrive per softmax warp of both CTAs
    }
    mbar_init(bar_o(0), 1);
    mbar_init(bar_o(1), 1);
    mbar_init(bar_td, 1);
    mbar_init(bar_red(0), kSoftmaxThreads);
    mbar_init(bar_red(1), kSoftmaxThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated, source table written
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_kt = s_tile0[nsrc];
  const int units = p.num_kv_heads * p.m_tiles_per_head;

  // Calls body(segment) for each segment of this pair, in order, until it
  // returns false; returns false if it did.  Static schedule: one segment,
  // the pair's (unit, split) item, slot = split.
  auto for_each_segment = [&](auto&& body) -> bool {
    if (kp.sched == kSchedStreamK) {
      Schedule sc;
      sc.init_stream_k(n_kt, units, gridDim.x >> 1, pair);
      Segment sg;
      while (sc.next(sg))
        if (!body(sg)) return false;
      return true;
    }
    Segment sg;
    sg.unit = pair;
    sg.kt0 = static_cast<int>(blockIdx.y) * p.tiles_per_split;
    sg.kt1 = min(sg.kt0 + p.tiles_per_split, n_kt);
    sg.slot = static_cast<int>(blockIdx.y);
    sg.nseg = static_cast<int>(gridDim.y);
    sg.last = sg.kt1 >= n_kt;
    return body(sg);
  };

  if (warp == kProducerWarp) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0) {
      uint32_t c = 0;
      int segs = 0;
      bool primed = false;
      int cached_src = -1, cached_lb = -1, cached_pb = 0;
      // Map block of logical block lb of source s (block-table entries
      // outside the map are reported and replaced by block 0, so every
      // issued load stays in bounds and the pipeline keeps its byte counts).
      auto map_block = [&](int s, int lb) -> int {
        if (s == cached_src && lb == cached_lb) return cached_pb;
        const KvSource& src = kp.src[s];
        long long b = src.table ? static_cast<long long>(src.table[lb]) : src.blk0 + lb;
        if (b < 0 || b >= kp.map_blocks) {
          atomicCAS(p.err, 0, kErrBlockTable);
          b = 0;
        }
        cached_src = s;
        cached_lb = lb;
        cached_pb = static_cast<int>(b);
        return cached_pb;
      };
      // Item order = converter and MMA consumption order: per segment K_0,
      // then (K_{j+1}, V_j) per tile.
      auto issue = [&](bool is_v, int kt, int head) {
        const int st = c % NR;
        if (!mbar_wait(bar_raw_empty(st), ((c / NR) & 1u) ^ 1u, abort_flag, p.err, kErrWaitKvEmpty)) return false;
        const TileLoc tl = locate_tile(s_tile0, s_valid, nsrc, kt);
        const uint32_t dst = sRaw + st * L::kRawBytes;
        if (!is_v) {
          // This CTA's K half: keys [64 rank, +64) of the tile; nothing to
          // load when all of them are past the valid count.
          const int key = tl.key0 + 64 * static_cast<int>(rank);
          const bool any = tl.valid > 64 * static_cast<int>(rank);
          mbar_arrive_expect_tx(bar_raw_full(st), any ? 64 * D : 0);
          if (any)
            tma_load_5d(dst, &tm_k, 0, key % kp.block_size, head, 0, map_block(tl.src, key / kp.block_size),
                        bar_raw_full(st));
        } else {
          // This CTA's V half (head dims [rank D/2, +D/2)) of all 128 keys,
          // as two 64-key boxes (a box never crosses a cache block: bs % 64
          // == 0).
          const int halves = tl.valid > 64 ? 2 : 1;
          mbar_arrive_expect_tx(bar_raw_full(st), halves * 64 * (D / 2));
          for (int h2 = 0; h2 < halves; ++h2) {
            const int key = tl.key0 + 64 * h2;
            tma_load_5d(dst + h2 * 64 * (D / 2), &tm_v, static_cast<int>(rank) * (D / 2), key % kp.block_size, head,
                        1, map_block(tl.src, key / kp.block_size), bar_raw_full(st));
          }
        }
        ++c;
        return true;
      };
      const bool ok = for_each_segment([&](const Segment& sg) -> bool {
        const int n = sg.kt1 - sg.kt0;
        if (n <= 0) return true;
        if (!primed) {
          tma_prefetch_desc(&tm_q);
          tma_prefetch_desc(&tm_k);
          tma_prefetch_desc(&tm_v);
          primed = true;
        }
        const int head = sg.unit / p.m_tiles_per_head;
        const int row0 = (sg.unit % p.m_tiles_per_head) * kPairRows + static_cast<int>(rank) * kTileM;
        // Q of this segment: once the previous segment's QK^T are done with sQ.
        if (segs > 0 && !mbar_wait(bar_q_empty, (segs - 1) & 1u, abort_flag, p.err, kErrWaitQ)) return false;
        mbar_arrive_expect_tx(bar_q_raw, L::kQBytes);
        for (int b = 0; b < D / kBoxCols; ++b) tma_load_3d(sQ + b * kBoxBytes, &tm_q, b * kBoxCols, row0, head, bar_q_raw);
        ++segs;
        if (!issue(false, sg.kt0, head)) return false;
        for (int j = 0; j < n; ++j) {
          if (j + 1 < n && !issue(false, sg.kt0 + j + 1, head)) return false;
          if (!issue(true, sg.kt0 + j, head)) return false;
        }
        return true;
      });
      if (!ok) {
        // Abort: let this CTA's copies still in flight land before it exits.
        for (uint32_t i = (c > (uint32_t)NR ? c - NR : 0); i < c; ++i)
          mbar_wait_teardown(bar_raw_full(i % NR), (i / NR) & 1u);
        if (segs > 0) mbar_wait_teardown(bar_q_raw, (segs - 1) & 1u);
      }
    }
    __syncwarp();
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------- e4m3 -> f16 converters --
    const int ct = threadIdx.x - kConvWarp0 * 32;  // 0 .. kConvThreads - 1
    static_assert(kConvThreads == 128, "16 quarter-warps of converter tasks");
    const ConvGeo geo_k = conv_geo(ct, D / 64, L::kKBox);
    const ConvGeo geo_v = conv_geo(ct, D / 128, L::kVBox);
    uint32_t c = 0;
    int segs = 0;
    auto wait_all = [&](uint32_t bar, uint32_t parity, int code) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err, code));
    };
    // One raw item -> its operand stage; rows of keys past the valid count
    // are written as zeros (their P is 0, and 0 * V must stay 0).
    auto convert = [&](bool is_v, int kt) -> bool {
      const int rs = c % NR, os = c % NS;
      if (!wait_all(bar_raw_full(rs), (c / NR) & 1u, kErrWaitKvFull)) return false;
      if (!wait_all(bar_op_empty(os), ((c / NS) & 1u) ^ 1u, kErrWaitKvEmpty)) return false;
      const TileLoc tl = locate_tile(s_tile0, s_valid, nsrc, kt);
      const uint32_t raw = sRaw + rs * L::kRawBytes;
      const uint32_t op = sOp + os * L::kOpBytes;
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      // K: raw [64 keys][D] -> f16 K half, D/64 boxes of [64 rows][128 B];
      // V: raw [128 keys][D/2] -> f16 V half (MN-major), D/128 boxes of
      // [128 keys][128 B].  Either way D/32 chunks per converter thread, in
      // batches of four whose loads are in flight together.
      const ConvGeo& g = is_v ? geo_v : geo_k;
      const int vrows = is_v ? tl.valid : tl.valid - 64 * static_cast<int>(rank);
      const int row_step = is_v ? 64 / (D / 64) : 32 / (D / 64);
      const uint32_t op_step = row_step * 128;
#pragma unroll 1
      for (int m0 = 0; m0 < D / 32; m0 += 4) {
        uint4 x[4];
#pragma unroll
        for (int m = 0; m < 4; ++m)
          x[m] = g.row + (m0 + m) * row_step < vrows ? lds128(raw + g.raw + (m0 + m) * 2048) : zero;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          uint4 lo, hi;
          e4m3x16_to_f16(x[m], lo, hi);
          const uint32_t o = op + (m0 + m) * op_step;
          sts128(o + g.lo, lo);
          sts128(o + g.hi, hi);
        }
      }
      // Generic-proxy smem writes -> visible to the tensor cores (async proxy).
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar_raw_empty(rs));
        mbar_arrive_remote(mapa_shared(bar_op_full(os), 0));
      }
      ++c;
      return true;
    };
    for_each_segment([&](const Segment& sg) -> bool {
      const int n = sg.kt1 - sg.kt0;
      if (n <= 0) return true;
      // Q of this segment: bf16 -> f16 in place (same swizzled positions).
      if (!wait_all(bar_q_raw, segs & 1u, kErrWaitQ)) return false;
      constexpr int kQPer = L::kQBytes / 16 / kConvThreads;
      static_assert(kQPer % 4 == 0, "Q chunks per converter thread");
#pragma unroll 1
      for (int m0 = 0; m0 < kQPer; m0 += 4) {
        uint4 x[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) x[m] = lds128(sQ + (ct + (m0 + m) * kConvThreads) * 16);
#pragma unroll
        for (int m = 0; m < 4; ++m)
          sts128(sQ + (ct + (m0 + m) * kConvThreads) * 16,
                 make_uint4(bf16x2_to_f16x2(x[m].x), bf16x2_to_f16x2(x[m].y), bf16x2_to_f16x2(x[m].z),
                            bf16x2_to_f16x2(x[m].w)));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(bar_q_ready, 0));
      ++segs;
      if (!convert(false, sg.kt0)) return false;
      for (int j = 0; j < n; ++j) {
        if (j + 1 < n && !convert(false, sg.kt0 + j + 1)) return false;
        if (!convert(true, sg.kt0 + j)) return false;
      }
      return true;
    });
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // --------------------------------------------- MMA issuer (leader only) --
    if (leader && lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kPairRows, kTileN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(kPairRows, D, false, true);
      uint32_t c = 0;
      uint32_t J = 0;  // tiles of all earlier segments
      int segs = 0;
      auto qk = [&](uint32_t jg) {
        const uint32_t s_tmem = tmem + kTmemS0 + (jg & 1) * kTileN;
        const int st = c % NS;
        if (!mbar_wait(bar_op_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
        tc_fence_after();
        const uint32_t kbase = sOp + st * L::kOpBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qa = sQ + (kk / 4) * kBoxBytes + (kk % 4) * 32;
          const uint32_t kb = kbase + (kk / 4) * L::kKBox + (kk % 4) * 32;
          umma_ss_pair(s_tmem, make_sw128_desc(qa, 16, 1024), make_sw128_desc(kb, 16, 1024), idesc_qk,
                       kk != 0 ? 1u : 0u);
        }
        umma_commit_pair(bar_op_empty(st), kBothCtas);
        ++c;
        umma_commit_pair(bar_s_full(jg & 1), kBothCtas);
        return true;
      };
      auto pv = [&](uint32_t jg, bool first) {
        if (!mbar_wait(bar_p_full(jg & 1), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitPFull)) return false;
        const int st = c % NS;
        if (!mbar_wait(bar_op_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kTmemS0 + (jg & 1) * kTileN;
        const uint32_t vbase = sOp + st * L::kOpBytes;
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {
          // A = P (TMEM columns of the S buffer, see attn_pair.cuh), B = V
          // half, MN-major: 64-dim chunks 16 KB apart, 8-key groups 1 KB apart.
          const uint32_t a_cols = kk * 8 + (kk >= 4 ? 32 : 0);
          umma_ts_pair(tmem, p_tmem + a_cols, make_sw128_desc(vbase + kk * 2048, L::kVBox, 1024), idesc_pv,
                       (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit_pair(bar_op_empty(st), kBothCtas);
        ++c;
        umma_commit_pair(bar_o(jg & 1), kBothCtas);
        return true;
      };
      for_each_segment([&](const Segment& sg) -> bool {
        if (sg.kt1 <= sg.kt0) return true;
        const uint32_t n = static_cast<uint32_t>(sg.kt1 - sg.kt0);
        // Q of this segment converted in both CTAs.  (O of the previous
        // segment has been read out: its softmax warps release P_0 of this
        // segment only after their epilogue.)
        if (!mbar_wait(bar_q_ready, segs & 1u, abort_flag, p.err, kErrWaitQ)) return false;
        tc_fence_after();
        if (!qk(J)) return false;
        if (n == 1) umma_commit_pair(bar_q_empty, kBothCtas);
        for (uint32_t j = 0; j < n; ++j) {
          if (j + 1 < n) {
            if (!qk(J + j + 1)) return false;
            if (j + 2 == n) umma_commit_pair(bar_q_empty, kBothCtas);  // last QK^T of the segment
          }
          if (!pv(J + j, j == 0)) return false;
        }
        J += n;
        ++segs;
        return true;
      });
      // Drain: completes when every MMA issued above has.
      umma_commit_pair(bar_td, kLeaderCta);
      mbar_wait_teardown(bar_td, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------- softmax / correction / epilogue --
    constexpr int kHalfKeys = kTileN / kSoftmaxWarpgroups;  // 64
    constexpr int kOCols = D / kSoftmaxWarpgroups;
    const int wg = warp >> 2;
    const int row = threadIdx.x & (kTileM - 1);  // == TMEM lane
    const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    // P_j = 2^((s - m_ref) * scale * log2 e) for this warpgroup's 64 keys
    // (ex2.approx on the MUFU), stored as f16 over this warpgroup's S
    // columns; returns the fp32 sum.
    auto make_p = [&](const float* sv, float m, uint32_t t_s) {
      return store_probs<kHalfKeys, true>(sv, m, sl2, t_s + wg * kHalfKeys);
    };
    uint32_t J = 0;
    if (n_kt == 0 && pair < units && kp.sched == kSchedStreamK) {
      // No keys at all (device-length mode): the pair of each unit marks its
      // partial slots empty so the combine ignores them.
      for (int u = pair; u < units; u += gridDim.x >> 1) {
        const int rih = (u % p.m_tiles_per_head) * kPairRows + static_cast<int>(rank) * kTileM + row;
        if (wg == 0 && rih < p.rows_per_head)
          for (int s = 0; s < p.max_segs; ++s)
            p.part_lse[static_cast<size_t>(p.split_base + s) * p.total_rows +
                       static_cast<size_t>(u / p.m_tiles_per_head) * p.rows_per_head + rih] = -INFINITY;
      }
    }
    for_each_segment([&](const Segment& sg) -> bool {
      bool ok = true;
      const int head = sg.unit / p.m_tiles_per_head;
      const int row0 = (sg.unit % p.m_tiles_per_head) * kPairRows + static_cast<int>(rank) * kTileM;
      const int rih = row0 + row;
      const int n = max(0, sg.kt1 - sg.kt0);
      float m_ref = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < n && ok; ++j) {
        const uint32_t jg = J + j;
        const int b = jg & 1;
        const int tile_valid = locate_tile(s_tile0, s_valid, nsrc, sg.kt0 + j).valid;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitSFull));
        if (!ok) break;
        tc_fence_after();
        const uint32_t t_s = t_row + kTmemS0 + b * kTileN;
        float s[kHalfKeys];
        load_scores<kHalfKeys>(t_s + wg * kHalfKeys, tile_valid - wg * kHalfKeys, s);
        const float pmax = row_max(s);
        red[(b * kSoftmaxWarpgroups + wg) * kTileM + row] = pmax;
        mbar_arrive(bar_red(b));
        // Pass 0 (tiles after the first): speculative P with the current
        // reference max, before the other half's max is known (see
        // attn_pair.cuh).  Pass 1: exchange the half maxima; P is recomputed
        // only when some row's max moved past the rescale threshold.  One
        // copy of the exponential code serves both passes (instruction cache).
        float tile_sum = 0.f;
        float alpha = 1.f;
        bool redo = false;
#pragma unroll 1
        for (int pass = j > 0 ? 0 : 1; pass < 2; ++pass) {
          if (pass == 1) {
            ok = __all_sync(0xffffffffu, mbar_wait(bar_red(b), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitRed));
            if (!ok) break;
            const float tmax = fmaxf(pmax, red[(b * kSoftmaxWarpgroups + (wg ^ 1)) * kTileM + row]);
            const bool need = (tmax - m_ref) * sl2 > kRescaleThreshold;  // always true on the first tile
            redo = __any_sync(0xffffffffu, need);
            if (need) {
              alpha = ex2_approx((m_ref - tmax) * sl2);  // 0 on the first tile
              m_ref = tmax;
              l *= alpha;
            }
            if (!redo) break;
          }
          tile_sum = make_p(s, m_ref, t_s);
        }
        if (!ok) break;
        l += tile_sum;
        if (j > 0 && redo) {
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_o((jg - 1) & 1), ((jg - 1) >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
          if (!ok) break;
          tc_fence_after();
          rescale_o<kOCols>(t_row + wg * kOCols, alpha);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar_p_full(b), 0));
      }
      if (ok && n > 0) {
        const uint32_t jl = J + n - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o(jl & 1), (jl >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
      }
      ok = named_bar_and(1, kSoftmaxThreads, ok && (*abort_flag == 0));
      if (!ok) return false;
      J += n;
      const bool live = rih < p.rows_per_head;
      const size_t grow = static_cast<size_t>(head) * p.rows_per_head + rih;
      const bool final_out = p.final_ok && sg.nseg == 1;
      if (!final_out && sg.slot >= p.max_segs) {  // the host's slot bound does not hold: keep the buffers intact
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kErrSchedule);
        return true;
      }
      if (n <= 0) {
        // Empty split (device-length mode): weight zero.
        if (!final_out && live && wg == 0)
          p.part_lse[static_cast<size_t>(p.split_base + sg.slot) * p.total_rows + grow] = -INFINITY;
        return true;
      }
      tc_fence_after();
      red[wg * kTileM + row] = l;
      named_bar_sync(2, kSoftmaxThreads);
      const float l_tot = l + red[(wg ^ 1) * kTileM + row];
      // Both halves read: the next segment may reuse the exchange slots.
      named_bar_sync(2, kSoftmaxThreads);
      const float inv_l = 1.f / l_tot;
      if (final_out) {
        store_o_bf16<kOCols>(t_row + wg * kOCols, inv_l, p.out + grow * D + wg * kOCols, live);
      } else {
        const size_t split_idx = static_cast<size_t>(p.split_base + sg.slot);
        store_o_partial<kOCols>(t_row + wg * kOCols, inv_l,
                                p.part_o + (split_idx * p.total_rows + grow) * D + wg * kOCols, live);
        if (live && wg == 0) {
          p.part_lse[split_idx * p.total_rows + grow] = m_ref * sl2 + __log2f(l_tot);
          // The segment that ends a unit marks the unit's unused slots empty.
          if (sg.last)
            for (int s = sg.nseg; s < p.max_segs; ++s)
              p.part_lse[static_cast<size_t>(p.split_base + s) * p.total_rows + grow] = -INFINITY;
        }
      }
      return true;
    });
  }

  // Both CTAs: the leader's MMAs (which read the peer's smem and TMEM) are
  // drained, every TMEM read of either CTA is done.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace pcp
