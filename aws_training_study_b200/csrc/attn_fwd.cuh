// History-attention forward for one launch: every (KV head, 128-row Q tile,
// key split) work unit computes softmax(Q K^T * scale) V over a contiguous
// range of 128-key tiles of a dense, compacted bf16 K/V buffer.
//
// Replaces the NKI kernel body of the reference (pcp_attention/kernel.py:
// 84-554).  Stage map, reference -> here:
//   resident Q load + pre-scale (kernel.py:141-173) -> TMA load of a 128-row
//       bf16 Q tile into 128B-swizzled smem once per CTA; scale applied in fp32.
//   K/V resident load (kernel.py:295-339) -> TMA producer warp streaming
//       32 KB half-tiles ([128 keys, 128 dims]) through an NS-deep smem ring.
//   QK^T into PSUM (kernel.py:383-394) -> tcgen05.mma kind::f16, M=128,
//       N=128 keys, fp32 accumulator S in TMEM (two buffers).
//   mask + max + fused exp/sum (kernel.py:396-437) -> softmax warpgroup, one
//       thread per row (TMEM lane), exp2 with fp32 running max/sum; keys past
//       the valid count in the final tile are -inf.
//   P transpose (kernel.py:439-462) -> none: P is written back to TMEM as bf16
//       (aliasing S) and used as the A operand of the PV MMA.
//   PV + rescale (kernel.py:464-511) -> tcgen05.mma A=P (TMEM), B=V (smem,
//       MN-major), O accumulates in TMEM across all tiles; O is rescaled in
//       TMEM only when the running max grows by more than 2^8 (lazy rescale).
//   finalise/store (kernel.py:516-553) -> O/l in fp32, bf16 via swizzled smem
//       + TMA store, or fp32 partial + log2-sum-exp for the split combine.
//
// Thread roles (320 threads, 1 CTA per SM):
//   warps 0-7 softmax / correction / epilogue in two warpgroups: warpgroup w
//     owns key columns [64w, 64w+64) of every S tile and head-dim columns
//     [w*D/2, (w+1)*D/2) of O; the two exchange their partial row max through
//     shared memory once per tile, which halves the per-tile latency of the
//     softmax that sits between the QK^T and PV MMAs,
//   warp 8 TMA producer, warp 9 TMEM allocator and single-thread MMA issuer.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include "ptx.cuh"

namespace pcp {

constexpr int kTileM = 128;       // query rows per CTA (TMEM lanes)
constexpr int kTileN = 128;       // keys per tile
constexpr int kHalfD = 128;       // head dims per smem stage
constexpr int kBoxCols = 64;      // bf16 columns per 128B-swizzled TMA box
constexpr int kBoxBytes = 128 * 128;  // one box: 128 rows x 128 B
constexpr int kStageBytes = 2 * kBoxBytes;  // [128 keys, 128 dims] bf16
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
  int write_final;       // 1: bf16 O via TMA; 0: fp32 partial O + lse
  float* part_o;         // [splits][total_rows][D]
  float* part_lse;       // [splits][total_rows]
  int* err;              // device error word
};

template <int D>
struct AttnSmem {
  static constexpr int kHalves = D / kHalfD;
  static constexpr int kStages = (D == 256) ? 5 : 6;
  static constexpr int kQBytes = D * 2 * kTileM;  // = D/64 boxes
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  // barriers: q_full, kv_full[NS], kv_empty[NS], s_full[2], p_full[2], o_done,
  // teardown, red[2] (row-max exchange between the softmax warpgroups)
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 1 + 1 + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  // Row-max exchange between the softmax warpgroups: [tile parity][wg][row].
  static constexpr int kRedOff = kMiscOff + 16;
  static constexpr int kBytes = kRedOff + 2 * kSoftmaxWarpgroups * kTileM * 4;
  // The dynamic smem base is declared 1024-aligned (128B-swizzle atoms); the
  // kernel verifies it and reports an error instead of running misaligned.
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 232448, "exceeds the 227 KB of shared memory per CTA");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    const AttnParams p) {
  using L = AttnSmem<D>;
  constexpr int NS = L::kStages;
  constexpr int NH = L::kHalves;

  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // uniform across the CTA: nothing has started yet
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, kErrSmemAlign);
    return;
  }
  const uint32_t sQ = sbase + L::kQOff;
  const uint32_t sStage = sbase + L::kStageOff;
  const uint32_t bars = sbase + L::kBarOff;
  const uint32_t bar_q = bars;
  auto bar_kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto bar_kv_empty = [&](int s) { return bars + 8u * (1 + NS + s); };
  auto bar_s_full = [&](int b) { return bars + 8u * (1 + 2 * NS + b); };
  auto bar_p_full = [&](int b) { return bars + 8u * (3 + 2 * NS + b); };
  const uint32_t bar_o = bars + 8u * (5 + 2 * NS);
  const uint32_t bar_td = bars + 8u * (6 + 2 * NS);
  auto bar_red = [&](int b) { return bars + 8u * (7 + 2 * NS + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int head = blockIdx.x / p.m_tiles_per_head;
  const int mt = blockIdx.x % p.m_tiles_per_head;
  const int split = blockIdx.y;
  const int n_key_tiles = (p.num_keys + kTileN - 1) / kTileN;
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(kt0 + p.tiles_per_split, n_key_tiles);
  const int n = kt1 - kt0;  // >= 1 by construction on the host

  if (warp == kProducerWarp && lane == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), kSoftmaxThreads);
    }
    mbar_init(bar_o, 1);
    mbar_init(bar_td, 1);
    mbar_init(bar_red(0), kSoftmaxThreads);
    mbar_init(bar_red(1), kSoftmaxThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar_q, L::kQBytes);
      for (int b = 0; b < D / kBoxCols; ++b)
        tma_load_3d(sQ + b * kBoxBytes, &tm_q, b * kBoxCols, mt * kTileM, head, bar_q);
      uint32_t c = 0;
      bool ok = true;
      auto issue = [&](const CUtensorMap* tm, int kt, int half) {
        const int st = c % NS;
        const uint32_t ph = (c / NS) & 1u;
        if (!mbar_wait(bar_kv_empty(st), ph ^ 1u, abort_flag, p.err, kErrWaitKvEmpty)) return false;
        const uint32_t dst = sStage + st * kStageBytes;
        mbar_arrive_expect_tx(bar_kv_full(st), kStageBytes);
        tma_load_3d(dst, tm, half * kHalfD, kt * kTileN, head, bar_kv_full(st));
        tma_load_3d(dst + kBoxBytes, tm, half * kHalfD + kBoxCols, kt * kTileN, head, bar_kv_full(st));
        ++c;
        return true;
      };
      for (int h = 0; h < NH && ok; ++h) ok = issue(&tm_k, kt0, h);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n)
          for (int h = 0; h < NH && ok; ++h) ok = issue(&tm_k, kt0 + j + 1, h);
        for (int h = 0; h < NH && ok; ++h) ok = issue(&tm_v, kt0 + j, h);
      }
      if (!ok) {
        // Abort: let the copies already in flight land before the CTA exits.
        for (uint32_t i = (c > (uint32_t)NS ? c - NS : 0); i < c; ++i)
          mbar_wait_teardown(bar_kv_full(i % NS), (i / NS) & 1u);
        mbar_wait_teardown(bar_q, 0);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // -------------------------------------------------------- MMA issuer --
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kTileM, kTileN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kTileM, kHalfD, false, true);
      uint32_t c = 0;
      bool ok = mbar_wait(bar_q, 0, abort_flag, p.err, kErrWaitQ);
      tc_fence_after();
      // S[j&1] = Q K_j^T, accumulated over the head dim in 16-wide k-steps.
      auto qk = [&](int j) {
        const uint32_t s_tmem = tmem + kTmemS0 + (j & 1) * kTileN;
        for (int h = 0; h < NH; ++h) {
          const int st = c % NS;
          if (!mbar_wait(bar_kv_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
          tc_fence_after();
          const uint32_t kbase = sStage + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kHalfD / 16; ++kk) {
            const uint32_t qa = sQ + (h * 2 + kk / 4) * kBoxBytes + (kk % 4) * 32;
            const uint32_t kb = kbase + (kk / 4) * kBoxBytes + (kk % 4) * 32;
            umma_ss(s_tmem, make_sw128_desc(qa, 16, 1024), make_sw128_desc(kb, 16, 1024), idesc_qk,
                    (h | kk) != 0);
          }
          umma_commit(bar_kv_empty(st));
          ++c;
        }
        umma_commit(bar_s_full(j & 1));
        return true;
      };
      // O[:, half] (+)= P_j V_j[:, half]; P_j read from TMEM (aliases S[j&1]).
      auto pv = [&](int j) {
        if (!mbar_wait(bar_p_full(j & 1), (j >> 1) & 1u, abort_flag, p.err, kErrWaitPFull)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kTmemS0 + (j & 1) * kTileN;
        for (int h = 0; h < NH; ++h) {
          const int st = c % NS;
          if (!mbar_wait(bar_kv_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
          tc_fence_after();
          const uint32_t vbase = sStage + st * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            // V tile is MN-major: 64-dim chunks 16 KB apart (LBO), 8-key
            // groups 1 KB apart (SBO); a 16-key step is 2 KB.
            umma_ts(tmem + h * kHalfD, p_tmem + kk * 8, make_sw128_desc(vbase + kk * 2048, kBoxBytes, 1024),
                    idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_kv_empty(st));
          ++c;
        }
        umma_commit(bar_o);
        return true;
      };
      if (ok) ok = qk(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = qk(j + 1);
        if (ok) ok = pv(j);
      }
      // Drain: the teardown barrier completes when every MMA issued above has.
      umma_commit(bar_td);
      mbar_wait_teardown(bar_td, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------- softmax / correction / epilogue --
    // Thread = query row (TMEM lane); warpgroup `wg` owns S key columns
    // [64 wg, 64 wg + 64) and O columns [wg D/2, (wg+1) D/2).  Both warpgroups
    // keep identical running maxima (they combine the same tile max), and
    // each keeps a partial row sum over its own columns.
    constexpr int kHalfKeys = kTileN / kSoftmaxWarpgroups;  // 64
    constexpr int kOCols = D / kSoftmaxWarpgroups;          // 128 or 64
    const int wg = warp >> 2;
    const int row = threadIdx.x & (kTileM - 1);  // == TMEM lane
    const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY;  // raw-score running reference max
    float l = 0.f;            // partial row sum over this warpgroup's columns
    bool ok = n > 0;
    // Every wait result is made warp-uniform (__all_sync) so that the
    // warp-collective tcgen05.ld/st below never run with part of a warp.
    for (int j = 0; j < n && ok; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (j >> 1) & 1u, abort_flag, p.err, kErrWaitSFull));
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = t_row + kTmemS0 + b * kTileN;
      float s[kHalfKeys];
      tmem_ld32(t_s + wg * kHalfKeys, s);
      tmem_ld32(t_s + wg * kHalfKeys + 32, s + 32);
      tmem_wait_ld();
      const int valid = p.num_keys - (kt0 + j) * kTileN - wg * kHalfKeys;
      if (valid < kHalfKeys) {
#pragma unroll
        for (int i = 0; i < kHalfKeys; ++i)
          if (i >= valid) s[i] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int i = 4; i < kHalfKeys; i += 4) {
        mx0 = fmaxf(mx0, s[i]);
        mx1 = fmaxf(mx1, s[i + 1]);
        mx2 = fmaxf(mx2, s[i + 2]);
        mx3 = fmaxf(mx3, s[i + 3]);
      }
      const float pmax = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      // Exchange partial maxima through smem, double-buffered by tile parity
      // (a warpgroup can be at most one tile ahead of the other), with a
      // bounded mbarrier wait.  After it both warpgroups have finished
      // reading S_j, so the P stores below may overwrite any of its columns.
      red[(b * kSoftmaxWarpgroups + wg) * kTileM + row] = pmax;
      mbar_arrive(bar_red(b));
      ok = __all_sync(0xffffffffu, mbar_wait(bar_red(b), (j >> 1) & 1u, abort_flag, p.err, kErrWaitRed));
      if (!ok) break;
      const float tmax = fmaxf(pmax, red[(b * kSoftmaxWarpgroups + (wg ^ 1)) * kTileM + row]);
      const bool need = (tmax - m_ref) * sl2 > kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = ex2_approx((m_ref - tmax) * sl2);  // 0 on the first tile
        m_ref = tmax;
        l *= alpha;
      }
      const float neg = -m_ref * sl2;
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c2 = 0; c2 < kHalfKeys / 32; ++c2) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(s[c2 * 32 + 2 * i], sl2, neg));
          const float p1 = ex2_approx(fmaf(s[c2 * 32 + 2 * i + 1], sl2, neg));
          sum0 += p0;
          sum1 += p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        // P (bf16 pairs) of keys [64 wg + 32 c2, +32) -> TMEM columns
        // [32 wg + 16 c2, +16) of the S buffer: the PV MMA's A operand.
        tmem_st16(t_s + wg * (kHalfKeys / 2) + c2 * 16, pk);
      }
      tmem_wait_st();
      l += sum0 + sum1;
      if (j > 0) {
        // PV_{j-1} must be complete before O may be rescaled (and before the
        // MMA warp may start PV_j, which it only does after p_full[j]).
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (j - 1) & 1u, abort_flag, p.err, kErrWaitODone));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < kOCols / 32; ++c) {
            float o[32];
            const uint32_t t_o = t_row + wg * kOCols + c * 32;
            tmem_ld32(t_o, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(t_o, o);
          }
          tmem_wait_st();
        }
      }
      tc_fence_before();
      mbar_arrive(bar_p_full(b));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_o, (n - 1) & 1u, abort_flag, p.err, kErrWaitODone));
    // All softmax threads reach this barrier (every wait above is bounded);
    // after it the epilogue decision is uniform across them, and no thread
    // still reads the row-max exchange buffer.
    ok = named_bar_and(1, kSoftmaxThreads, ok && (*abort_flag == 0));
    if (ok) {
      tc_fence_after();
      red[wg * kTileM + row] = l;
      named_bar_sync(2, kSoftmaxThreads);
      const float l_tot = l + red[(wg ^ 1) * kTileM + row];
      const float inv_l = 1.f / l_tot;
      if (p.write_final) {
        // bf16 O -> Q's smem (all MMAs are complete) in the 128B-swizzled box
        // layout the O tensor map expects, then one thread issues TMA stores.
#pragma unroll 1
        for (int c = 0; c < kOCols / 32; ++c) {
          float o[32];
          const int col = wg * kOCols + c * 32;
          tmem_ld32(t_row + col, o);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(o[2 * i] * inv_l, o[2 * i + 1] * inv_l);
          const int box = col / kBoxCols;
          uint8_t* rowp = smem + L::kQOff + box * kBoxBytes + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = ((col % kBoxCols) / 8) + q;
            const int phys = chunk ^ (row & 7);
            *reinterpret_cast<uint4*>(rowp + phys * 16) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(3, kSoftmaxThreads);
        if (threadIdx.x == 0) {
          for (int box = 0; box < D / kBoxCols; ++box)
            tma_store_3d(&tm_o, sQ + box * kBoxBytes, box * kBoxCols, mt * kTileM, head);
          tma_store_commit();
          tma_store_wait0();
        }
      } else {
        const int rih = mt * kTileM + row;
        const size_t split_idx = static_cast<size_t>(p.split_base + split);
        const size_t grow = static_cast<size_t>(head) * p.rows_per_head + rih;
        float* dst = p.part_o + (split_idx * p.total_rows + grow) * D + wg * kOCols;
        const bool live = rih < p.rows_per_head;
#pragma unroll 1
        for (int c = 0; c < kOCols / 32; ++c) {
          float o[32];
          tmem_ld32(t_row + wg * kOCols + c * 32, o);
          tmem_wait_ld();
          if (live) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + c * 32 + i) =
                  make_float4(o[i] * inv_l, o[i + 1] * inv_l, o[i + 2] * inv_l, o[i + 3] * inv_l);
          }
        }
        if (live && wg == 0) p.part_lse[split_idx * p.total_rows + grow] = m_ref * sl2 + __log2f(l_tot);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace pcp
