// History-attention forward on CTA pairs (tcgen05 cta_group::2).
//
// Stages, numerics and the map to the reference's NKI kernel
// (pcp_attention/kernel.py:84-554) are in attn_common.cuh.  Every work unit
// is a cluster of two CTAs on two SMs that share one 256-row MMA:
//   * CTA r of the pair owns query rows [256 t + 128 r, +128) of one KV head:
//     its Q rows in its smem, its S/P and O rows in its TMEM.
//   * QK^T: S[256, 128 keys] = Q K^T with B = K split by keys: CTA r holds
//     keys [64 r, 64 r + 64) of the tile ([64 keys, D] in smem).
//   * PV:   O[256, D] += P V with B = V split by head dim: CTA r holds
//     V[128 keys, D/2 * r .. +D/2] (MN-major).  A = P from each CTA's TMEM.
//   * The leader (rank 0) issues every MMA; completion is multicast to both
//     CTAs' mbarriers.  Both CTAs' TMA loads count their bytes on the
//     leader's barriers; both softmax warpgroups arrive on the leader's P
//     barrier (one arrive per warp).
// Per CTA and 128-key tile this moves 64 KB of K/V through TMA instead of
// 128 KB, and the tensor cores read 96 KB + 32 KB of smem operands instead
// of 128 KB + 64 KB, so the smem ring holds 2.5 tiles of look-ahead.
// No TMA multicast is used: each CTA loads only its own smem.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "attn_common.cuh"
#include "attn_softmax.cuh"
#include "ptx.cuh"

namespace pcp {

// Thread roles of the dense-K/V pair kernels (this file and
// attn_pair_sk.cuh) for head dim D: kWG softmax warpgroups, each owning
// kTileN / kWG keys of every row of a tile and D / kWG columns of O, then the
// TMA warp and the MMA warp.  Two at both head dims: four (32 keys each) ran
// configs[4]'s D = 128 shape at 1000 TFLOP/s against 1049 with two -- the
// softmax there is bound by its instruction throughput per sub-partition,
// which more warps do not raise, not by one row's latency.
template <int D>
struct PairRoles {
  static constexpr int kWG = 2;
  static constexpr int kSoftmaxThreads = 128 * kWG;
  static constexpr int kSoftmaxWarps = kSoftmaxThreads / 32;
  static constexpr int kThreads = kSoftmaxThreads + 64;
  static constexpr int kProducerWarp = kSoftmaxWarps;
  static constexpr int kMmaWarp = kProducerWarp + 1;
  static constexpr int kKeys = kTileN / kWG;  // keys per softmax thread per tile
  static constexpr int kOCols = D / kWG;      // O columns per softmax thread
  // TMEM column of the P (16-bit, two per column) of keys [16 kk, +16): each
  // warpgroup packs its keys into the first half of its own S columns.
  static __device__ __forceinline__ uint32_t p_col(int kk) {
    return static_cast<uint32_t>((16 * kk / kKeys) * kKeys + (16 * kk % kKeys) / 2);
  }
};

template <int D>
struct PairSmem {
  static constexpr int kQBytes = D * 2 * kTileM;           // own 128 rows (D/64 boxes of 16 KB)
  static constexpr int kStageBytes = 128 * D;              // K half [64, D] or V half [128, D/2], bf16
  static constexpr int kKBox = 64 * 128;                   // K box: 64 rows x 128 B
  static constexpr int kVBox = 128 * 128;                  // V box: 128 rows x 128 B
  static constexpr int kStages = (D == 256) ? 5 : 12;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  // q_full, kv_full[NS], kv_empty[NS], s_full[2], p_full[2], o_done[2], teardown, red[2]
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1 + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kRedOff = kMiscOff + 16;
  static constexpr int kBytes = kRedOff + 2 * PairRoles<D>::kWG * kTileM * 4;
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 232448, "exceeds the 227 KB of shared memory per CTA");
};

constexpr int kPairRows = 2 * kTileM;
constexpr uint16_t kBothCtas = 0x3;
constexpr uint16_t kLeaderCta = 0x1;
constexpr int kSoftmaxWarps = kSoftmaxThreads / 32;

// p.m_tiles_per_head counts 256-row pair tiles here.
template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairRoles<D>::kThreads, 1)
    attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                         const AttnParams p) {
  using L = PairSmem<D>;
  using R = PairRoles<D>;
  constexpr int NS = L::kStages;
  constexpr int kWG = R::kWG;

  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // identical in both CTAs: neither starts
    if (threadIdx.x == 0 && p.err) atomicCAS(p.err, 0, kErrSmemAlign);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t sQ = sbase + L::kQOff;
  const uint32_t sStage = sbase + L::kStageOff;
  const uint32_t bars = sbase + L::kBarOff;
  const uint32_t bar_q = bars;
  auto bar_kv_full = [&](int s) { return bars + 8u * (1 + s); };
  auto bar_kv_empty = [&](int s) { return bars + 8u * (1 + NS + s); };
  auto bar_s_full = [&](int b) { return bars + 8u * (1 + 2 * NS + b); };
  auto bar_p_full = [&](int b) { return bars + 8u * (3 + 2 * NS + b); };
  // o_done[b] completes once per PV_j with j % 2 == b (phase j / 2).
  auto bar_o = [&](int b) { return bars + 8u * (5 + 2 * NS + b); };
  const uint32_t bar_td = bars + 8u * (7 + 2 * NS);
  auto bar_red = [&](int b) { return bars + 8u * (8 + 2 * NS + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;
  const int head = pair / p.m_tiles_per_head;
  const int pt = pair % p.m_tiles_per_head;
  const int row0 = pt * kPairRows + static_cast<int>(rank) * kTileM;  // first query row of this CTA
  const int split = blockIdx.y;
  const int num_keys = p.num_keys_dev ? min(max(*p.num_keys_dev, 0), p.num_keys) : p.num_keys;
  int n_key_tiles = (num_keys + kTileN - 1) / kTileN;
  if (p.causal) {
    // Last key tile any of the pair's 256 rows can see (rows past the end
    // are padding; a tile that wraps into the next Q head holds Qloc - 1).
    const int r_first = pt * kPairRows;
    const int r_last = min(r_first + kPairRows, p.rows_per_head) - 1;
    const int i_max = (r_first / p.q_local_len != r_last / p.q_local_len) ? p.q_local_len - 1 : r_last % p.q_local_len;
    const int g_max = striped_position(i_max, p.stripe_ranks, p.stripe_width, p.stripe_rank);
    n_key_tiles = min(n_key_tiles, g_max / kTileN + 1);
  }
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(kt0 + p.tiles_per_split, n_key_tiles);
  const int n = kt1 - kt0;  // >= 1 on the host plan; <= 0 only for an empty split in device-length mode

  if (warp == R::kProducerWarp && lane == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_s_full(b), 1);
      mbar_init(bar_p_full(b), 2 * R::kSoftmaxWarps);  // one arrive per softmax warp of both CTAs
    }
    mbar_init(bar_o(0), 1);
    mbar_init(bar_o(1), 1);
    mbar_init(bar_td, 1);
    mbar_init(bar_red(0), R::kSoftmaxThreads);
    mbar_init(bar_red(1), R::kSoftmaxThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == R::kMmaWarp) {
    tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == R::kProducerWarp) {
    // ------------------------------------------------------ TMA producer --
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      if (leader) mbar_arrive_expect_tx(bar_q, 2 * L::kQBytes);
      const uint32_t q_lead = mapa_shared(bar_q, 0);
      for (int b = 0; b < D / kBoxCols; ++b)
        tma_load_3d_pair(sQ + b * kBoxBytes, &tm_q, b * kBoxCols, row0, head, q_lead);
      uint32_t c = 0;
      bool ok = true;
      // Item order = MMA consumption order: K_0, then (K_{j+1}, V_j) per tile.
      auto issue = [&](bool is_v, int kt) {
        const int st = c % NS;
        if (!mbar_wait(bar_kv_empty(st), ((c / NS) & 1u) ^ 1u, abort_flag, p.err, kErrWaitKvEmpty)) return false;
        if (leader) mbar_arrive_expect_tx(bar_kv_full(st), 2 * L::kStageBytes);
        const uint32_t full_lead = mapa_shared(bar_kv_full(st), 0);
        const uint32_t dst = sStage + st * L::kStageBytes;
        if (!is_v) {
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d_pair(dst + b * L::kKBox, &tm_k, b * kBoxCols, kt * kTileN + static_cast<int>(rank) * 64,
                             head, full_lead);
        } else {
          for (int b = 0; b < D / 2 / kBoxCols; ++b)
            tma_load_3d_pair(dst + b * L::kVBox, &tm_v, static_cast<int>(rank) * (D / 2) + b * kBoxCols,
                             kt * kTileN, head, full_lead);
        }
        ++c;
        return true;
      };
      ok = issue(false, kt0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = issue(false, kt0 + j + 1);
        if (ok) ok = issue(true, kt0 + j);
      }
      if (!ok) {
        // Abort: let copies already in flight land before the CTA exits.
        if (leader) {
          for (uint32_t i = (c > (uint32_t)NS ? c - NS : 0); i < c; ++i)
            mbar_wait_teardown(bar_kv_full(i % NS), (i / NS) & 1u);
          mbar_wait_teardown(bar_q, 0);
        } else {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == R::kMmaWarp) {
    // --------------------------------------------- MMA issuer (leader only) --
    if (leader && lane == 0 && n > 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kPairRows, kTileN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kPairRows, D, false, true);
      uint32_t c = 0;
      bool ok = mbar_wait(bar_q, 0, abort_flag, p.err, kErrWaitQ);
      tc_fence_after();
      auto qk = [&](int j) {
        const uint32_t s_tmem = tmem + kTmemS0 + (j & 1) * kTileN;
        const int st = c % NS;
        if (!mbar_wait(bar_kv_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
        tc_fence_after();
        const uint32_t kbase = sStage + st * L::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qa = sQ + (kk / 4) * kBoxBytes + (kk % 4) * 32;
          const uint32_t kb = kbase + (kk / 4) * L::kKBox + (kk % 4) * 32;
          umma_ss_pair(s_tmem, make_sw128_desc(qa, 16, 1024), make_sw128_desc(kb, 16, 1024), idesc_qk,
                       kk != 0 ? 1u : 0u);
        }
        umma_commit_pair(bar_kv_empty(st), kBothCtas);
        ++c;
        umma_commit_pair(bar_s_full(j & 1), kBothCtas);
        return true;
      };
      auto pv = [&](int j) {
        if (!mbar_wait(bar_p_full(j & 1), (j >> 1) & 1u, abort_flag, p.err, kErrWaitPFull)) return false;
        const int st = c % NS;
        if (!mbar_wait(bar_kv_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kTmemS0 + (j & 1) * kTileN;
        const uint32_t vbase = sStage + st * L::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {
          // A = P: each softmax warpgroup packed its keys into the first half
          // of its own S columns (R::p_col); 16 keys = 8 columns per step.
          // B = V half, MN-major: 64-dim chunks 16 KB apart (LBO), 8-key
          // groups 1 KB apart (SBO); a 16-key step is 2 KB.
          const uint32_t a_cols = R::p_col(kk);
          umma_ts_pair(tmem, p_tmem + a_cols, make_sw128_desc(vbase + kk * 2048, L::kVBox, 1024), idesc_pv,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_pair(bar_kv_empty(st), kBothCtas);
        ++c;
        umma_commit_pair(bar_o(j & 1), kBothCtas);
        return true;
      };
      if (ok) ok = qk(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) ok = qk(j + 1);
        if (ok) ok = pv(j);
      }
      // Drain: completes when every MMA issued above has.
      umma_commit_pair(bar_td, kLeaderCta);
      mbar_wait_teardown(bar_td, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------- softmax / correction / epilogue --
    constexpr int kHalfKeys = R::kKeys;  // keys of this warpgroup per tile
    constexpr int kOCols = R::kOCols;
    const int wg = warp >> 2;
    const int row = threadIdx.x & (kTileM - 1);  // == TMEM lane
    const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    // Keys this row may see: all valid keys, or (causal) those up to its own
    // global position -- at least key 0, so the first tile is never empty.
    int key_limit = num_keys;
    if (p.causal)
      key_limit = min(key_limit, striped_position((row0 + row) % p.q_local_len, p.stripe_ranks, p.stripe_width,
                                                  p.stripe_rank) + 1);
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = n > 0;
    // P_j = 2^((s - m_ref) * scale * log2 e) for this warpgroup's 64 keys
    // (ex2.approx on the MUFU; moving a share of them to an FMA-pipe
    // polynomial measured slower at both head dims).  Stores P (bf16) over
    // this warpgroup's S columns and returns the fp32 sum.
    // P of keys [64 wg + 32 c2, +32) goes to TMEM columns [64 wg + 16 c2, +16):
    // inside this warpgroup's own S columns, so the stores never touch S
    // values the other warpgroup has yet to read.
    auto make_p = [&](const float* sv, float m, uint32_t t_s) {
      return store_probs<kHalfKeys>(sv, m, sl2, t_s + wg * kHalfKeys);
    };
    for (int j = 0; j < n && ok; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (j >> 1) & 1u, abort_flag, p.err, kErrWaitSFull));
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_s = t_row + kTmemS0 + b * kTileN;
      float s[kHalfKeys];
      load_scores<kHalfKeys>(t_s + wg * kHalfKeys, key_limit - (kt0 + j) * kTileN - wg * kHalfKeys, s);
      const float pmax = row_max(s);
      // Publish this half's max (double-buffered by tile parity; a
      // warpgroup is at most one tile ahead of the other).
      red[(b * kWG + wg) * kTileM + row] = pmax;
      mbar_arrive(bar_red(b));
      // Tiles after the first: compute P with the current reference max
      // before the other half's max is known -- it only matters when the
      // row max moved by more than the rescale threshold, which is rare.
      float tile_sum = 0.f;
      if (j > 0) tile_sum = make_p(s, m_ref, t_s);
      ok = __all_sync(0xffffffffu, mbar_wait(bar_red(b), (j >> 1) & 1u, abort_flag, p.err, kErrWaitRed));
      if (!ok) break;
      float tmax = pmax;
#pragma unroll
      for (int w = 1; w < kWG; ++w) tmax = fmaxf(tmax, red[(b * kWG + (wg ^ w)) * kTileM + row]);
      const bool need = (tmax - m_ref) * sl2 > kRescaleThreshold;  // always true on the first tile
      const bool redo = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (need) {
        alpha = ex2_approx((m_ref - tmax) * sl2);  // 0 on the first tile
        m_ref = tmax;
        l *= alpha;
      }
      if (redo) tile_sum = make_p(s, m_ref, t_s);
      l += tile_sum;
      // O is rescaled only when the reference max moved (rare): then PV_{j-1}
      // must be complete first.  Otherwise P_j is released at once, so the
      // MMA warp can issue PV_j without waiting for PV_{j-1} to finish.
      // (s_full[j] already implies PV_{j-2} is complete: QK_j was issued
      // after it, and tcgen05 MMAs complete in issue order.)
      if (j > 0 && redo) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(bar_o((j - 1) & 1), ((j - 1) >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
        if (!ok) break;
        tc_fence_after();
        rescale_o<kOCols>(t_row + wg * kOCols, alpha);
      }
      // One arrive per warp on the leader's P barrier (all lanes' TMEM stores
      // are complete: tcgen05.wait::st is warp-collective).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(bar_p_full(b), 0));
    }
    if (ok)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar_o((n - 1) & 1), ((n - 1) >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
    ok = named_bar_and(1, R::kSoftmaxThreads, ok && (*abort_flag == 0));
    if (ok) {
      tc_fence_after();
      red[wg * kTileM + row] = l;
      named_bar_sync(2, R::kSoftmaxThreads);
      float l_tot = l;
#pragma unroll
      for (int w = 1; w < kWG; ++w) l_tot += red[(wg ^ w) * kTileM + row];
      const float inv_l = 1.f / l_tot;
      if (p.write_final) {
        // bf16 O through the Q buffer (every QK^T is complete) and a TMA store.
        stage_o_sw128<kOCols>(t_row + wg * kOCols, inv_l, smem + L::kQOff, kBoxBytes, wg * kOCols, row);
        fence_proxy_async_smem();
        named_bar_sync(3, R::kSoftmaxThreads);
        if (threadIdx.x == 0 && row0 < p.rows_per_head) {  // no store of a tile wholly past the rows
          for (int box = 0; box < D / kBoxCols; ++box)
            tma_store_3d(&tm_o, sQ + box * kBoxBytes, box * kBoxCols, row0, head);
          tma_store_commit();
          tma_store_wait0();
        }
      } else {
        const int rih = row0 + row;
        const size_t split_idx = static_cast<size_t>(p.split_base + split);
        const size_t grow = static_cast<size_t>(head) * p.rows_per_head + rih;
        float* dst = p.part_o + (split_idx * p.total_rows + grow) * D + wg * kOCols;
        const bool live = rih < p.rows_per_head;
        store_o_partial<kOCols>(t_row + wg * kOCols, inv_l, dst, live);
        if (live && wg == 0) p.part_lse[split_idx * p.total_rows + grow] = m_ref * sl2 + __log2f(l_tot);
      }
    } else if (n <= 0 && !p.write_final && wg == 0) {
      // Empty split (device-length mode): weight zero in the combine.
      const int rih = row0 + row;
      if (rih < p.rows_per_head)
        p.part_lse[static_cast<size_t>(p.split_base + split) * p.total_rows +
                   static_cast<size_t>(head) * p.rows_per_head + rih] = -INFINITY;
    }
  }

  // Both CTAs: the leader's MMAs (which read the peer's smem and TMEM) are
  // drained, every TMEM read and TMA store of either CTA is done.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (warp == R::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace pcp
