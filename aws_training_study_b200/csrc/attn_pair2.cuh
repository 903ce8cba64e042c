// History attention at head dim 128 on CTA pairs with two query tiles in
// flight (ping-pong).
//
// At D = 128 one 128-key tile costs the pair ~730 tensor cycles for QK^T and
// as many for PV, while its softmax spends ~1150 cycles of one SM
// sub-partition's XU pipe (ex2 and the bf16 packing of P, measured with
// ncu): with one query tile the softmax of tile j only overlaps QK^T of tile
// j+1, and the tensor pipe idles for the rest.  Here a pair holds two
// 256-row query tiles, A and B, of the same KV head, and every K/V tile is
// used by both.  The MMA warp issues, per key tile j,
//     PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1),
// so the softmax of A(j+1) overlaps PV_B(j) and QK_B(j+1), and that of B(j+1)
// overlaps PV_A(j+1) and QK_A(j+2): two MMAs of slack each, and the two
// softmaxes run on different warps.  TMEM (512 columns): O_A [0,128),
// O_B [128,256), S_A [256,384), S_B [384,512) -- one S buffer per tile.
// Because the tensor pipe completes MMAs in issue order, "S_A(j+1) ready"
// also means PV_A(j) is done, so a rare O rescale needs no further wait.
//
// The rest is attn_fwd_pair_kernel's (attn_pair.cuh): CTA r of the pair owns
// rows [128 r, +128) of each tile (its Q in its smem, its S/P and O in its
// TMEM), B = K split by keys / V split by head dim between the two CTAs, one
// thread of the leader issues every cta_group::2 MMA, TMA loads counted on
// the leader's barriers (no multicast), speculative P with lazy rescale.
// Warps 0-7 are tile A's two softmax warpgroups, 8-15 tile B's; warps 16-19
// form the control warpgroup: warp 16 the TMA producer, warp 17 the MMA
// issuer, 18-19 idle.  The control warpgroup exists so that registers can
// move: launched at 96 per thread (640 threads, one CTA per SM), it drops to
// 64 and each softmax thread rises to 104, which its 64 S values, 16 packed
// P words and the row state need: no role spills (at 96 for all, the softmax
// spilled; 112 for the softmax leaves 32 for the TMA and MMA loops, which
// then spill).  Non-causal history launches with a
// dense bf16 K/V; one item per (512-row unit, key split).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "attn_common.cuh"
#include "attn_pair.cuh"
#include "ptx.cuh"

namespace pcp {

struct Pair2Roles {
  static constexpr int kTiles = 2;
  static constexpr int kWGPerTile = 2;
  static constexpr int kSoftmaxThreads = 128 * kWGPerTile * kTiles;  // 512
  static constexpr int kTileThreads = 128 * kWGPerTile;              // 256 per query tile
  static constexpr int kThreads = kSoftmaxThreads + 128;             // 640
  static constexpr int kProducerWarp = kSoftmaxThreads / 32;         // 16
  static constexpr int kMmaWarp = kProducerWarp + 1;                 // 17
  // Registers per thread: at launch (what 640 threads x 1 CTA leave of the
  // SM's 65536, in steps of 8), then softmax / control warpgroups.
  static constexpr int kLaunchRegs = 96;
  static constexpr int kSoftmaxRegs = 104;
  static constexpr int kCtlRegs = 64;
  static constexpr int kKeys = kTileN / kWGPerTile;                  // 64 keys per softmax thread
  static constexpr int kUnitRows = 2 * kPairRows;                    // 512 query rows per pair
};
static_assert(Pair2Roles::kSoftmaxThreads * Pair2Roles::kSoftmaxRegs + 128 * Pair2Roles::kCtlRegs <=
                  Pair2Roles::kThreads * Pair2Roles::kLaunchRegs,
              "register split exceeds the launch's pool");
// Per SM sub-partition: four softmax warps and one control warp.
static_assert((4 * Pair2Roles::kSoftmaxRegs + Pair2Roles::kCtlRegs) * 32 <= 16384 &&
                  5 * 32 * Pair2Roles::kLaunchRegs <= 16384,
              "register split exceeds a sub-partition's register file");

template <int D>
struct Pair2Smem {
  static_assert(D == 128, "the ping-pong kernel serves head dim 128");
  static constexpr int kQBytes = D * 2 * kTileM;   // one tile's own 128 rows (32 KB)
  static constexpr int kStageBytes = 128 * D;       // K half [64, D] or V half [128, D/2], bf16
  static constexpr int kKBox = 64 * 128;
  static constexpr int kVBox = 128 * 128;
  static constexpr int kStages = 9;
  static constexpr int kQOff = 0;                   // tile A's Q, then tile B's
  static constexpr int kStageOff = 2 * kQBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  // q_full, kv_full[NS], kv_empty[NS], s_full[2], p_full[2], o_done[2], teardown, red[2 tiles][2]
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1 + 4;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kRedOff = kMiscOff + 16;
  // red[tile][parity][warpgroup of the tile][row]
  static constexpr int kBytes = kRedOff + 2 * 2 * 2 * kTileM * 4;
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 232448, "exceeds the 227 KB of shared memory per CTA");
};

// p.m_tiles_per_head counts 512-row units here.
template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Pair2Roles::kThreads, 1)
    attn_fwd_pair2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                          const AttnParams p) {
  using L = Pair2Smem<D>;
  using R = Pair2Roles;
  constexpr int NS = L::kStages;

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
  // Per query tile t: S_t ready (phase j & 1), P_t stored, PV_t done.
  auto bar_s_full = [&](int t) { return bars + 8u * (1 + 2 * NS + t); };
  auto bar_p_full = [&](int t) { return bars + 8u * (3 + 2 * NS + t); };
  auto bar_o = [&](int t) { return bars + 8u * (5 + 2 * NS + t); };
  const uint32_t bar_td = bars + 8u * (7 + 2 * NS);
  auto bar_red = [&](int t, int b) { return bars + 8u * (8 + 2 * NS + 2 * t + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;
  const int head = pair / p.m_tiles_per_head;
  const int ut = pair % p.m_tiles_per_head;
  // First query row of this CTA in tile t (rows past the end are padding).
  auto tile_row0 = [&](int t) { return ut * R::kUnitRows + t * kPairRows + static_cast<int>(rank) * kTileM; };
  const int split = blockIdx.y;
  const int num_keys = p.num_keys_dev ? min(max(*p.num_keys_dev, 0), p.num_keys) : p.num_keys;
  const int n_key_tiles = (num_keys + kTileN - 1) / kTileN;
  const int kt0 = split * p.tiles_per_split;
  const int kt1 = min(kt0 + p.tiles_per_split, n_key_tiles);
  const int n = kt1 - kt0;  // >= 1 on the host plan; <= 0 only for an empty split in device-length mode

  if (warp == R::kProducerWarp && lane == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar_s_full(t), 1);
      mbar_init(bar_p_full(t), 2 * R::kTileThreads / 32);  // one arrive per softmax warp of the tile, both CTAs
      mbar_init(bar_o(t), 1);
      mbar_init(bar_red(t, 0), R::kTileThreads);
      mbar_init(bar_red(t, 1), R::kTileThreads);
    }
    mbar_init(bar_td, 1);
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
  // Register split (setmaxnreg, warpgroup-uniform).  Each warpgroup's
  // setmaxnreg sits at the top of its own branch: ptxas gives every region
  // one register budget, and a join between the setmaxnreg and a role's code
  // would leave that code with the smaller one.
  if (warp >= R::kProducerWarp) {
    setmaxnreg_dec<R::kCtlRegs>();
    if (warp == R::kProducerWarp) {
      // ------------------------------------------------------ TMA producer --
      if (lane == 0 && n > 0) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
        if (leader) mbar_arrive_expect_tx(bar_q, 2 * 2 * L::kQBytes);
        const uint32_t q_lead = mapa_shared(bar_q, 0);
        for (int t = 0; t < 2; ++t)
          for (int b = 0; b < D / kBoxCols; ++b)
            tma_load_3d_pair(sQ + t * L::kQBytes + b * kBoxBytes, &tm_q, b * kBoxCols, tile_row0(t), head, q_lead);
        uint32_t c = 0;
        bool ok = true;
        // Item order = first-use order of the MMAs: K_0, then (V_j, K_{j+1}).
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
          ok = issue(true, kt0 + j);
          if (ok && j + 1 < n) ok = issue(false, kt0 + j + 1);
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
        bool ok = mbar_wait(bar_q, 0, abort_flag, p.err, kErrWaitQ);
        tc_fence_after();
        // Stage of item c (K_0 = 0, V_j = 2j + 1, K_{j+1} = 2j + 2); the first
        // use of an item waits for its bytes.
        auto wait_item = [&](uint32_t c) {
          if (!mbar_wait(bar_kv_full(c % NS), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
          tc_fence_after();
          return true;
        };
        auto qk = [&](int t, uint32_t c) {
          const uint32_t s_tmem = tmem + kTmemS0 + t * kTileN;
          const uint32_t qbase = sQ + t * L::kQBytes;
          const uint32_t kbase = sStage + (c % NS) * L::kStageBytes;
  #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t qa = qbase + (kk / 4) * kBoxBytes + (kk % 4) * 32;
            const uint32_t kb = kbase + (kk / 4) * L::kKBox + (kk % 4) * 32;
            umma_ss_pair(s_tmem, make_sw128_desc(qa, 16, 1024), make_sw128_desc(kb, 16, 1024), idesc_qk,
                         kk != 0 ? 1u : 0u);
          }
          umma_commit_pair(bar_s_full(t), kBothCtas);
        };
        auto pv = [&](int t, uint32_t c, int j) {
          if (!mbar_wait(bar_p_full(t), j & 1, abort_flag, p.err, kErrWaitPFull)) return false;
          tc_fence_after();
          const uint32_t p_tmem = tmem + kTmemS0 + t * kTileN;
          const uint32_t o_tmem = tmem + t * D;
          const uint32_t vbase = sStage + (c % NS) * L::kStageBytes;
  #pragma unroll
          for (int kk = 0; kk < kTileN / 16; ++kk) {
            // A = P (packed into the first half of each warpgroup's 64 S
            // columns), B = V half, MN-major (see attn_pair.cuh).
            const uint32_t a_cols = kk * 8 + (kk >= 4 ? 32 : 0);
            umma_ts_pair(o_tmem, p_tmem + a_cols, make_sw128_desc(vbase + kk * 2048, L::kVBox, 1024), idesc_pv,
                         (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(bar_o(t), kBothCtas);
          return true;
        };
        if (ok) ok = wait_item(0);
        if (ok) {
          qk(0, 0);
          qk(1, 0);
          umma_commit_pair(bar_kv_empty(0), kBothCtas);  // K_0 read by both tiles
        }
        for (int j = 0; j < n && ok; ++j) {
          const uint32_t cv = 2 * j + 1, ck = 2 * j + 2;
          const bool more = j + 1 < n;
          ok = wait_item(cv) && pv(0, cv, j);
          if (ok && more) {
            ok = wait_item(ck);
            if (ok) qk(0, ck);
          }
          if (ok) ok = pv(1, cv, j);
          if (ok) umma_commit_pair(bar_kv_empty(cv % NS), kBothCtas);  // V_j read by both tiles
          if (ok && more) {
            qk(1, ck);
            umma_commit_pair(bar_kv_empty(ck % NS), kBothCtas);  // K_{j+1} read by both tiles
          }
        }
        // Drain: completes when every MMA issued above has.
        umma_commit_pair(bar_td, kLeaderCta);
        mbar_wait_teardown(bar_td, 0);
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<R::kSoftmaxRegs>();
    // ---------------------------------------- softmax / correction / epilogue --
    constexpr int kHalfKeys = R::kKeys;  // 64
    constexpr int kOCols = D / R::kWGPerTile;
    const int t = warp >> 3;              // query tile of this warp
    const int wg = (warp >> 2) & 1;       // warpgroup within the tile
    const uint32_t bar_base = 1 + 3 * t;  // named barriers 1..3 (tile A), 4..6 (tile B)
    const int row = threadIdx.x & (kTileM - 1);  // == TMEM lane
    const int row0 = tile_row0(t);
    const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t t_s = t_row + kTmemS0 + t * kTileN;
    const uint32_t t_o = t_row + t * D;
    float* red_t = red + t * 2 * 2 * kTileM;
    const float sl2 = p.scale_log2;
    const int key_limit = num_keys;
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = n > 0;
    auto make_p = [&](const float* sv, float m) { return store_probs<kHalfKeys>(sv, m, sl2, t_s + wg * kHalfKeys); };
    for (int j = 0; j < n && ok; ++j) {
      const int b = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(t), j & 1, abort_flag, p.err, kErrWaitSFull));
      if (!ok) break;
      tc_fence_after();
      float s[kHalfKeys];
      load_scores<kHalfKeys>(t_s + wg * kHalfKeys, key_limit - (kt0 + j) * kTileN - wg * kHalfKeys, s);
      const float pmax = row_max(s);
      red_t[(b * 2 + wg) * kTileM + row] = pmax;
      mbar_arrive(bar_red(t, b));
      // Speculative P with the current reference max (see attn_pair.cuh).
      float tile_sum = 0.f;
      if (j > 0) tile_sum = make_p(s, m_ref);
      ok = __all_sync(0xffffffffu, mbar_wait(bar_red(t, b), (j >> 1) & 1u, abort_flag, p.err, kErrWaitRed));
      if (!ok) break;
      const float tmax = fmaxf(pmax, red_t[(b * 2 + (wg ^ 1)) * kTileM + row]);
      const bool need = (tmax - m_ref) * sl2 > kRescaleThreshold;  // always true on the first tile
      const bool redo = __any_sync(0xffffffffu, need);
      float alpha = 1.f;
      if (need) {
        alpha = ex2_approx((m_ref - tmax) * sl2);  // 0 on the first tile
        m_ref = tmax;
        l *= alpha;
      }
      if (redo) tile_sum = make_p(s, m_ref);
      l += tile_sum;
      // S_t(j) ready means PV_t(j-1) is complete (issued before QK_t(j), and
      // the tensor pipe completes in order): O_t may be rescaled right away.
      if (j > 0 && redo) rescale_o<kOCols>(t_o + wg * kOCols, alpha);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(bar_p_full(t), 0));
    }
    if (ok)
      ok = __all_sync(0xffffffffu, mbar_wait(bar_o(t), (n - 1) & 1, abort_flag, p.err, kErrWaitODone));
    ok = named_bar_and(bar_base, R::kTileThreads, ok && (*abort_flag == 0));
    if (ok) {
      tc_fence_after();
      red_t[wg * kTileM + row] = l;
      named_bar_sync(bar_base + 1, R::kTileThreads);
      const float l_tot = l + red_t[(wg ^ 1) * kTileM + row];
      const float inv_l = 1.f / l_tot;
      if (p.write_final) {
        // This tile's Q buffer holds its bf16 O for the TMA store (every
        // QK^T of both tiles completed before the last PV of either).
        stage_o_sw128<kOCols>(t_o + wg * kOCols, inv_l, smem + L::kQOff + t * L::kQBytes, kBoxBytes, wg * kOCols,
                              row);
        fence_proxy_async_smem();
        named_bar_sync(bar_base + 2, R::kTileThreads);
        if ((threadIdx.x & (R::kTileThreads - 1)) == 0 && row0 < p.rows_per_head) {
          for (int box = 0; box < D / kBoxCols; ++box)
            tma_store_3d(&tm_o, sQ + t * L::kQBytes + box * kBoxBytes, box * kBoxCols, row0, head);
          tma_store_commit();
          tma_store_wait0();
        }
      } else {
        const int rih = row0 + row;
        const size_t split_idx = static_cast<size_t>(p.split_base + split);
        const size_t grow = static_cast<size_t>(head) * p.rows_per_head + rih;
        float* dst = p.part_o + (split_idx * p.total_rows + grow) * D + wg * kOCols;
        const bool live = rih < p.rows_per_head;
        store_o_partial<kOCols>(t_o + wg * kOCols, inv_l, dst, live);
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
