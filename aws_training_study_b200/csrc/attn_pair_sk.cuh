// History-attention forward on CTA pairs, stream-K schedule.
//
// The same per-tile pipeline as attn_fwd_pair_kernel (attn_pair.cuh: TMA
// producer, one MMA thread issuing cta_group::2 tcgen05 MMAs for the pair,
// two softmax warpgroups per CTA with lazy rescale), but on a persistent
// grid: G CTA pairs (one per two SMs) take equal contiguous ranges of the
// U * n_kt (unit, key tile) steps in unit-major order and walk them as
// segments (a run of key tiles of one unit).  Every pair gets the same work,
// the prologue (barriers, TMEM) is paid once, and only units cut by a range
// boundary leave partials ([split_base, split_base + max_segs) slots per
// unit; a unit one segment covers is written as bf16 O when final_ok).
// Segment k+1 reloads Q once segment k's last QK^T has read it (q_empty);
// every barrier phase follows one tile counter across segments.
//
// Used for the last launch of a forward when its K/V fits in L2: its pairs
// read K/V at unrelated offsets (a larger working set would stream from HBM
// once per pair rather than once per wave), and it holds every SM until it
// ends (an NCCL exchange still in flight would get no SM).
// No TMA multicast is used: each CTA loads only its own smem.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "attn_common.cuh"
#include "attn_pair.cuh"
#include "ptx.cuh"

namespace pcp {

template <int D>
struct PairSmemSK {
  static constexpr int kQBytes = D * 2 * kTileM;           // own 128 rows (D/64 boxes of 16 KB)
  static constexpr int kStageBytes = 128 * D;              // K half [64, D] or V half [128, D/2], bf16
  static constexpr int kKBox = 64 * 128;                   // K box: 64 rows x 128 B
  static constexpr int kVBox = 128 * 128;                  // V box: 128 rows x 128 B
  static constexpr int kStages = (D == 256) ? 5 : 12;
  static constexpr int kQOff = 0;
  static constexpr int kStageOff = kQBytes;
  static constexpr int kBarOff = kStageOff + kStages * kStageBytes;
  // q_full, kv_full[NS], kv_empty[NS], s_full[2], p_full[2], o_done[2], teardown, red[2], q_empty
  static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 1 + 2 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kRedOff = kMiscOff + 16;
  static constexpr int kBytes = kRedOff + 2 * PairRoles<D>::kWG * kTileM * 4;
  static constexpr int kAlloc = kBytes;
  static_assert(kAlloc <= 232448, "exceeds the 227 KB of shared memory per CTA");
};


// One run of key tiles [kt0, kt1) of one unit, and where its result goes.
struct Segment {
  int unit;
  int kt0, kt1;
  int slot;  // partial slot of this segment within its unit
  int nseg;  // segments the unit is cut into
  bool last; // the segment ends the unit's key range
};

// Stream-K segments of one CTA pair, identical in every role of both CTAs
// (host-callable too: pcp_stream_k_segments exposes it for tests).
struct Schedule {
  int n_kt, units;
  long long T, t, t_end;
  int pairs, g;

  __host__ __device__ void init_stream_k(int n_kt_, int units_, int grid_pairs, int pair) {
    n_kt = n_kt_;
    units = units_;
    T = static_cast<long long>(units) * n_kt;
    // At least two tiles per pair (bounds the segments of any unit by
    // ceil(2G/U) + 1); pairs past that have no work.
    pairs = static_cast<int>(stream_k_pairs(T, grid_pairs));
    g = pair;
    if (g < pairs && T > 0) {
      t = T * g / pairs;
      t_end = T * (g + 1) / pairs;
    } else {
      t = t_end = 0;
    }
  }
  // First pair whose range holds tile x (ranges [T g / G, T (g + 1) / G)).
  __host__ __device__ long long pair_of(long long x) const { return stream_k_pair_of(x, T, pairs); }
  __host__ __device__ bool next(Segment& s) {
    if (t >= t_end) return false;
    const int u = static_cast<int>(t / n_kt);
    const long long ub = static_cast<long long>(u) * n_kt;
    s.unit = u;
    s.kt0 = static_cast<int>(t - ub);
    const long long end = t_end - ub;
    s.kt1 = static_cast<int>(end < n_kt ? end : n_kt);
    const long long g0 = pair_of(ub);
    s.slot = static_cast<int>(g - g0);
    s.nseg = static_cast<int>(pair_of(ub + n_kt - 1) - g0 + 1);
    s.last = s.kt1 == n_kt;
    t = ub + s.kt1;
    return true;
  }
};

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairRoles<D>::kThreads, 1)
    attn_fwd_pair_sk_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using L = PairSmemSK<D>;
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
  // o_done[b] completes once per PV of tile J with J % 2 == b (phase J / 2).
  auto bar_o = [&](int b) { return bars + 8u * (5 + 2 * NS + b); };
  const uint32_t bar_td = bars + 8u * (7 + 2 * NS);
  auto bar_red = [&](int b) { return bars + 8u * (8 + 2 * NS + b); };
  // q_empty completes once per segment, when its last QK^T has read Q.
  const uint32_t bar_q_empty = bars + 8u * (10 + 2 * NS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;
  const int num_keys = p.num_keys_dev ? min(max(*p.num_keys_dev, 0), p.num_keys) : p.num_keys;
  const int n_kt = (num_keys + kTileN - 1) / kTileN;
  const int units = p.num_kv_heads * p.m_tiles_per_head;

  // Calls body(segment) for each segment of this pair, in order, until it
  // returns false; returns false if it did.
  auto for_each_segment = [&](auto&& body) -> bool {
    Schedule sc;
    sc.init_stream_k(n_kt, units, gridDim.x >> 1, pair);
    Segment sg;
    while (sc.next(sg))
      if (!body(sg)) return false;
    return true;
  };

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
    mbar_init(bar_q_empty, 1);
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
    if (lane == 0) {
      uint32_t c = 0;
      int segs = 0;
      bool primed = false;
      // Item order = MMA consumption order: per segment K_0, then
      // (K_{j+1}, V_j) per tile.
      auto issue = [&](bool is_v, int kt, int head) {
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
        if (segs > 0 && !mbar_wait(bar_q_empty, (segs - 1) & 1u, abort_flag, p.err, kErrWaitQ))
          return false;
        if (leader) mbar_arrive_expect_tx(bar_q, 2 * L::kQBytes);
        const uint32_t q_lead = mapa_shared(bar_q, 0);
        for (int b = 0; b < D / kBoxCols; ++b)
          tma_load_3d_pair(sQ + b * kBoxBytes, &tm_q, b * kBoxCols, row0, head, q_lead);
        ++segs;
        if (!issue(false, sg.kt0, head)) return false;
        for (int j = 0; j < n; ++j) {
          if (j + 1 < n && !issue(false, sg.kt0 + j + 1, head)) return false;
          if (!issue(true, sg.kt0 + j, head)) return false;
        }
        return true;
      });
      if (!ok) {
        // Abort: let copies already in flight land before the CTA exits.
        if (leader) {
          for (uint32_t i = (c > (uint32_t)NS ? c - NS : 0); i < c; ++i)
            mbar_wait_teardown(bar_kv_full(i % NS), (i / NS) & 1u);
          if (segs > 0) mbar_wait_teardown(bar_q, (segs - 1) & 1u);
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
    if (leader && lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kPairRows, kTileN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kPairRows, D, false, true);
      uint32_t c = 0;
      uint32_t J = 0;  // tiles of all earlier segments
      int segs = 0;
      auto qk = [&](uint32_t jg) {
        const uint32_t s_tmem = tmem + kTmemS0 + (jg & 1) * kTileN;
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
        umma_commit_pair(bar_s_full(jg & 1), kBothCtas);
        return true;
      };
      auto pv = [&](uint32_t jg, bool first) {
        if (!mbar_wait(bar_p_full(jg & 1), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitPFull)) return false;
        const int st = c % NS;
        if (!mbar_wait(bar_kv_full(st), (c / NS) & 1u, abort_flag, p.err, kErrWaitKvFull)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + kTmemS0 + (jg & 1) * kTileN;
        const uint32_t vbase = sStage + st * L::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {
          // A = P: each softmax warpgroup packed its keys into the first half
          // of its own S columns (PairRoles::p_col); 16 keys = 8 columns per
          // step.  B = V half, MN-major: 64-dim chunks 16 KB apart (LBO),
          // 8-key groups 1 KB apart (SBO); a 16-key step is 2 KB.
          const uint32_t a_cols = R::p_col(kk);
          umma_ts_pair(tmem, p_tmem + a_cols, make_sw128_desc(vbase + kk * 2048, L::kVBox, 1024), idesc_pv,
                       (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit_pair(bar_kv_empty(st), kBothCtas);
        ++c;
        umma_commit_pair(bar_o(jg & 1), kBothCtas);
        return true;
      };
      for_each_segment([&](const Segment& sg) -> bool {
        if (sg.kt1 <= sg.kt0) return true;
        const uint32_t n = static_cast<uint32_t>(sg.kt1 - sg.kt0);
        // Q of this segment in both CTAs.  (O of the previous segment has
        // been read out: its softmax warps release P_0 of this segment only
        // after their epilogue.)
        if (!mbar_wait(bar_q, segs & 1u, abort_flag, p.err, kErrWaitQ)) return false;
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
    constexpr int kHalfKeys = R::kKeys;  // keys of this warpgroup per tile
    constexpr int kOCols = R::kOCols;
    const int wg = warp >> 2;
    const int row = threadIdx.x & (kTileM - 1);  // == TMEM lane
    const uint32_t t_row = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
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
    uint32_t J = 0;
    if (n_kt == 0 && pair < units) {
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
      const int key_limit = num_keys;  // history launches only (the causal launch is static)
      float m_ref = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < n && ok; ++j) {
        const uint32_t jg = J + j;
        const int b = jg & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_s_full(b), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitSFull));
        if (!ok) break;
        tc_fence_after();
        const uint32_t t_s = t_row + kTmemS0 + b * kTileN;
        float s[kHalfKeys];
        load_scores<kHalfKeys>(t_s + wg * kHalfKeys, key_limit - (sg.kt0 + j) * kTileN - wg * kHalfKeys, s);
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
        ok = __all_sync(0xffffffffu, mbar_wait(bar_red(b), (jg >> 1) & 1u, abort_flag, p.err, kErrWaitRed));
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
        // O is rescaled only when the reference max moved (rare): then PV of
        // the previous tile must be complete first.  Otherwise P_j is released
        // at once, so the MMA warp can issue PV_j without waiting for PV_{j-1}.
        // (s_full of tile J already implies PV of tile J-2 is complete: its
        // QK^T was issued after it, and tcgen05 MMAs complete in issue order.)
        if (j > 0 && redo) {
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_o((jg - 1) & 1), ((jg - 1) >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
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
      if (ok && n > 0) {
        const uint32_t jl = J + n - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(bar_o(jl & 1), (jl >> 1) & 1u, abort_flag, p.err, kErrWaitODone));
      }
      ok = named_bar_and(1, R::kSoftmaxThreads, ok && (*abort_flag == 0));
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
        // Empty split (static schedule, device-length mode): weight zero.
        if (!final_out && live && wg == 0)
          p.part_lse[static_cast<size_t>(p.split_base + sg.slot) * p.total_rows + grow] = -INFINITY;
        return true;
      }
      tc_fence_after();
      red[wg * kTileM + row] = l;
      named_bar_sync(2, R::kSoftmaxThreads);
      float l_tot = l;
#pragma unroll
      for (int w = 1; w < kWG; ++w) l_tot += red[(wg ^ w) * kTileM + row];
      // Every share read: the next segment may reuse the exchange slots.
      named_bar_sync(2, R::kSoftmaxThreads);
      const float inv_l = 1.f / l_tot;
      if (final_out) {
        // Stream-K: sQ may already hold the next segment's Q; store directly.
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
  if (warp == R::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace pcp
