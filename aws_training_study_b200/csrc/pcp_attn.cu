// Host side of the C ABI declared in include/pcp_attn.h: launch planning,
// TMA tensor maps, the stateless single-GPU entry, and the per-rank ring
// handle (NCCL send/recv ring on a high-priority stream overlapped with the
// attention of the local shard).
#include "pcp_attn.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <thread>
#include <vector>

#include "attn_pair.cuh"
#include "attn_pair_sk.cuh"
#include "attn_pair2.cuh"
#include "attn_kv.cuh"
#include "kv_stage.cuh"

namespace {

thread_local char g_err[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define CUDA_TRY(x)                                                                                     \
  do {                                                                                                  \
    cudaError_t e_ = (x);                                                                               \
    if (e_ != cudaSuccess)                                                                              \
      return fail(e_ == cudaErrorMemoryAllocation ? PCP_ERR_OUT_OF_MEMORY : PCP_ERR_CUDA, "%s: %s (%s:%d)", \
                  #x, cudaGetErrorString(e_), __FILE__, __LINE__);                                     \
  } while (0)

#define PCP_TRY(x)          \
  do {                      \
    int s_ = (x);           \
    if (s_ != PCP_OK) return s_; \
  } while (0)

constexpr int kMaxTotalSplits = 32;
constexpr size_t kPartialBudget = size_t(1) << 30;  // bytes of split partials a handle may hold

// ------------------------------------------------------------ tensor maps --
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 tensor [heads][rows][cols] (cols contiguous, heads `head_stride` elements
// apart), boxes of 64 cols x `box_rows` rows x 1 head with 128-byte swizzle.
int make_tmap(CUtensorMap* tm, const void* base, uint64_t cols, uint64_t rows, uint64_t heads,
              uint64_t head_stride, uint32_t box_rows = 128) {
  auto fn = encode_fn();
  if (!fn) return fail(PCP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(PCP_ERR_INVALID_ARGUMENT, "TMA base not 16-byte aligned");
  cuuint64_t dims[3] = {cols, rows, heads};
  cuuint64_t strides[2] = {cols * 2, head_stride * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PCP_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return PCP_OK;
}

// e4m3 cache blocks [blocks][2][Hkv][bs][D] (the packed payload), as a 5-D
// byte tensor {D, bs, Hkv, K/V, blocks}; boxes of `box_x` bytes x 64 rows of
// one head of K or V of one block, no swizzle.
int make_tmap_blocks(CUtensorMap* tm, const void* base, const pcp_dims_t& d, int64_t blocks, uint32_t box_x) {
  auto fn = encode_fn();
  if (!fn) return fail(PCP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(PCP_ERR_INVALID_ARGUMENT, "KV cache not 16-byte aligned");
  const uint64_t D = d.head_dim, bs = d.block_size, H = d.num_kv_heads;
  cuuint64_t dims[5] = {D, bs, H, 2, static_cast<cuuint64_t>(std::max<int64_t>(blocks, 1))};
  cuuint64_t strides[4] = {D, bs * D, H * bs * D, 2 * H * bs * D};
  cuuint32_t box[5] = {box_x, 64, 1, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PCP_ERR_CUDA, "cuTensorMapEncodeTiled (cache blocks) failed (%d)", static_cast<int>(r));
  return PCP_OK;
}

// --------------------------------------------------------------- planning --
int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

// Attention schedules: the wave-scheduled kernel (attn_pair.cuh) or the
// stream-K kernel (attn_pair_sk.cuh).
constexpr int kModeStatic = 0;   // one (unit, key split) item per CTA pair, in waves
constexpr int kModeStreamK = 1;  // equal contiguous (unit, tile) ranges per persistent pair
// Stream-K only while the launch's bf16 K/V stays well inside the 126 MB L2
// (its pairs read K/V at unrelated offsets).
constexpr int64_t kStreamKMaxKvBytes = int64_t(48) << 20;

// How a history launch reads the KV cache:
//   * dense: kv_unpack_kernel expands the valid tokens into a dense bf16
//     workspace once per forward, and attn_fwd_pair(_sk)_kernel reads it;
//   * in place (e4m3 caches whose 64-key boxes never cross a cache block):
//     attn_fwd_kv_kernel loads the cache blocks with TMA and upcasts them to
//     f16 in shared memory -- no extra pass and no dense copy, but every
//     256-row query unit converts every key tile again.
// Measured on one B200 with configs[3]'s heads and 131072-token history
// (whole forward, TFLOP/s, dense / in place): 1024 query rows per KV head
// 887 / 1053, 4096 rows 1115 / 1148, 16384 rows 1510 / 1279, 65536 rows
// 1481 / 1257 (in place with the conversion skipped: 1572).  The
// conversion pays while a KV head has few 256-row query units: `auto` reads
// in place up to kInPlaceMaxRows query rows per KV head.
constexpr int64_t kInPlaceMaxRows = 4096;
std::atomic<int> g_kv_path{PCP_KV_PATH_AUTO};  // process default (pcp_set_kv_path(NULL, ...))

bool kv_in_place_ok(const pcp_dims_t& d) { return d.kv_dtype == PCP_KV_E4M3 && d.block_size % 64 == 0; }
int64_t rows_per_head(const pcp_dims_t& d);
bool choose_in_place(const pcp_dims_t& d, int mode) {
  if (!kv_in_place_ok(d) || mode == PCP_KV_PATH_DENSE) return false;
  return mode == PCP_KV_PATH_IN_PLACE || rows_per_head(d) <= kInPlaceMaxRows;
}
// Bytes of K and V one launch over `keys` keys reads: its L2 working set.
int64_t kv_bytes(const pcp_dims_t& d, int64_t keys, bool in_place) {
  return keys * d.num_kv_heads * d.head_dim * (in_place ? 2 : 4);
}

struct SplitPlan {
  int splits = 1;           // partial slots per unit the launch may write
  int tiles_per_split = 1;  // static: key tiles per split
  int mode = kModeStatic;
  int pairs = 1;            // stream-K: CTA pairs in the grid
};

// Stream-K: one CTA pair per two SMs (fewer when there are not two tiles per
// pair), each pair an equal share of the steps; a unit is then cut into at
// most min(G, ceil(2G/U) + 1) segments, which must fit `slot_cap` partial
// slots (fewer pairs when they do not).
SplitPlan plan_stream_k(int64_t units, int64_t n_kt, int sms, int slot_cap) {
  SplitPlan pl;
  pl.mode = kModeStreamK;
  int64_t g = pcp::stream_k_pairs(std::max<int64_t>(1, units * n_kt), std::max(1, sms / 2));
  auto segs = [&](int64_t gg) { return std::min<int64_t>(gg, ceil_div(2 * gg, std::max<int64_t>(1, units)) + 1); };
  while (g > 1 && segs(g) > std::max(1, slot_cap)) --g;
  pl.pairs = static_cast<int>(g);
  pl.splits = static_cast<int>(segs(g));
  return pl;
}

// Static: key splits chosen so that the (unit, split) items fill whole waves
// of the SM pairs.  Cost model: waves * (tiles per item + 2 tiles of fixed
// prologue/epilogue cost), with a small bias against splitting.
SplitPlan plan_static(int64_t units, int64_t n_kt, int sms, int slot_cap) {
  const int64_t slots = std::max(1, sms / 2);
  SplitPlan best;
  best.mode = kModeStatic;
  best.splits = 1;
  best.tiles_per_split = static_cast<int>(std::max<int64_t>(1, n_kt));
  double best_cost = 1e300;
  const int smax = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(std::max(1, slot_cap), n_kt)));
  for (int s = 1; s <= smax; ++s) {
    const int64_t tps = ceil_div(std::max<int64_t>(1, n_kt), s);
    const int64_t s_eff = ceil_div(std::max<int64_t>(1, n_kt), tps);
    const int64_t waves = ceil_div(units * s_eff, slots);
    const double cost = static_cast<double>(waves) * (static_cast<double>(tps) + 2.0) + (s_eff > 1 ? 0.5 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best.splits = static_cast<int>(s_eff);
      best.tiles_per_split = static_cast<int>(tps);
    }
  }
  return best;
}

int check_dims(const pcp_dims_t* d) {
  if (!d) return fail(PCP_ERR_INVALID_ARGUMENT, "dims is NULL");
  if (d->pcp_size <= 0 || d->local_q_len <= 0 || d->max_local_blocks <= 0 || d->block_size <= 0 ||
      d->num_q_heads <= 0 || d->num_kv_heads <= 0 || d->head_dim <= 0)
    return fail(PCP_ERR_INVALID_ARGUMENT, "all dims must be positive");
  if (d->num_q_heads % d->num_kv_heads)
    return fail(PCP_ERR_INVALID_ARGUMENT, "num_q_heads must be divisible by num_kv_heads");
  if (d->head_dim != 128 && d->head_dim != 256)
    return fail(PCP_ERR_UNSUPPORTED, "head_dim %d unsupported by the CUDA kernel (128 or 256)", d->head_dim);
  if (d->kv_dtype != PCP_KV_E4M3 && d->kv_dtype != PCP_KV_BF16)
    return fail(PCP_ERR_INVALID_ARGUMENT, "kv_dtype %d unknown", d->kv_dtype);
  if (d->pcp_size > pcp::kMaxSources) return fail(PCP_ERR_UNSUPPORTED, "pcp_size above %d", pcp::kMaxSources);
  const int64_t rows = static_cast<int64_t>(d->num_q_heads / d->num_kv_heads) * d->local_q_len;
  if (rows > (int64_t(1) << 30)) return fail(PCP_ERR_UNSUPPORTED, "too many query rows per KV head");
  return PCP_OK;
}

pcp::UnpackSource contiguous_src(const void* base, int valid, int64_t dst_offset, int dev_index = -1) {
  return {static_cast<const uint8_t*>(base), nullptr, 0, valid, static_cast<int>(dst_offset), dev_index};
}
pcp::UnpackSource paged_src(const void* pool, const int32_t* table, int64_t pool_blocks, int valid, int64_t dst_offset,
                            int dev_index = -1) {
  return {static_cast<const uint8_t*>(pool), table, pool_blocks, valid, static_cast<int>(dst_offset), dev_index};
}

// Device-length mode: per-part valid key counts written by the unpack, in
// the workspace header (after the error word).
constexpr size_t kPartKeysOff = 64;
constexpr int kMaxParts = 8;
int* part_keys_slot(uint8_t* ws, int part) { return reinterpret_cast<int*>(ws + kPartKeysOff) + part; }

int64_t payload_bytes(const pcp_dims_t& d) {
  return 2LL * d.num_kv_heads * d.block_size * d.head_dim * (d.kv_dtype == PCP_KV_BF16 ? 2 : 1);
}
int64_t rows_per_head(const pcp_dims_t& d) { return static_cast<int64_t>(d.num_q_heads / d.num_kv_heads) * d.local_q_len; }
int64_t total_rows(const pcp_dims_t& d) { return static_cast<int64_t>(d.num_q_heads) * d.local_q_len; }
// Work units of one split: 256-row CTA-pair tiles over every KV head.
int64_t m_units(const pcp_dims_t& d) { return d.num_kv_heads * ceil_div(rows_per_head(d), pcp::kPairRows); }
// Dense static-schedule history launches at head dim 128 with at least 512
// query rows per KV head run on attn_fwd_pair2_kernel (two query tiles per
// CTA pair, ping-pong), whose work units are 512 query rows.
bool pingpong(const pcp_dims_t& d, bool in_place) {
  return d.head_dim == 128 && !in_place && rows_per_head(d) >= pcp::Pair2Roles::kUnitRows;
}
// Work units of a static-schedule history launch.
int64_t static_units(const pcp_dims_t& d, bool in_place) {
  return pingpong(d, in_place) ? d.num_kv_heads * ceil_div(rows_per_head(d), pcp::Pair2Roles::kUnitRows)
                               : m_units(d);
}

// Relative cost of a plan in key tiles per SM pair: stream-K walks
// ceil(steps / pairs) tiles plus ~2 tiles of prologue and partial write;
// static runs waves of (tiles per item + 2).
double plan_cost(const SplitPlan& pl, int64_t units, int64_t n_kt, int sms) {
  if (pl.mode == kModeStreamK)
    return static_cast<double>(ceil_div(units * n_kt, std::max(1, pl.pairs))) + 2.0;
  const int64_t waves = ceil_div(units * pl.splits, std::max(1, sms / 2));
  return static_cast<double>(waves) * (pl.tiles_per_split + 2.0);
}

// The schedule of a history launch over `tiles` key tiles (or their bound)
// of `keys` keys.  `last`: no exchange is in flight while it runs (the
// forward's last launch).  Stream-K is kept only when the partial-slot cap
// leaves it a grid at least as fast as the static schedule's (a cap of one
// or two slots can shrink the stream-K grid to a few pairs).
SplitPlan plan_splits(const pcp_dims_t& d, int64_t tiles, int64_t keys, int sms, int slot_cap, bool last,
                      bool in_place) {
  const int64_t n_kt = std::max<int64_t>(1, tiles);
  const int64_t su = static_units(d, in_place);
  const SplitPlan st = plan_static(su, n_kt, sms, slot_cap);
  if (!last || kv_bytes(d, keys, in_place) > kStreamKMaxKvBytes) return st;
  const SplitPlan sk = plan_stream_k(m_units(d), n_kt, sms, slot_cap);
  return plan_cost(sk, m_units(d), n_kt, sms) <= plan_cost(st, su, n_kt, sms) ? sk : st;
}

// A plan made for `planned` tiles run over `actual` >= planned tiles (in
// place, each source's last tile may be partial): the static schedule keeps
// at most its split count and covers every tile; a stream-K grid covers any
// tile count and never needs more slots than planned.
SplitPlan fit_plan(SplitPlan pl, int64_t actual) {
  if (pl.mode == kModeStatic) {
    const int64_t n = std::max<int64_t>(1, actual);
    pl.tiles_per_split = static_cast<int>(ceil_div(n, pl.splits));
    pl.splits = static_cast<int>(ceil_div(n, pl.tiles_per_split));
  }
  return pl;
}


int num_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

int max_splits_for(const pcp_dims_t& d) {
  const size_t per_split = static_cast<size_t>(total_rows(d)) * d.head_dim * 4 + static_cast<size_t>(total_rows(d)) * 4;
  const size_t cap = std::max<size_t>(2, kPartialBudget / std::max<size_t>(per_split, 1));
  return static_cast<int>(std::min<size_t>(kMaxTotalSplits, cap));
}

// Workspace: [error word][K bf16][V bf16][partial O fp32][partial lse fp32].
struct Workspace {
  size_t k_off = 0, v_off = 0, po_off = 0, pl_off = 0, total = 0;
  int64_t key_stride = 0;
  int max_splits = 0;
};

Workspace ws_layout(const pcp_dims_t& d, int64_t key_cap, int split_cap) {
  Workspace w;
  w.key_stride = align_up(static_cast<size_t>(std::max<int64_t>(key_cap, 1)), pcp::kTileN);
  const size_t kv = static_cast<size_t>(d.num_kv_heads) * w.key_stride * d.head_dim * 2;
  w.k_off = 1024;
  w.v_off = align_up(w.k_off + kv, 1024);
  w.po_off = align_up(w.v_off + kv, 1024);
  w.max_splits = split_cap;
  const size_t po = split_cap > 1 ? static_cast<size_t>(split_cap) * total_rows(d) * d.head_dim * 4 : 0;
  w.pl_off = align_up(w.po_off + po, 1024);
  const size_t pl = split_cap > 1 ? static_cast<size_t>(split_cap) * total_rows(d) * 4 : 0;
  w.total = align_up(w.pl_off + pl, 1024);
  return w;
}

// Opts a kernel into its dynamic shared memory once per device.
template <typename Kernel>
int set_smem_attr(Kernel kernel, int bytes, int* done_mask) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(*done_mask & (1 << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail(PCP_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    *done_mask |= (1 << dev);
  }
  return PCP_OK;
}

// Static schedule (attn_pair.cuh) or stream-K (attn_pair_sk.cuh).
template <int D, bool kStreamK>
int launch_pair_kernel(dim3 grid, cudaStream_t st, const CUtensorMap& tq, const CUtensorMap& tk,
                       const CUtensorMap& tv, const CUtensorMap& to, const pcp::AttnParams& p) {
  static int done = 0;
  if constexpr (kStreamK) {
    PCP_TRY(set_smem_attr(pcp::attn_fwd_pair_sk_kernel<D>, pcp::PairSmemSK<D>::kAlloc, &done));
    pcp::attn_fwd_pair_sk_kernel<D><<<grid, pcp::PairRoles<D>::kThreads, pcp::PairSmemSK<D>::kAlloc, st>>>(tq, tk, tv, p);
  } else {
    PCP_TRY(set_smem_attr(pcp::attn_fwd_pair_kernel<D>, pcp::PairSmem<D>::kAlloc, &done));
    pcp::attn_fwd_pair_kernel<D><<<grid, pcp::PairRoles<D>::kThreads, pcp::PairSmem<D>::kAlloc, st>>>(tq, tk, tv, to, p);
  }
  return PCP_OK;
}

struct LaunchCounter {
  int kernels = 0;
  int attn = 0;
};

int launch_unpack(const pcp_dims_t& d, const std::vector<pcp::UnpackSource>& srcs, const Workspace& w, uint8_t* ws,
                  cudaStream_t st, LaunchCounter* lc, const int32_t* valid_dev = nullptr,
                  int* part_keys = nullptr) {
  if (srcs.empty()) return PCP_OK;
  if (srcs.size() > static_cast<size_t>(pcp::kMaxSources)) return fail(PCP_ERR_UNSUPPORTED, "too many sources");
  pcp::UnpackParams p{};
  int max_valid = 0;
  for (size_t i = 0; i < srcs.size(); ++i) {
    p.src[i] = srcs[i];
    max_valid = std::max(max_valid, srcs[i].valid);
    if (reinterpret_cast<uintptr_t>(srcs[i].base) % 16)
      return fail(PCP_ERR_INVALID_ARGUMENT, "packed_kv must be 16-byte aligned");
  }
  p.num_sources = static_cast<int>(srcs.size());
  p.num_kv_heads = d.num_kv_heads;
  p.block_size = d.block_size;
  p.head_dim = d.head_dim;
  p.kv_is_bf16 = d.kv_dtype == PCP_KV_BF16;
  p.key_stride = static_cast<int>(w.key_stride);
  p.k_out = reinterpret_cast<__nv_bfloat16*>(ws + w.k_off);
  p.v_out = reinterpret_cast<__nv_bfloat16*>(ws + w.v_off);
  p.err = reinterpret_cast<int*>(ws);
  p.valid_dev = valid_dev;
  p.part_keys = part_keys;
  const int64_t live_blocks = ceil_div(max_valid, d.block_size);
  const int64_t items = live_blocks * 2 * d.num_kv_heads * d.block_size * (d.head_dim / 16);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, 256), 4 * 148));
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(srcs.size()));
  pcp::kv_unpack_kernel<<<grid, 256, 0, st>>>(p);
  CUDA_TRY(cudaGetLastError());
  if (lc) lc->kernels++;
  return PCP_OK;
}

// Causal current-token launch: the query shard's rank and stripe width
// (stripe_width 0: plain history launch).
struct Causal {
  int rank = 0;
  int stripe_width = 0;
};

// Attention over `num_keys` dense keys starting at key `key_off` of the
// workspace K/V.  Writes bf16 `out` directly (final) or split partials.
int launch_attention(const pcp_dims_t& d, const void* q, const Workspace& w, uint8_t* ws, int64_t key_off,
                     int64_t num_keys, const SplitPlan& plan, int split_base, bool final_out, void* out,
                     cudaStream_t st, LaunchCounter* lc, const Causal& causal = Causal{},
                     const int* num_keys_dev = nullptr) {
  const int64_t R = rows_per_head(d);
  const int64_t mt = ceil_div(R, pcp::kPairRows);  // CTA-pair tiles per KV head
  CUtensorMap tq, tk, tv, to;
  const auto* kb = reinterpret_cast<const __nv_bfloat16*>(ws + w.k_off) + key_off * d.head_dim;
  const auto* vb = reinterpret_cast<const __nv_bfloat16*>(ws + w.v_off) + key_off * d.head_dim;
  PCP_TRY(make_tmap(&tq, q, d.head_dim, R, d.num_kv_heads, R * d.head_dim));
  PCP_TRY(make_tmap(&tk, kb, d.head_dim, num_keys, d.num_kv_heads, w.key_stride * d.head_dim, 64));
  PCP_TRY(make_tmap(&tv, vb, d.head_dim, num_keys, d.num_kv_heads, w.key_stride * d.head_dim));
  PCP_TRY(make_tmap(&to, final_out ? out : q, d.head_dim, R, d.num_kv_heads, R * d.head_dim));
  pcp::AttnParams p{};
  p.rows_per_head = static_cast<int>(R);
  p.m_tiles_per_head = static_cast<int>(mt);
  p.num_kv_heads = d.num_kv_heads;
  p.num_keys = static_cast<int>(num_keys);
  p.tiles_per_split = plan.tiles_per_split;
  p.split_base = split_base;
  p.total_rows = static_cast<int>(total_rows(d));
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(d.head_dim)) * 1.4426950408889634);
  // Stream-K decides per unit (final_ok); static writes bf16 O only when
  // each unit is one item (one split), else every split leaves a partial.
  p.write_final = (final_out && plan.splits == 1) ? 1 : 0;
  p.final_ok = final_out ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.max_segs = plan.splits;
  p.part_o = reinterpret_cast<float*>(ws + w.po_off);
  p.part_lse = reinterpret_cast<float*>(ws + w.pl_off);
  p.err = reinterpret_cast<int*>(ws);
  p.causal = causal.stripe_width > 0 ? 1 : 0;
  p.q_local_len = d.local_q_len;
  p.stripe_ranks = d.pcp_size;
  p.stripe_width = std::max(1, causal.stripe_width);
  p.stripe_rank = causal.rank;
  p.num_keys_dev = num_keys_dev;
  // Two CTAs (one cluster) per pair; the cluster shape is compiled in.
  // Stream-K: a fixed set of pairs; static: one pair per unit and split.
  const bool sk = plan.mode == kModeStreamK;
  if (!sk && causal.stripe_width == 0 && pingpong(d, false)) {
    // Two query tiles per pair: units of 512 rows.
    const int64_t mt2 = ceil_div(R, pcp::Pair2Roles::kUnitRows);
    p.m_tiles_per_head = static_cast<int>(mt2);
    const dim3 grid2(static_cast<unsigned>(2 * d.num_kv_heads * mt2), static_cast<unsigned>(plan.splits));
    static int done2 = 0;
    PCP_TRY(set_smem_attr(pcp::attn_fwd_pair2_kernel<128>, pcp::Pair2Smem<128>::kAlloc, &done2));
    // The kernel's register split (setmaxnreg) assumes its launch count: a
    // build that compiled it with another one is refused, never launched.
    static std::atomic<int> regs = 0;
    if (regs.load() == 0) {
      cudaFuncAttributes fa{};
      CUDA_TRY(cudaFuncGetAttributes(&fa, pcp::attn_fwd_pair2_kernel<128>));
      regs.store(fa.numRegs);
    }
    if (regs.load() != pcp::Pair2Roles::kLaunchRegs)
      return fail(PCP_ERR_UNSUPPORTED, "attn_fwd_pair2_kernel has %d registers per thread; its split needs %d",
                  regs.load(), pcp::Pair2Roles::kLaunchRegs);
    pcp::attn_fwd_pair2_kernel<128><<<grid2, pcp::Pair2Roles::kThreads, pcp::Pair2Smem<128>::kAlloc, st>>>(
        tq, tk, tv, to, p);
    CUDA_TRY(cudaGetLastError());
    if (lc) {
      lc->kernels++;
      lc->attn++;
    }
    return PCP_OK;
  }
  dim3 grid = sk ? dim3(static_cast<unsigned>(2 * plan.pairs), 1)
                            : dim3(static_cast<unsigned>(2 * d.num_kv_heads * mt), static_cast<unsigned>(plan.splits));
  if (d.head_dim == 256) {
    PCP_TRY((sk ? launch_pair_kernel<256, true>(grid, st, tq, tk, tv, to, p)
                : launch_pair_kernel<256, false>(grid, st, tq, tk, tv, to, p)));
  } else {
    PCP_TRY((sk ? launch_pair_kernel<128, true>(grid, st, tq, tk, tv, to, p)
                : launch_pair_kernel<128, false>(grid, st, tq, tk, tv, to, p)));
  }
  CUDA_TRY(cudaGetLastError());
  if (lc) {
    lc->kernels++;
    lc->attn++;
  }
  return PCP_OK;
}

// Current tokens of all P ranks ([P][Hkv][Qloc][D] bf16 each for K and V)
// -> dense workspace keys [key_off, key_off + P * Qloc) in global order.
int launch_scatter(const pcp_dims_t& d, const void* k_all, const void* v_all, int stripe_width, const Workspace& w,
                   uint8_t* ws, int64_t key_off, cudaStream_t st, LaunchCounter* lc) {
  if (reinterpret_cast<uintptr_t>(k_all) % 16 || reinterpret_cast<uintptr_t>(v_all) % 16)
    return fail(PCP_ERR_INVALID_ARGUMENT, "current K/V must be 16-byte aligned");
  pcp::ScatterParams p{};
  p.k_src = static_cast<const __nv_bfloat16*>(k_all);
  p.v_src = static_cast<const __nv_bfloat16*>(v_all);
  p.num_sources = d.pcp_size;
  p.num_kv_heads = d.num_kv_heads;
  p.local_len = d.local_q_len;
  p.head_dim = d.head_dim;
  p.stripe_width = stripe_width;
  p.key_stride = static_cast<int>(w.key_stride);
  p.key_off = static_cast<int>(key_off);
  p.k_out = reinterpret_cast<__nv_bfloat16*>(ws + w.k_off);
  p.v_out = reinterpret_cast<__nv_bfloat16*>(ws + w.v_off);
  const int64_t items = 2LL * d.pcp_size * d.num_kv_heads * d.local_q_len * (d.head_dim / 8);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, 256), 8 * 148));
  pcp::current_scatter_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  CUDA_TRY(cudaGetLastError());
  if (lc) lc->kernels++;
  return PCP_OK;
}

// Current-token keys of one forward (global order) and the check of their
// shape: P * Qloc keys, Qloc a whole number of stripes.
int64_t current_keys(const pcp_dims_t& d) { return static_cast<int64_t>(d.pcp_size) * d.local_q_len; }

int check_stripe(const pcp_dims_t& d, int stripe_width) {
  if (stripe_width <= 0 || d.local_q_len % stripe_width)
    return fail(PCP_ERR_INVALID_ARGUMENT, "interleave_size %d must be positive and divide local_q_len %d",
                stripe_width, d.local_q_len);
  if (current_keys(d) > (int64_t(1) << 30)) return fail(PCP_ERR_UNSUPPORTED, "too many current tokens");
  return PCP_OK;
}

// The causal current-token launch: one split, every pair tile stops at its
// last query's position.
SplitPlan causal_plan(const pcp_dims_t& d) {
  SplitPlan pl;
  pl.splits = 1;
  pl.tiles_per_split = static_cast<int>(ceil_div(current_keys(d), pcp::kTileN));
  pl.mode = kModeStatic;
  return pl;
}

// `single`: the plan of the only launch, which wrote its single-segment
// units as final output (rows the combine skips); null when every unit's
// result is in the partials.
// `count` / `count_dev`: the single launch's keys (dense) or key tiles (in
// place, `count_is_tiles`), as its kernel saw them.
int launch_combine(const pcp_dims_t& d, const Workspace& w, uint8_t* ws, int splits, void* out, cudaStream_t st,
                   LaunchCounter* lc, const SplitPlan* single = nullptr, int64_t count = 0,
                   const int* count_dev = nullptr, bool count_is_tiles = false) {
  pcp::CombineParams p{};
  if (single) {
    p.skip_single = 1;
    p.units = static_cast<int>(m_units(d));
    p.grid_pairs = single->pairs;
    p.rows_per_head = static_cast<int>(rows_per_head(d));
    p.m_tiles = static_cast<int>(ceil_div(rows_per_head(d), pcp::kPairRows));
    p.count = static_cast<int>(count);
    p.count_dev = count_dev;
    p.count_is_keys = count_is_tiles ? 0 : 1;
  }
  p.part_o = reinterpret_cast<const float*>(ws + w.po_off);
  p.part_lse = reinterpret_cast<const float*>(ws + w.pl_off);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.num_splits = splits;
  p.rows = static_cast<int>(total_rows(d));
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(p.rows, 8), 16 * 148));
  if (d.head_dim == 256)
    pcp::combine_kernel<256><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  else
    pcp::combine_kernel<128><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  CUDA_TRY(cudaGetLastError());
  if (lc) lc->kernels++;
  return PCP_OK;
}

// One attention "part" = a set of history sources attended in one launch:
// read in place from their cache blocks, or unpacked into a key range of the
// dense workspace first.
struct Part {
  bool in_place = false;
  std::vector<pcp::UnpackSource> srcs;  // every source (dense path: what the unpack reads)
  int64_t key_off = 0;                  // dense path: first workspace key
  int64_t keys = 0;
  int64_t tiles = 0;                    // key tiles of the launch (or their bound)
  SplitPlan plan;
  bool last = true;  // the forward's last history launch (no exchange in flight)
  int sms = 0;       // SMs the launch may use (0: all); fewer leave SMs to an exchange in flight
  // In place: the buffer holding the sources' blocks, its block count, and
  // the block-table entries / first blocks of the sources.
  const void* map_base = nullptr;
  int64_t map_blocks = 0;
  std::vector<pcp::KvSource> kv;
};

// Appends a history source of `valid` tokens (device-length mode: the bound)
// to a part.  Dense path: an unpack source at the part's next key.  In
// place: source `src` of the part's map, its logical block b at map block
// blk0 + b or table[b].
void add_source(const pcp_dims_t& d, Part* part, const uint8_t* base, const int32_t* table, int64_t pool_blocks,
                int valid, int dev_index, bool device_lengths) {
  const int64_t pay = payload_bytes(d);
  if (valid > 0) {
    const int64_t dst = device_lengths ? part->key_off : part->key_off + part->keys;
    part->srcs.push_back(table ? paged_src(base, table, pool_blocks, valid, dst, dev_index)
                               : contiguous_src(base, valid, dst, dev_index));
    pcp::KvSource k{};
    k.table = table;
    k.blk0 = (table || !part->map_base) ? 0 : (base - static_cast<const uint8_t*>(part->map_base)) / pay;
    k.valid = valid;
    k.dev_index = dev_index;
    part->kv.push_back(k);
  }
  part->keys += valid;
  part->tiles += part->in_place ? ceil_div(valid, pcp::kTileN) : 0;
}

// Key tiles a part's launch walks: per source when in place, over the
// compacted keys otherwise.
int64_t part_tiles(const Part& part) {
  return part.in_place ? part.tiles : ceil_div(part.keys, pcp::kTileN);
}

int plan_part(const pcp_dims_t& d, Part* part, int sms, int max_splits) {
  if (part->keys == 0) return PCP_OK;
  if (part->sms > 0 && part->sms < sms) {
    // A launch that shares the GPU with an exchange: a persistent grid on
    // part->sms SMs (stream-K; the caller checked that its K/V fits in L2).
    part->plan = plan_stream_k(m_units(d), part_tiles(*part), part->sms, max_splits);
    return PCP_OK;
  }
  part->plan = plan_splits(d, part_tiles(*part), part->keys, sms, max_splits, part->last, part->in_place);
  return PCP_OK;
}

// Attention over the e4m3 cache blocks of `part` read in place
// (attn_fwd_kv_kernel).  Writes bf16 `out` directly (final, one segment per
// unit) or split partials.  `tiles_dev` (device-length mode): where the
// kernel stores the key tiles it walked, for the combine.
int launch_attention_kv(const pcp_dims_t& d, const void* q, const Part& part, uint8_t* ws, const Workspace& w,
                        int split_base, bool final_out, void* out, cudaStream_t st, LaunchCounter* lc,
                        const int32_t* valid_dev = nullptr, int* tiles_dev = nullptr) {
  const SplitPlan& plan = part.plan;
  if (part.kv.size() > static_cast<size_t>(pcp::kMaxSources)) return fail(PCP_ERR_UNSUPPORTED, "too many sources");
  const int64_t R = rows_per_head(d);
  const int64_t mt = ceil_div(R, pcp::kPairRows);
  CUtensorMap tq, tk, tv;
  PCP_TRY(make_tmap(&tq, q, d.head_dim, R, d.num_kv_heads, R * d.head_dim));
  PCP_TRY(make_tmap_blocks(&tk, part.map_base, d, part.map_blocks, d.head_dim));
  PCP_TRY(make_tmap_blocks(&tv, part.map_base, d, part.map_blocks, d.head_dim / 2));
  pcp::KvParams kp{};
  pcp::AttnParams& p = kp.a;
  p.rows_per_head = static_cast<int>(R);
  p.m_tiles_per_head = static_cast<int>(mt);
  p.num_kv_heads = d.num_kv_heads;
  p.tiles_per_split = plan.tiles_per_split;
  p.split_base = split_base;
  p.total_rows = static_cast<int>(total_rows(d));
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(d.head_dim)) * 1.4426950408889634);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.max_segs = plan.splits;
  p.final_ok = final_out ? 1 : 0;
  p.part_o = reinterpret_cast<float*>(ws + w.po_off);
  p.part_lse = reinterpret_cast<float*>(ws + w.pl_off);
  p.err = reinterpret_cast<int*>(ws);
  for (size_t i = 0; i < part.kv.size(); ++i) kp.src[i] = part.kv[i];
  kp.num_sources = static_cast<int>(part.kv.size());
  kp.block_size = d.block_size;
  kp.map_blocks = part.map_blocks;
  kp.valid_dev = valid_dev;
  kp.tiles_out = tiles_dev;
  const bool sk = plan.mode == kModeStreamK;
  kp.sched = sk ? pcp::kSchedStreamK : pcp::kSchedStatic;
  const dim3 grid = sk ? dim3(static_cast<unsigned>(2 * plan.pairs), 1)
                       : dim3(static_cast<unsigned>(2 * d.num_kv_heads * mt), static_cast<unsigned>(plan.splits));
  static int done = 0;
  if (d.head_dim == 256) {
    PCP_TRY(set_smem_attr(pcp::attn_fwd_kv_kernel<256>, pcp::KvSmem<256>::kAlloc, &done));
    pcp::attn_fwd_kv_kernel<256><<<grid, pcp::kKvThreads, pcp::KvSmem<256>::kAlloc, st>>>(tq, tk, tv, kp);
  } else {
    static int done128 = 0;
    PCP_TRY(set_smem_attr(pcp::attn_fwd_kv_kernel<128>, pcp::KvSmem<128>::kAlloc, &done128));
    pcp::attn_fwd_kv_kernel<128><<<grid, pcp::kKvThreads, pcp::KvSmem<128>::kAlloc, st>>>(tq, tk, tv, kp);
  }
  CUDA_TRY(cudaGetLastError());
  if (lc) {
    lc->kernels++;
    lc->attn++;
  }
  return PCP_OK;
}

// The part of a stateless call: `num_sources` shards back to back in
// `packed_kv`, `max_local_blocks` blocks each, source s with valid_len[s]
// tokens.
int packed_part(const pcp_dims_t& d, const void* packed_kv, int num_sources, const int32_t* valid_len, Part* part,
                int mode) {
  const int64_t cap = static_cast<int64_t>(d.max_local_blocks) * d.block_size;
  const int64_t pay = payload_bytes(d);
  part->in_place = choose_in_place(d, mode);
  part->map_base = packed_kv;
  part->map_blocks = static_cast<int64_t>(num_sources) * d.max_local_blocks;
  for (int s = 0; s < num_sources; ++s) {
    if (valid_len[s] < 0 || valid_len[s] > cap)
      return fail(PCP_ERR_INVALID_ARGUMENT, "valid_len[%d]=%d outside [0, %lld]", s, valid_len[s],
                  static_cast<long long>(cap));
    if (valid_len[s] > 0 && !packed_kv) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL packed_kv");
    add_source(d, part, static_cast<const uint8_t*>(packed_kv) + static_cast<size_t>(s) * d.max_local_blocks * pay,
               nullptr, 0, valid_len[s], -1, false);
  }
  return PCP_OK;
}

// Dense workspace keys of a history over `keys` keys: none when the cache is
// read in place.
int64_t dense_keys(int64_t keys, bool in_place) { return in_place ? 0 : keys; }

// Plan of a stateless launch: made from the total key count alone (all the
// workspace-size queries see), then fitted to the part's actual key tiles.
SplitPlan stateless_plan(const pcp_dims_t& d, const Part& part, int slot_cap) {
  const SplitPlan pl =
      plan_splits(d, ceil_div(part.keys, pcp::kTileN), part.keys, num_sms(), slot_cap, true, part.in_place);
  return fit_plan(pl, part_tiles(part));
}

// The launches of one stateless history part: its attention (in place, or
// unpack + dense) writing bf16 `out` where one segment covers a unit, and
// the combine when it left partials.
int run_single_part(const pcp_dims_t& d, const void* q, const Part& part, const Workspace& w, uint8_t* ws, void* out,
                    cudaStream_t st) {
  const bool in_place = part.in_place;
  if (in_place) {
    PCP_TRY(launch_attention_kv(d, q, part, ws, w, 0, true, out, st, nullptr));
  } else {
    PCP_TRY(launch_unpack(d, part.srcs, w, ws, st, nullptr));
    PCP_TRY(launch_attention(d, q, w, ws, 0, part.keys, part.plan, 0, true, out, st, nullptr));
  }
  if (part.plan.splits > 1)
    PCP_TRY(launch_combine(d, w, ws, part.plan.splits, out, st, nullptr,
                           part.plan.mode == kModeStreamK ? &part.plan : nullptr,
                           in_place ? part.tiles : part.keys, nullptr, in_place));
  return PCP_OK;
}

// ---------------------------------------------------------- bounded-wait probe --
__global__ void bounded_wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    pcp::mbar_init(pcp::smem_u32(&bar), 1);
    pcp::fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must give up by itself.
  if (threadIdx.x == 0) {
    const uint32_t b = pcp::smem_u32(&bar);
    const uint64_t t0 = pcp::globaltimer_ns();
    bool done = false;
    while (!done) {
      if (pcp::mbar_try_wait(b, 0)) break;
      if (pcp::globaltimer_ns() - t0 > limit_ns) {
        atomicCAS(err, 0, 199);
        done = true;
      }
    }
  }
  __syncthreads();
}

}  // namespace

// ============================================================ C ABI ======
struct pcp_handle {
  pcp_dims_t d{};
  int rank = 0;
  int device = 0;
  int sms = 148;
  ncclComm_t comm = nullptr;
  bool comm_failed = false;
  cudaStream_t comm_stream = nullptr;
  cudaStream_t last_stream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_comm = nullptr;
  cudaEvent_t ev_group[2] = {nullptr, nullptr};  // direct exchange: shards of each peer group landed
  std::vector<cudaEvent_t> ev_step;              // pipelined exchange: shards of each step chunk landed
  cudaEvent_t ev_cur = nullptr;                  // current tokens' K/V of every rank landed
  uint8_t* ring = nullptr;  // [P][max_local_blocks][payload]: slot s receives source s
  uint8_t* stage = nullptr;  // [max_local_blocks][payload]: a paged shard's blocks gathered for sending
  uint8_t* cur_k = nullptr;  // [P][Hkv][Qloc][D] bf16: current tokens' K of every rank (P > 1)
  uint8_t* cur_v = nullptr;
  int exchange = PCP_EXCHANGE_DIRECT;
  int kv_path = -1;   // PCP_KV_PATH_* for this handle; -1: the process default
  int comm_sms = 16;  // SMs left to the direct exchange while the local shard is attended (P >= 4)
  uint8_t* ws = nullptr;
  Workspace w;
  // Staging of the host-buffer entries: two slots of device Q, packed KV and
  // O, so that one call's copies (H2D on h2d_stream, D2H on d2h_stream)
  // overlap another call's forward.
  struct HostSlot {
    void* q = nullptr;
    void* kv = nullptr;
    void* out = nullptr;
    cudaEvent_t loaded = nullptr;   // inputs copied in
    cudaEvent_t done = nullptr;     // forward finished (inputs free, output written)
    cudaEvent_t fetched = nullptr;  // output copied out
    bool used = false;
  };
  HostSlot slots[2];
  int next_slot = 0;
  cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
  // Profiling: CUDA event pairs recorded around every launch (on the
  // stream it is launched on) while profiling is on; resolved lazily.
  bool profiling = false;
  struct Span {
    cudaEvent_t start, end;
    int slot;  // 0 ring exchange, 1 unpack, 2 attention, 3 combine
  };
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<Span> spans;
  pcp_stats_t last{};   // counts of the last forward
  pcp_stats_t accum{};  // counts accumulated since profiling was enabled
};

namespace {

int wait_nccl(ncclComm_t comm, ncclResult_t r, int timeout_ms) {
  if (r == ncclSuccess) return PCP_OK;
  if (r != ncclInProgress) return fail(PCP_ERR_NCCL, "NCCL: %s", ncclGetErrorString(r));
  // A non-blocking communicator finishes enqueueing a group on its own
  // thread, usually within microseconds: poll with yields for the first
  // 2 ms (a forward's host path must stay well under its device time), then
  // with short sleeps up to the timeout.
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t st = ncclInProgress;
  while (true) {
    ncclCommGetAsyncError(comm, &st);
    if (st != ncclInProgress) break;
    const auto waited = std::chrono::steady_clock::now() - t0;
    if (waited > std::chrono::milliseconds(timeout_ms)) {
      return fail(PCP_ERR_PEER, "NCCL operation still in progress after %d ms (peer missing?)", timeout_ms);
    }
    if (waited < std::chrono::milliseconds(2))
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  if (st != ncclSuccess) return fail(PCP_ERR_NCCL, "NCCL async error: %s", ncclGetErrorString(st));
  return PCP_OK;
}

cudaEvent_t take_event(pcp_handle* h) {
  if (h->ev_used == h->ev_pool.size()) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    h->ev_pool.push_back(e);
  }
  return h->ev_pool[h->ev_used++];
}

// Returns the span index (or -1 when profiling is off).
int prof_begin(pcp_handle* h, int slot, cudaStream_t st) {
  if (!h->profiling) return -1;
  cudaEvent_t a = take_event(h), b = take_event(h);
  if (!a || !b) return -1;
  cudaEventRecord(a, st);
  h->spans.push_back({a, b, slot});
  return static_cast<int>(h->spans.size()) - 1;
}

void prof_end(pcp_handle* h, int idx, cudaStream_t st) {
  if (idx >= 0) cudaEventRecord(h->spans[idx].end, st);
}

// This rank's history shard: contiguous packed blocks (table NULL), or
// logical blocks of a block pool read through a device block table.
struct LocalKV {
  const void* base = nullptr;
  const int32_t* table = nullptr;
  int64_t pool_blocks = 0;
};

int launch_block_gather(const pcp_dims_t& d, const LocalKV& local, int live_blocks, void* dst, uint8_t* ws,
                        cudaStream_t st) {
  if (live_blocks <= 0) return PCP_OK;
  pcp::BlockGatherParams p{};
  p.pool = static_cast<const uint8_t*>(local.base);
  p.table = local.table;
  p.pool_blocks = local.pool_blocks;
  p.live_blocks = live_blocks;
  p.payload = payload_bytes(d);
  p.out = static_cast<uint8_t*>(dst);
  p.err = reinterpret_cast<int*>(ws);
  const int64_t items = p.payload / 16 * live_blocks;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, 256), 2 * 148));
  pcp::block_gather_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  CUDA_TRY(cudaGetLastError());
  return PCP_OK;
}

// k_cur / v_cur (optional, both or neither): this rank's current tokens'
// K/V shard [Hkv][Qloc][D] bf16, striped like Q with `stripe_width`; they are
// gathered from every rank and attended causally as one more split.
// Restores the handle's profiling switch on scope exit (forwards recorded
// into a CUDA graph take no profiling spans).
struct ProfilingOff {
  pcp_handle* h;
  bool saved;
  ProfilingOff(pcp_handle* hh, bool off) : h(hh), saved(hh->profiling) {
    if (off) h->profiling = false;
  }
  ~ProfilingOff() { h->profiling = saved; }
};

// valid_dev (optional, device int32[P]): device-length mode.  valid_len then
// holds each source's upper bound (the bucket): transfers, key regions,
// split plans and grids are sized by the bounds, while the kernels read the
// actual counts from valid_dev -- so one CUDA graph recorded for a bucket
// serves every length inside it and still skips every tile past them.
int forward_impl(pcp_handle* h, const void* q, const LocalKV& local, const int32_t* valid_len, const void* k_cur,
                 const void* v_cur, int stripe_width, void* out, cudaStream_t st,
                 const int32_t* valid_dev = nullptr) {
  const pcp_dims_t& d = h->d;
  const int P = d.pcp_size;
  const int r = h->rank;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  CUDA_TRY(cudaStreamIsCapturing(st, &capture));
  ProfilingOff prof_guard(h, capture != cudaStreamCaptureStatusNone);
  if (!q || !local.base || !valid_len || !out) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  if (local.table && local.pool_blocks <= 0) return fail(PCP_ERR_INVALID_ARGUMENT, "empty block pool");
  const bool with_cur = k_cur != nullptr || v_cur != nullptr;
  if (with_cur) {
    if (!k_cur || !v_cur) return fail(PCP_ERR_INVALID_ARGUMENT, "current K and V must both be given");
    PCP_TRY(check_stripe(d, stripe_width));
  }
  const int64_t cap = static_cast<int64_t>(d.max_local_blocks) * d.block_size;
  int64_t total = 0;
  for (int s = 0; s < P; ++s) {
    if (valid_len[s] < 0 || valid_len[s] > cap)
      return fail(PCP_ERR_INVALID_ARGUMENT, "valid_len[%d]=%d outside [0, %lld]", s, valid_len[s],
                  static_cast<long long>(cap));
    total += valid_len[s];
  }
  if (total == 0 && !with_cur) return fail(PCP_ERR_INVALID_ARGUMENT, "no valid history tokens");
  // How the history is read (the handle's setting, else the process
  // default), and the dense workspace keys: the unpacked history (none in
  // place), then the current tokens of a prefill.
  const bool in_place = choose_in_place(d, h->kv_path >= 0 ? h->kv_path : g_kv_path.load());
  const int64_t cur_off = dense_keys(total, in_place);
  if (cur_off + (with_cur ? current_keys(d) : 0) > h->w.key_stride)
    return fail(PCP_ERR_UNSUPPORTED, "workspace holds %lld keys", static_cast<long long>(h->w.key_stride));
  CUDA_TRY(cudaSetDevice(h->device));
  h->last_stream = st;
  LaunchCounter lc;
  const int64_t pay = payload_bytes(d);
  const int max_splits = h->w.max_splits;

  // Parts: the local shard, then the remote shards (one part, or one per
  // peer group with the direct exchange), each attended in its own launch
  // once its shards have landed; their split partials meet in one combine.
  std::vector<Part> parts(1);
  std::vector<cudaEvent_t> ready(1, nullptr);  // event a part waits for (null: none)
  parts[0].in_place = in_place;
  parts[0].key_off = 0;
  parts[0].map_base = local.base;
  parts[0].map_blocks = local.table ? local.pool_blocks : d.max_local_blocks;
  add_source(d, &parts[0], static_cast<const uint8_t*>(local.base), local.table, local.pool_blocks, valid_len[r], r,
             valid_dev != nullptr);
  int64_t next_key = parts[0].keys;
  int64_t sent = 0;
  // Cleared before the ring stream starts: its block gather may report too.
  CUDA_TRY(cudaMemsetAsync(h->ws, 0, 4, st));
  if (P > 1) {
    CUDA_TRY(cudaEventRecord(h->ev_in, st));
    CUDA_TRY(cudaStreamWaitEvent(h->comm_stream, h->ev_in, 0));
    const int pc = prof_begin(h, 0, h->comm_stream);
    if (with_cur) {
      // Current tokens first: small, and attended right after the local shard.
      const size_t n = static_cast<size_t>(d.num_kv_heads) * d.local_q_len * d.head_dim;
      ncclResult_t nr = ncclGroupStart();
      if (nr != ncclSuccess) return fail(PCP_ERR_NCCL, "ncclGroupStart: %s", ncclGetErrorString(nr));
      ncclAllGather(k_cur, h->cur_k, n, ncclBfloat16, h->comm, h->comm_stream);
      ncclAllGather(v_cur, h->cur_v, n, ncclBfloat16, h->comm, h->comm_stream);
      PCP_TRY(wait_nccl(h->comm, ncclGroupEnd(), 600000));
      CUDA_TRY(cudaEventRecord(h->ev_cur, h->comm_stream));
      sent += static_cast<int64_t>(2 * n * 2) * (P - 1);
    }
    auto live = [&](int src) { return static_cast<size_t>(ceil_div(valid_len[src], d.block_size)) * pay; };
    // All-gather slots are as long as the longest live shard; the other
    // modes keep one full shard per slot.
    size_t slot_stride = static_cast<size_t>(d.max_local_blocks) * pay;
    if (h->exchange == PCP_EXCHANGE_ALLGATHER) {
      slot_stride = 0;
      for (int src = 0; src < P; ++src) slot_stride = std::max(slot_stride, live(src));
    }
    auto slot = [&](int src) { return h->ring + static_cast<size_t>(src) * slot_stride; };
    // What this rank sends: its packed shard, or (paged) its live blocks
    // gathered into a contiguous buffer first -- slot r for the all-gather,
    // the staging buffer otherwise.
    const void* own = local.base;
    if (local.table) {
      void* dst = h->exchange == PCP_EXCHANGE_ALLGATHER ? static_cast<void*>(slot(r)) : h->stage;
      PCP_TRY(launch_block_gather(d, local, static_cast<int>(ceil_div(valid_len[r], d.block_size)), dst, h->ws,
                                  h->comm_stream));
      own = dst;
    }
    // Remote part over ring steps [s0, s1): sources (rank - s) % P, in ring
    // order; in place, their blocks are read from the receive slots.
    auto add_part = [&](int s0, int s1, cudaEvent_t ev) {
      Part part;
      part.in_place = in_place;
      part.key_off = next_key;
      part.map_base = h->ring;
      part.map_blocks = static_cast<int64_t>(P) * static_cast<int64_t>(slot_stride / pay);
      for (int step = s0; step < s1; ++step) {
        const int src = ((r - step) % P + P) % P;
        add_source(d, &part, slot(src), nullptr, 0, valid_len[src], src, valid_dev != nullptr);
      }
      next_key += part.keys;
      parts.push_back(part);
      ready.push_back(ev);
    };
    if (h->exchange == PCP_EXCHANGE_RING) {
      // Store-and-forward ring (reference.py:68-71 order, kernel.py:276-293):
      // hop s sends the shard received at hop s-1 (own shard at s = 1) to
      // rank+1 and receives source (rank - s) % P from rank-1.
      for (int hop = 1; hop < P; ++hop) {
        const int ssrc = ((r - hop + 1) % P + P) % P;
        const int rsrc = ((r - hop) % P + P) % P;
        const void* sbuf = hop == 1 ? own : slot(ssrc);
        ncclResult_t nr = ncclGroupStart();
        if (nr != ncclSuccess) return fail(PCP_ERR_NCCL, "ncclGroupStart: %s", ncclGetErrorString(nr));
        if (live(ssrc)) ncclSend(sbuf, live(ssrc), ncclUint8, (r + 1) % P, h->comm, h->comm_stream);
        if (live(rsrc)) ncclRecv(slot(rsrc), live(rsrc), ncclUint8, (r - 1 + P) % P, h->comm, h->comm_stream);
        PCP_TRY(wait_nccl(h->comm, ncclGroupEnd(), 600000));
        sent += static_cast<int64_t>(live(ssrc));
      }
      CUDA_TRY(cudaEventRecord(h->ev_comm, h->comm_stream));
      add_part(1, P, h->ev_comm);
    } else if (h->exchange == PCP_EXCHANGE_ALLGATHER) {
      // One all-gather of equal-length slots (the longest live shard; at most
      // one block longer than any other): lets NCCL use NVLink SHARP
      // (multicast through the switch) where the system offers it.
      if (slot_stride) {
        if (own != slot(r))
          CUDA_TRY(cudaMemcpyAsync(slot(r), own, live(r), cudaMemcpyDeviceToDevice, h->comm_stream));
        PCP_TRY(wait_nccl(h->comm, ncclAllGather(slot(r), h->ring, slot_stride, ncclUint8, h->comm, h->comm_stream),
                          600000));
        sent += static_cast<int64_t>(slot_stride) * (P - 1);
      }
      CUDA_TRY(cudaEventRecord(h->ev_comm, h->comm_stream));
      add_part(1, P, h->ev_comm);
    } else if (h->exchange == PCP_EXCHANGE_PIPELINE) {
      // Direct sends and receives, one NCCL group per chunk of ring steps
      // (one step per chunk up to kMaxParts - 1 chunks): each chunk's shards
      // are attended as soon as they land while the later chunks travel.
      const int chunks = std::min<int>(P - 1, static_cast<int>(h->ev_step.size()));
      for (int k = 0; k < chunks; ++k) {
        const int s0 = 1 + (P - 1) * k / chunks;
        const int s1 = 1 + (P - 1) * (k + 1) / chunks;
        ncclResult_t nr = ncclGroupStart();
        if (nr != ncclSuccess) return fail(PCP_ERR_NCCL, "ncclGroupStart: %s", ncclGetErrorString(nr));
        for (int step = s0; step < s1; ++step) {
          const int to = (r + step) % P;
          const int from = ((r - step) % P + P) % P;
          if (live(r)) ncclSend(own, live(r), ncclUint8, to, h->comm, h->comm_stream);
          if (live(from)) ncclRecv(slot(from), live(from), ncclUint8, from, h->comm, h->comm_stream);
          sent += static_cast<int64_t>(live(r));
        }
        PCP_TRY(wait_nccl(h->comm, ncclGroupEnd(), 600000));
        CUDA_TRY(cudaEventRecord(h->ev_step[k], h->comm_stream));
        add_part(s0, s1, h->ev_step[k]);
      }
    } else {
      // Direct exchange over NVSwitch: each rank sends its own shard to every
      // peer and receives every peer's shard straight from its owner -- the
      // same bytes per rank as the ring, no forwarding chain, and no shard
      // returns to its owner.  Pairs match across ranks: at step s rank r
      // sends to r+s, which receives from (r+s)-s = r in the same group.
      // With at least 4 ranks the exchange is long enough to matter, and
      // NCCL's kernels need SMs while the local shard is attended:
      //   * local K/V fits in L2: attend it on a persistent grid that leaves
      //     comm_sms SMs to NCCL; all peers travel in one group meanwhile;
      //   * else, when the local wave-scheduled launch fills every SM pair
      //     (NCCL then only gets SMs between waves): two groups (ring steps
      //     1..ceil((P-1)/2), then the rest), the first group's shards
      //     attended while the second group's travel;
      //   * else one group (fewer launches and split partials).
      const bool reserve = P >= 4 && h->comm_sms > 0 && h->comm_sms < h->sms && parts[0].keys > 0 &&
                           kv_bytes(d, valid_len[r], in_place) <= kStreamKMaxKvBytes;
      if (reserve) parts[0].sms = h->sms - h->comm_sms;
      Part probe = parts[0];
      probe.last = false;
      probe.sms = 0;
      plan_part(d, &probe, h->sms, max_splits);
      const bool local_fills_gpu =
          probe.keys && static_units(d, in_place) * probe.plan.splits >= std::max(1, h->sms / 2);
      const int groups = (P >= 4 && !reserve && local_fills_gpu) ? 2 : 1;
      const int split_step = 1 + (P - 1 + 1) / 2;
      for (int g = 0; g < groups; ++g) {
        const int s0 = g == 0 ? 1 : split_step;
        const int s1 = (g == 0 && groups == 2) ? split_step : P;
        ncclResult_t nr = ncclGroupStart();
        if (nr != ncclSuccess) return fail(PCP_ERR_NCCL, "ncclGroupStart: %s", ncclGetErrorString(nr));
        for (int step = s0; step < s1; ++step) {
          const int to = (r + step) % P;
          const int from = ((r - step) % P + P) % P;
          if (live(r)) ncclSend(own, live(r), ncclUint8, to, h->comm, h->comm_stream);
          if (live(from)) ncclRecv(slot(from), live(from), ncclUint8, from, h->comm, h->comm_stream);
          sent += static_cast<int64_t>(live(r));
        }
        PCP_TRY(wait_nccl(h->comm, ncclGroupEnd(), 600000));
        CUDA_TRY(cudaEventRecord(h->ev_group[g], h->comm_stream));
        add_part(s0, s1, h->ev_group[g]);
      }
    }
    prof_end(h, pc, h->comm_stream);
  }
  // Split plans; keep the total within the partial buffers by shrinking the
  // part with the most splits (the current tokens take one split).
  const int hist_cap = max_splits - (with_cur ? 1 : 0);
  // Only the last launch that has keys runs with no exchange in flight.
  int last_live = -1;
  for (size_t i = 0; i < parts.size(); ++i) {
    parts[i].last = false;
    if (parts[i].keys) last_live = static_cast<int>(i);
  }
  if (last_live >= 0) parts[last_live].last = true;
  // Pipelined exchange: every launch but the last shares the GPU with chunks
  // still in flight -- on a persistent grid that leaves comm_sms SMs to NCCL
  // where its K/V fits in L2.
  if (P > 1 && h->exchange == PCP_EXCHANGE_PIPELINE && h->comm_sms > 0 && h->comm_sms < h->sms)
    for (auto& part : parts)
      if (part.keys && !part.last && kv_bytes(d, part.keys, in_place) <= kStreamKMaxKvBytes)
        part.sms = h->sms - h->comm_sms;
  int total_splits = 0;
  for (auto& part : parts) {
    plan_part(d, &part, h->sms, hist_cap);
    total_splits += part.keys ? part.plan.splits : 0;
  }
  while (total_splits > hist_cap) {
    Part* big = nullptr;
    for (auto& part : parts)
      if (part.keys && (!big || part.plan.splits > big->plan.splits)) big = &part;
    if (!big || big->plan.splits == 1) return fail(PCP_ERR_UNSUPPORTED, "too many launches for the partial buffers");
    const int others = total_splits - big->plan.splits;
    plan_part(d, big, h->sms, std::max(1, std::min(big->plan.splits - 1, hist_cap - others)));
    total_splits = others + big->plan.splits;
  }
  if (with_cur) ++total_splits;
  int live_parts = 0;
  const Part* only = nullptr;
  for (const auto& part : parts)
    if (part.keys) {
      ++live_parts;
      only = &part;
    }
  // One history launch and nothing else: it writes its single-segment units
  // as final output.  Only the current tokens: the causal launch does.
  const bool single = live_parts == 1 && !with_cur;
  const bool cur_only = live_parts == 0 && with_cur;
  if (parts.size() > static_cast<size_t>(kMaxParts)) return fail(PCP_ERR_UNSUPPORTED, "too many parts");
  int split_base = 0;
  // Current tokens: scatter every rank's shard into sequence order after the
  // history keys, then one causal launch.
  auto launch_current = [&]() -> int {
    if (P > 1) CUDA_TRY(cudaStreamWaitEvent(st, h->ev_cur, 0));
    int sp = prof_begin(h, 1, st);
    PCP_TRY(launch_scatter(d, P > 1 ? h->cur_k : k_cur, P > 1 ? h->cur_v : v_cur, stripe_width, h->w, h->ws, cur_off,
                           st, &lc));
    prof_end(h, sp, st);
    sp = prof_begin(h, 2, st);
    PCP_TRY(launch_attention(d, q, h->w, h->ws, cur_off, current_keys(d), causal_plan(d), split_base, cur_only, out,
                             st, &lc, Causal{r, stripe_width}));
    prof_end(h, sp, st);
    split_base += 1;
    return PCP_OK;
  };
  for (size_t i = 0; i < parts.size(); ++i) {
    if (i == 1 && with_cur) PCP_TRY(launch_current());
    if (ready[i]) CUDA_TRY(cudaStreamWaitEvent(st, ready[i], 0));
    const Part& part = parts[i];
    if (!part.keys) continue;
    int* count_dev = valid_dev ? part_keys_slot(h->ws, static_cast<int>(i)) : nullptr;
    if (in_place) {
      const int sp = prof_begin(h, 2, st);
      PCP_TRY(launch_attention_kv(d, q, part, h->ws, h->w, split_base, single, out, st, &lc, valid_dev, count_dev));
      prof_end(h, sp, st);
    } else {
      int sp = prof_begin(h, 1, st);
      PCP_TRY(launch_unpack(d, part.srcs, h->w, h->ws, st, &lc, valid_dev, count_dev));
      prof_end(h, sp, st);
      sp = prof_begin(h, 2, st);
      PCP_TRY(launch_attention(d, q, h->w, h->ws, part.key_off, part.keys, part.plan, split_base, single, out, st,
                               &lc, Causal{}, count_dev));
      prof_end(h, sp, st);
    }
    split_base += part.plan.splits;
  }
  if (parts.size() == 1 && with_cur) PCP_TRY(launch_current());
  if (single ? only->plan.splits > 1 : !cur_only) {
    const int sp = prof_begin(h, 3, st);
    const int only_idx = single ? static_cast<int>(only - parts.data()) : 0;
    const bool skip = single && only->plan.mode == kModeStreamK;
    PCP_TRY(launch_combine(d, h->w, h->ws, total_splits, out, st, &lc, skip ? &only->plan : nullptr,
                           single ? (in_place ? only->tiles : only->keys) : 0,
                           single && valid_dev ? part_keys_slot(h->ws, only_idx) : nullptr, in_place));
    prof_end(h, sp, st);
  }
  pcp_stats_t& L = h->last;
  L = pcp_stats_t{};
  L.kernel_launches = lc.kernels;
  L.attn_launches = lc.attn;
  L.splits = total_splits;
  L.forwards = 1;
  L.ring_bytes = sent;
  L.keys = total;
  L.kv_in_place = in_place ? 1 : 0;
  if (h->profiling) {
    pcp_stats_t& A = h->accum;
    A.kernel_launches += lc.kernels;
    A.attn_launches += lc.attn;
    A.splits = total_splits;
    A.forwards += 1;
    A.ring_bytes += sent;
    A.keys = total;
    A.kv_in_place = in_place ? 1 : 0;
  }
  return PCP_OK;
}

}  // namespace

extern "C" {

const char* pcp_last_error(void) { return g_err; }

int pcp_abi_version(void) { return PCP_ATTN_ABI_VERSION; }

int64_t pcp_source_valid_len(int64_t total_len, int32_t pcp_size, int32_t interleave_size, int32_t rank) {
  if (total_len < 0 || pcp_size <= 0 || interleave_size <= 0 || rank < 0 || rank >= pcp_size) return -1;
  const int64_t stride = static_cast<int64_t>(pcp_size) * interleave_size;
  const int64_t full = total_len / stride, tail = total_len % stride;
  const int64_t extra = std::min<int64_t>(std::max<int64_t>(tail - static_cast<int64_t>(rank) * interleave_size, 0),
                                          interleave_size);
  return full * interleave_size + extra;
}

int pcp_ring_schedule(int32_t rank, int32_t pcp_size, int32_t hop, int32_t* send_source, int32_t* recv_source,
                      int32_t* send_to, int32_t* recv_from) {
  if (pcp_size <= 0 || rank < 0 || rank >= pcp_size || hop < 1 || hop >= pcp_size)
    return fail(PCP_ERR_INVALID_ARGUMENT, "hop %d outside [1, %d) or rank %d outside [0, %d)", hop, pcp_size, rank,
                pcp_size);
  if (send_source) *send_source = ((rank - hop + 1) % pcp_size + pcp_size) % pcp_size;
  if (recv_source) *recv_source = ((rank - hop) % pcp_size + pcp_size) % pcp_size;
  if (send_to) *send_to = (rank + 1) % pcp_size;
  if (recv_from) *recv_from = (rank - 1 + pcp_size) % pcp_size;
  return PCP_OK;
}

int pcp_nccl_unique_id_bytes(void) { return static_cast<int>(sizeof(ncclUniqueId)); }

int pcp_get_nccl_unique_id(void* out) {
  if (!out) return fail(PCP_ERR_INVALID_ARGUMENT, "out is NULL");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return fail(PCP_ERR_NCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
  std::memcpy(out, &id, sizeof(id));
  return PCP_OK;
}

int pcp_history_attention_workspace_size(const pcp_dims_t* dims, int64_t total_valid, size_t* bytes) {
  PCP_TRY(check_dims(dims));
  if (!bytes || total_valid < 0) return fail(PCP_ERR_INVALID_ARGUMENT, "bad arguments");
  const int ms = max_splits_for(*dims);
  const bool ip = choose_in_place(*dims, g_kv_path.load());
  const SplitPlan plan =
      plan_splits(*dims, ceil_div(total_valid, pcp::kTileN), total_valid, num_sms(), ms, true, ip);
  *bytes = ws_layout(*dims, dense_keys(total_valid, ip), plan.splits).total;
  return PCP_OK;
}

int pcp_history_attention(const pcp_dims_t* dims, const void* q, const void* packed_kv, int32_t num_sources,
                          const int32_t* valid_len, void* out, void* workspace, size_t workspace_bytes,
                          void* stream) {
  PCP_TRY(check_dims(dims));
  const pcp_dims_t& d = *dims;
  if (!q || !packed_kv || !valid_len || !out || !workspace)
    return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  if (num_sources <= 0 || num_sources > pcp::kMaxSources)
    return fail(PCP_ERR_INVALID_ARGUMENT, "num_sources %d outside [1, %d]", num_sources, pcp::kMaxSources);
  Part part;
  PCP_TRY(packed_part(d, packed_kv, num_sources, valid_len, &part, g_kv_path.load()));
  if (part.keys == 0) return fail(PCP_ERR_INVALID_ARGUMENT, "no valid history tokens");
  part.plan = stateless_plan(d, part, max_splits_for(d));
  const Workspace w = ws_layout(d, dense_keys(part.keys, part.in_place), part.plan.splits);
  if (workspace_bytes < w.total)
    return fail(PCP_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is below the %zu required", workspace_bytes, w.total);
  auto* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemsetAsync(ws, 0, 4, st));
  return run_single_part(d, q, part, w, ws, out, st);
}

int pcp_prefill_attention_workspace_size(const pcp_dims_t* dims, int64_t total_valid, size_t* bytes) {
  PCP_TRY(check_dims(dims));
  if (!bytes || total_valid < 0) return fail(PCP_ERR_INVALID_ARGUMENT, "bad arguments");
  int splits = 0;
  const bool ip = choose_in_place(*dims, g_kv_path.load());
  if (total_valid > 0)
    splits = plan_splits(*dims, ceil_div(total_valid, pcp::kTileN), total_valid, num_sms(),
                         max_splits_for(*dims) - 1, true, ip).splits;
  *bytes = ws_layout(*dims, dense_keys(total_valid, ip) + current_keys(*dims), splits + 1).total;
  return PCP_OK;
}

int pcp_prefill_attention(const pcp_dims_t* dims, int32_t interleave_size, int32_t rank, const void* q,
                          const void* packed_kv, int32_t num_sources, const int32_t* valid_len, const void* k_cur_all,
                          const void* v_cur_all, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  PCP_TRY(check_dims(dims));
  const pcp_dims_t& d = *dims;
  if (!q || (!valid_len && num_sources > 0) || !k_cur_all || !v_cur_all || !out || !workspace)
    return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  PCP_TRY(check_stripe(d, interleave_size));
  if (rank < 0 || rank >= d.pcp_size) return fail(PCP_ERR_INVALID_ARGUMENT, "rank %d outside [0, %d)", rank, d.pcp_size);
  if (num_sources < 0 || num_sources > pcp::kMaxSources)
    return fail(PCP_ERR_INVALID_ARGUMENT, "num_sources %d outside [0, %d]", num_sources, pcp::kMaxSources);
  Part part;
  PCP_TRY(packed_part(d, packed_kv, num_sources, valid_len, &part, g_kv_path.load()));
  int splits = 0;
  if (part.keys) {
    part.plan = stateless_plan(d, part, max_splits_for(d) - 1);
    splits = part.plan.splits;
  }
  // The current tokens go to the dense workspace after the dense history
  // keys (none when the history is read in place).
  const int64_t cur_off = dense_keys(part.keys, part.in_place);
  const Workspace w = ws_layout(d, cur_off + current_keys(d), splits + 1);
  if (workspace_bytes < w.total)
    return fail(PCP_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is below the %zu required", workspace_bytes, w.total);
  auto* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool direct = splits == 0;
  CUDA_TRY(cudaMemsetAsync(ws, 0, 4, st));
  if (part.keys) {
    if (part.in_place) {
      PCP_TRY(launch_attention_kv(d, q, part, ws, w, 0, false, out, st, nullptr));
    } else {
      PCP_TRY(launch_unpack(d, part.srcs, w, ws, st, nullptr));
      PCP_TRY(launch_attention(d, q, w, ws, 0, part.keys, part.plan, 0, false, out, st, nullptr));
    }
  }
  PCP_TRY(launch_scatter(d, k_cur_all, v_cur_all, interleave_size, w, ws, cur_off, st, nullptr));
  PCP_TRY(launch_attention(d, q, w, ws, cur_off, current_keys(d), causal_plan(d), splits, direct, out, st, nullptr,
                           Causal{rank, interleave_size}));
  if (!direct) PCP_TRY(launch_combine(d, w, ws, splits + 1, out, st, nullptr));
  return PCP_OK;
}

int pcp_history_attention_paged(const pcp_dims_t* dims, const void* q, const void* cache_pool, int64_t pool_blocks,
                                const int32_t* block_tables, int32_t num_sources, const int32_t* valid_len, void* out,
                                void* workspace, size_t workspace_bytes, void* stream) {
  PCP_TRY(check_dims(dims));
  const pcp_dims_t& d = *dims;
  if (!q || !cache_pool || !block_tables || !valid_len || !out || !workspace)
    return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  if (pool_blocks <= 0) return fail(PCP_ERR_INVALID_ARGUMENT, "empty block pool");
  if (num_sources <= 0 || num_sources > pcp::kMaxSources)
    return fail(PCP_ERR_INVALID_ARGUMENT, "num_sources %d outside [1, %d]", num_sources, pcp::kMaxSources);
  const int64_t cap = static_cast<int64_t>(d.max_local_blocks) * d.block_size;
  Part part;
  part.in_place = choose_in_place(d, g_kv_path.load());
  part.map_base = cache_pool;
  part.map_blocks = pool_blocks;
  for (int s = 0; s < num_sources; ++s) {
    if (valid_len[s] < 0 || valid_len[s] > cap)
      return fail(PCP_ERR_INVALID_ARGUMENT, "valid_len[%d]=%d outside [0, %lld]", s, valid_len[s],
                  static_cast<long long>(cap));
    add_source(d, &part, static_cast<const uint8_t*>(cache_pool),
               block_tables + static_cast<size_t>(s) * d.max_local_blocks, pool_blocks, valid_len[s], -1, false);
  }
  if (part.keys == 0) return fail(PCP_ERR_INVALID_ARGUMENT, "no valid history tokens");
  part.plan = stateless_plan(d, part, max_splits_for(d));
  const Workspace w = ws_layout(d, dense_keys(part.keys, part.in_place), part.plan.splits);
  if (workspace_bytes < w.total)
    return fail(PCP_ERR_INVALID_ARGUMENT, "workspace of %zu bytes is below the %zu required", workspace_bytes, w.total);
  auto* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemsetAsync(ws, 0, 4, st));
  return run_single_part(d, q, part, w, ws, out, st);
}

int pcp_cache_write(const pcp_dims_t* dims, int32_t interleave_size, int32_t rank, int64_t first_position,
                    int32_t num_tokens, const void* k_src, const void* v_src, const int32_t* block_table,
                    int32_t table_len, void* cache_pool, int64_t pool_blocks, int32_t* device_status, void* stream) {
  PCP_TRY(check_dims(dims));
  const pcp_dims_t& d = *dims;
  if ((num_tokens > 0 && (!k_src || !v_src)) || !block_table || !cache_pool || !device_status)
    return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  if (interleave_size <= 0 || d.block_size % interleave_size)
    return fail(PCP_ERR_INVALID_ARGUMENT, "interleave_size %d must be positive and divide block_size %d",
                interleave_size, d.block_size);
  if (rank < 0 || rank >= d.pcp_size) return fail(PCP_ERR_INVALID_ARGUMENT, "rank %d outside [0, %d)", rank, d.pcp_size);
  if (first_position < 0 || num_tokens < 0 || table_len < 0 || pool_blocks <= 0)
    return fail(PCP_ERR_INVALID_ARGUMENT, "negative position / token count / table length or empty pool");
  if (reinterpret_cast<uintptr_t>(k_src) % 16 || reinterpret_cast<uintptr_t>(v_src) % 16 ||
      reinterpret_cast<uintptr_t>(cache_pool) % 16)
    return fail(PCP_ERR_INVALID_ARGUMENT, "K/V sources and the pool must be 16-byte aligned");
  // Slots this rank owns below position x: whole stripes of P*I, plus the
  // part of the last one that reaches into this rank's I positions.
  const int64_t stride = static_cast<int64_t>(d.pcp_size) * interleave_size;
  auto owned_below = [&](int64_t x) {
    return (x / stride) * interleave_size +
           std::min<int64_t>(std::max<int64_t>(x % stride - static_cast<int64_t>(rank) * interleave_size, 0),
                             interleave_size);
  };
  const int64_t local0 = owned_below(first_position);
  const int64_t owned = owned_below(first_position + num_tokens) - local0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemsetAsync(device_status, 0, sizeof(int32_t), st));
  if (owned == 0) return PCP_OK;
  if (ceil_div(local0 + owned, d.block_size) > table_len)
    return fail(PCP_ERR_INVALID_ARGUMENT, "block table of %d entries is too short for local slot %lld", table_len,
                static_cast<long long>(local0 + owned - 1));
  pcp::CacheWriteParams p{};
  p.k_src = static_cast<const __nv_bfloat16*>(k_src);
  p.v_src = static_cast<const __nv_bfloat16*>(v_src);
  p.num_tokens = num_tokens;
  p.first = first_position;
  p.local0 = local0;
  p.owned = static_cast<int>(owned);
  p.ranks = d.pcp_size;
  p.width = interleave_size;
  p.rank = rank;
  p.num_kv_heads = d.num_kv_heads;
  p.block_size = d.block_size;
  p.head_dim = d.head_dim;
  p.kv_is_bf16 = d.kv_dtype == PCP_KV_BF16;
  p.table = block_table;
  p.table_len = table_len;
  p.pool_blocks = pool_blocks;
  p.pool = static_cast<uint8_t*>(cache_pool);
  p.err = device_status;
  const int64_t items = 2 * owned * d.num_kv_heads * (d.head_dim / 8);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, 256), 4 * 148));
  pcp::cache_write_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
  CUDA_TRY(cudaGetLastError());
  return PCP_OK;
}

int pcp_history_attention_status(const void* workspace, void* stream) {
  if (!workspace) return fail(PCP_ERR_INVALID_ARGUMENT, "workspace is NULL");
  int err = 0;
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  CUDA_TRY(cudaMemcpy(&err, workspace, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return fail(PCP_ERR_DEVICE_TIMEOUT, "device wait timed out in the attention kernel (code %d)", err);
  return PCP_OK;
}

}  // extern "C"

// ----------------------------------------------- allocation-free entry ----
// Fixed scratch of pcp_history_attention_noalloc: error word, dense bf16 K/V
// and split partials, laid out exactly as a pcp_history_attention workspace.
// A static device array, so it exists on every device that loads this
// library, for the life of the process.
static __device__ __align__(256) uint8_t g_noalloc_scratch[PCP_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (with that device current).  In host code the symbol is only a
// host-side stand-in, never a device address, so kernels get this pointer.
int noalloc_scratch(void** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(PCP_ERR_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(PCP_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return PCP_OK;
}

}  // namespace

extern "C" {

int pcp_history_attention_noalloc(const pcp_dims_t* dims, const void* q, const void* packed_kv, int32_t num_sources,
                                  const int32_t* valid_len, void* out, int32_t* device_status, void* stream) {
  PCP_TRY(check_dims(dims));
  const pcp_dims_t& d = *dims;
  if (!q || !packed_kv || !valid_len || !out || !device_status)
    return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  if (num_sources <= 0 || num_sources > pcp::kMaxSources)
    return fail(PCP_ERR_INVALID_ARGUMENT, "num_sources %d outside [1, %d]", num_sources, pcp::kMaxSources);
  // The largest split plan whose workspace fits the fixed scratch (a cap
  // that starves stream-K of pairs falls back to the static schedule inside
  // plan_splits).  When the dense path chosen by default does not fit, an
  // e4m3 cache is read in place instead (no dense copy in the scratch).
  const int sms = num_sms();
  Part part;
  Workspace w;
  auto fit = [&](int mode) -> int {
    part = Part{};
    PCP_TRY(packed_part(d, packed_kv, num_sources, valid_len, &part, mode));
    if (part.keys == 0) return fail(PCP_ERR_INVALID_ARGUMENT, "no valid history tokens");
    int split_cap = max_splits_for(d);
    while (true) {
      part.plan = plan_splits(d, part_tiles(part), part.keys, sms, split_cap, true, part.in_place);
      w = ws_layout(d, dense_keys(part.keys, part.in_place), part.plan.splits);
      if (w.total <= PCP_NOALLOC_SCRATCH_BYTES) return PCP_OK;
      if (part.plan.splits == 1)
        return fail(PCP_ERR_UNSUPPORTED,
                    "problem needs %zu scratch bytes; the allocation-free entry has %u (use pcp_history_attention "
                    "with a caller workspace)",
                    w.total, PCP_NOALLOC_SCRATCH_BYTES);
      split_cap = part.plan.splits - 1;
    }
  };
  const int mode = g_kv_path.load();
  int rc = fit(mode);
  if (rc == PCP_ERR_UNSUPPORTED && !part.in_place && mode != PCP_KV_PATH_DENSE && kv_in_place_ok(d))
    rc = fit(PCP_KV_PATH_IN_PLACE);
  PCP_TRY(rc);
  void* scratch = nullptr;
  PCP_TRY(noalloc_scratch(&scratch));
  auto* ws = static_cast<uint8_t*>(scratch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The error word is the only scratch state that must start at zero: dense
  // K/V rows past num_keys are never read (TMA zero-fills past the tensor
  // map's extent) and every partial the combine reads is rewritten.
  CUDA_TRY(cudaMemsetAsync(ws, 0, 4, st));
  PCP_TRY(run_single_part(d, q, part, w, ws, out, st));
  CUDA_TRY(cudaMemcpyAsync(device_status, ws, sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  return PCP_OK;
}

int pcp_create(const pcp_dims_t* dims, int32_t rank, int32_t device, const void* nccl_unique_id,
               pcp_handle_t** out) {
  PCP_TRY(check_dims(dims));
  if (!out) return fail(PCP_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  const pcp_dims_t& d = *dims;
  if (rank < 0 || rank >= d.pcp_size) return fail(PCP_ERR_INVALID_ARGUMENT, "rank %d outside [0, %d)", rank, d.pcp_size);
  if (d.pcp_size > 1 && !nccl_unique_id) return fail(PCP_ERR_INVALID_ARGUMENT, "pcp_size > 1 needs an NCCL unique id");
  CUDA_TRY(cudaSetDevice(device));
  auto* h = new pcp_handle();
  h->d = d;
  h->rank = rank;
  h->device = device;
  h->sms = num_sms();
  auto cleanup = [&](int code) {
    pcp_destroy(h);
    return code;
  };
  // Dense keys: every source's history plus the current tokens of a prefill.
  // Dense keys for every source (the handle may read either way; see
  // pcp_set_kv_path) plus the current tokens of a prefill.
  const int64_t key_cap = static_cast<int64_t>(d.pcp_size) * d.max_local_blocks * d.block_size + current_keys(d);
  h->w = ws_layout(d, key_cap, max_splits_for(d));
  if (cudaMalloc(&h->ws, h->w.total) != cudaSuccess)
    return cleanup(fail(PCP_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu workspace bytes failed", h->w.total));
  if (cudaMemset(h->ws, 0, h->w.k_off) != cudaSuccess) return cleanup(fail(PCP_ERR_CUDA, "cudaMemset failed"));
  if (d.pcp_size > 1) {
    const size_t ring_bytes = static_cast<size_t>(d.pcp_size) * d.max_local_blocks * payload_bytes(d);
    if (cudaMalloc(&h->ring, ring_bytes) != cudaSuccess)
      return cleanup(fail(PCP_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu ring bytes failed", ring_bytes));
    const size_t stage_bytes = static_cast<size_t>(d.max_local_blocks) * payload_bytes(d);
    if (cudaMalloc(&h->stage, stage_bytes) != cudaSuccess)
      return cleanup(fail(PCP_ERR_OUT_OF_MEMORY, "cudaMalloc of %zu staging bytes failed", stage_bytes));
    const size_t cur_bytes = static_cast<size_t>(current_keys(d)) * d.num_kv_heads * d.head_dim * 2;
    if (cudaMalloc(&h->cur_k, cur_bytes) != cudaSuccess || cudaMalloc(&h->cur_v, cur_bytes) != cudaSuccess)
      return cleanup(fail(PCP_ERR_OUT_OF_MEMORY, "cudaMalloc of 2 x %zu current-token bytes failed", cur_bytes));
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if (cudaStreamCreateWithPriority(&h->comm_stream, cudaStreamNonBlocking, hi) != cudaSuccess)
      return cleanup(fail(PCP_ERR_CUDA, "stream creation failed"));
    if (cudaEventCreateWithFlags(&h->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h->ev_comm, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h->ev_group[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h->ev_group[1], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&h->ev_cur, cudaEventDisableTiming) != cudaSuccess)
      return cleanup(fail(PCP_ERR_CUDA, "event creation failed"));
    h->ev_step.assign(std::min(d.pcp_size - 1, kMaxParts - 1), nullptr);
    for (auto& e : h->ev_step)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return cleanup(fail(PCP_ERR_CUDA, "event creation failed"));
    ncclUniqueId id;
    std::memcpy(&id, nccl_unique_id, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&h->comm, d.pcp_size, id, rank, &cfg);
    const int s = wait_nccl(h->comm, r, 600000);
    if (s != PCP_OK) {
      h->comm_failed = true;
      return cleanup(s);
    }
  }
  *out = h;
  return PCP_OK;
}

int pcp_forward(pcp_handle_t* h, const void* q, const void* packed_kv, const int32_t* valid_len, void* out,
                void* stream) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (h->comm_failed) return fail(PCP_ERR_PEER, "the ring communicator was aborted");
  LocalKV local;
  local.base = packed_kv;
  return forward_impl(h, q, local, valid_len, nullptr, nullptr, 0, out, static_cast<cudaStream_t>(stream));
}

int pcp_forward_bucketed(pcp_handle_t* h, const void* q, const void* packed_kv, const int32_t* valid_len_dev,
                         const int32_t* bucket_len, void* out, void* stream) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (h->comm_failed) return fail(PCP_ERR_PEER, "the ring communicator was aborted");
  if (!valid_len_dev || !bucket_len) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL valid_len_dev or bucket_len");
  LocalKV local;
  local.base = packed_kv;
  return forward_impl(h, q, local, bucket_len, nullptr, nullptr, 0, out, static_cast<cudaStream_t>(stream),
                      valid_len_dev);
}

int pcp_forward_paged(pcp_handle_t* h, const void* q, const void* cache_pool, int64_t pool_blocks,
                      const int32_t* block_table, const int32_t* valid_len, void* out, void* stream) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (h->comm_failed) return fail(PCP_ERR_PEER, "the ring communicator was aborted");
  if (!block_table) return fail(PCP_ERR_INVALID_ARGUMENT, "block_table is NULL");
  LocalKV local;
  local.base = cache_pool;
  local.table = block_table;
  local.pool_blocks = pool_blocks;
  return forward_impl(h, q, local, valid_len, nullptr, nullptr, 0, out, static_cast<cudaStream_t>(stream));
}

int pcp_forward_prefill(pcp_handle_t* h, int32_t interleave_size, const void* q, const void* packed_kv,
                        const int32_t* valid_len, const void* k_cur, const void* v_cur, void* out, void* stream) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (h->comm_failed) return fail(PCP_ERR_PEER, "the ring communicator was aborted");
  if (!k_cur || !v_cur) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL current K/V");
  LocalKV local;
  local.base = packed_kv;
  return forward_impl(h, q, local, valid_len, k_cur, v_cur, interleave_size, out, static_cast<cudaStream_t>(stream));
}

int pcp_forward_host_async(pcp_handle_t* h, const void* q_host, const void* packed_kv_host,
                           const int32_t* valid_len, void* out_host, void* stream) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (!q_host || !packed_kv_host || !valid_len || !out_host) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL buffer");
  const pcp_dims_t& d = h->d;
  const int r = h->rank;
  if (valid_len[r] < 0 || valid_len[r] > static_cast<int64_t>(d.max_local_blocks) * d.block_size)
    return fail(PCP_ERR_INVALID_ARGUMENT, "valid_len[%d] out of range", r);
  CUDA_TRY(cudaSetDevice(h->device));
  const size_t qbytes = static_cast<size_t>(d.num_q_heads) * d.local_q_len * d.head_dim * 2;
  const size_t kvbytes = static_cast<size_t>(d.max_local_blocks) * payload_bytes(d);
  if (!h->h2d_stream) {
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    CUDA_TRY(cudaStreamCreateWithPriority(&h->h2d_stream, cudaStreamNonBlocking, hi));
    CUDA_TRY(cudaStreamCreateWithPriority(&h->d2h_stream, cudaStreamNonBlocking, hi));
    for (auto& sl : h->slots) {
      CUDA_TRY(cudaMalloc(&sl.q, qbytes));
      CUDA_TRY(cudaMalloc(&sl.kv, kvbytes));
      CUDA_TRY(cudaMalloc(&sl.out, qbytes));
      CUDA_TRY(cudaEventCreateWithFlags(&sl.loaded, cudaEventDisableTiming));
      CUDA_TRY(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming));
      CUDA_TRY(cudaEventCreateWithFlags(&sl.fetched, cudaEventDisableTiming));
    }
  }
  auto& sl = h->slots[h->next_slot];
  const size_t live = static_cast<size_t>(ceil_div(valid_len[r], d.block_size)) * payload_bytes(d);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The slot's previous call must have finished its forward (which read q and
  // sent kv) before new inputs land, and its output copy before the forward
  // writes out again.
  if (sl.used) CUDA_TRY(cudaStreamWaitEvent(h->h2d_stream, sl.done, 0));
  CUDA_TRY(cudaMemcpyAsync(sl.q, q_host, qbytes, cudaMemcpyHostToDevice, h->h2d_stream));
  if (live) CUDA_TRY(cudaMemcpyAsync(sl.kv, packed_kv_host, live, cudaMemcpyHostToDevice, h->h2d_stream));
  CUDA_TRY(cudaEventRecord(sl.loaded, h->h2d_stream));
  CUDA_TRY(cudaStreamWaitEvent(st, sl.loaded, 0));
  if (sl.used) CUDA_TRY(cudaStreamWaitEvent(st, sl.fetched, 0));
  PCP_TRY(pcp_forward(h, sl.q, sl.kv, valid_len, sl.out, stream));
  CUDA_TRY(cudaEventRecord(sl.done, st));
  CUDA_TRY(cudaStreamWaitEvent(h->d2h_stream, sl.done, 0));
  CUDA_TRY(cudaMemcpyAsync(out_host, sl.out, qbytes, cudaMemcpyDeviceToHost, h->d2h_stream));
  CUDA_TRY(cudaEventRecord(sl.fetched, h->d2h_stream));
  sl.used = true;
  h->next_slot ^= 1;
  return PCP_OK;
}

int pcp_forward_host_wait(pcp_handle_t* h) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  CUDA_TRY(cudaSetDevice(h->device));
  if (h->h2d_stream) {
    CUDA_TRY(cudaStreamSynchronize(h->h2d_stream));
    CUDA_TRY(cudaStreamSynchronize(h->d2h_stream));
  }
  return PCP_OK;
}

int pcp_forward_host(pcp_handle_t* h, const void* q_host, const void* packed_kv_host, const int32_t* valid_len,
                     void* out_host, void* stream) {
  PCP_TRY(pcp_forward_host_async(h, q_host, packed_kv_host, valid_len, out_host, stream));
  PCP_TRY(pcp_forward_host_wait(h));
  CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  return PCP_OK;
}

int pcp_device_status(pcp_handle_t* h, int32_t timeout_ms) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  CUDA_TRY(cudaSetDevice(h->device));
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t a = cudaStreamQuery(h->last_stream);
    cudaError_t b = h->comm_stream ? cudaStreamQuery(h->comm_stream) : cudaSuccess;
    if (a != cudaSuccess && a != cudaErrorNotReady) return fail(PCP_ERR_CUDA, "stream: %s", cudaGetErrorString(a));
    if (b != cudaSuccess && b != cudaErrorNotReady) return fail(PCP_ERR_CUDA, "comm stream: %s", cudaGetErrorString(b));
    if (h->comm) {
      ncclResult_t st = ncclSuccess;
      ncclCommGetAsyncError(h->comm, &st);
      if (st != ncclSuccess && st != ncclInProgress) {
        ncclCommAbort(h->comm);
        h->comm = nullptr;
        h->comm_failed = true;
        return fail(PCP_ERR_PEER, "NCCL async error: %s", ncclGetErrorString(st));
      }
    }
    if (a == cudaSuccess && b == cudaSuccess) break;
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      if (h->comm) {
        ncclCommAbort(h->comm);
        h->comm = nullptr;
        h->comm_failed = true;
      }
      return fail(PCP_ERR_DEVICE_TIMEOUT, "forward not complete after %d ms; ring aborted", timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  int err = 0;
  CUDA_TRY(cudaMemcpy(&err, h->ws, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return fail(PCP_ERR_DEVICE_TIMEOUT, "device wait timed out in the attention kernel (code %d)", err);
  return PCP_OK;
}

int pcp_set_exchange(pcp_handle_t* h, int32_t mode) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (mode != PCP_EXCHANGE_DIRECT && mode != PCP_EXCHANGE_RING && mode != PCP_EXCHANGE_ALLGATHER &&
      mode != PCP_EXCHANGE_PIPELINE)
    return fail(PCP_ERR_INVALID_ARGUMENT, "exchange mode %d unknown", mode);
  h->exchange = mode;
  return PCP_OK;
}

int pcp_stream_k_plan(int64_t units, int64_t key_tiles, int32_t sms, int32_t slot_cap, int32_t* pairs,
                      int32_t* slots) {
  if (units <= 0 || key_tiles < 0 || sms <= 0 || slot_cap <= 0 || !pairs || !slots)
    return fail(PCP_ERR_INVALID_ARGUMENT, "bad arguments");
  const SplitPlan pl = plan_stream_k(units, key_tiles, sms, slot_cap);
  *pairs = pl.pairs;
  *slots = pl.splits;
  return PCP_OK;
}

int pcp_stream_k_segments(int32_t units, int32_t key_tiles, int32_t grid_pairs, int32_t pair, int32_t* segments,
                          int32_t max_segments, int32_t* count) {
  if (units <= 0 || key_tiles < 0 || grid_pairs <= 0 || pair < 0 || pair >= grid_pairs || !count ||
      (max_segments > 0 && !segments))
    return fail(PCP_ERR_INVALID_ARGUMENT, "bad arguments");
  pcp::Schedule sc;
  sc.init_stream_k(key_tiles, units, grid_pairs, pair);
  pcp::Segment sg;
  int n = 0;
  while (sc.next(sg)) {
    if (n < max_segments) {
      int32_t* o = segments + 6 * n;
      o[0] = sg.unit;
      o[1] = sg.kt0;
      o[2] = sg.kt1;
      o[3] = sg.slot;
      o[4] = sg.nseg;
      o[5] = sg.last ? 1 : 0;
    }
    ++n;
  }
  *count = n;
  return n > max_segments ? fail(PCP_ERR_INVALID_ARGUMENT, "%d segments, room for %d", n, max_segments) : PCP_OK;
}

int pcp_set_kv_path(pcp_handle_t* h, int32_t mode) {
  if (mode != PCP_KV_PATH_AUTO && mode != PCP_KV_PATH_DENSE && mode != PCP_KV_PATH_IN_PLACE)
    return fail(PCP_ERR_INVALID_ARGUMENT, "kv path %d unknown", mode);
  if (h)
    h->kv_path = mode;
  else
    g_kv_path.store(mode);
  return PCP_OK;
}

int pcp_set_comm_sms(pcp_handle_t* h, int32_t sms) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (sms < 0 || sms >= h->sms) return fail(PCP_ERR_INVALID_ARGUMENT, "comm_sms %d outside [0, %d)", sms, h->sms);
  h->comm_sms = sms & ~1;  // whole SM pairs
  return PCP_OK;
}

int pcp_set_profiling(pcp_handle_t* h, int32_t enable) {
  if (!h) return fail(PCP_ERR_INVALID_ARGUMENT, "handle is NULL");
  if (enable) {
    // Events still referenced by recorded spans must be complete before reuse.
    CUDA_TRY(cudaSetDevice(h->device));
    for (auto& sp : h->spans) cudaEventSynchronize(sp.end);
    h->spans.clear();
    h->ev_used = 0;
    h->accum = pcp_stats_t{};
  }
  h->profiling = enable != 0;
  return PCP_OK;
}

int pcp_get_stats(const pcp_handle_t* hc, pcp_stats_t* out) {
  if (!hc || !out) return fail(PCP_ERR_INVALID_ARGUMENT, "NULL argument");
  auto* h = const_cast<pcp_handle_t*>(hc);
  if (!h->profiling) {
    *out = h->last;
    return PCP_OK;
  }
  CUDA_TRY(cudaSetDevice(h->device));
  pcp_stats_t s = h->accum;
  double ms[4] = {0, 0, 0, 0};
  for (const auto& sp : h->spans) {
    float t = 0.f;
    CUDA_TRY(cudaEventSynchronize(sp.end));
    CUDA_TRY(cudaEventElapsedTime(&t, sp.start, sp.end));
    ms[sp.slot] += t;
  }
  s.comm_ms = ms[0];
  s.unpack_ms = ms[1];
  s.attn_ms = ms[2];
  s.combine_ms = ms[3];
  *out = s;
  return PCP_OK;
}

int pcp_destroy(pcp_handle_t* h) {
  if (!h) return PCP_OK;
  cudaSetDevice(h->device);
  if (h->comm) {
    if (h->comm_failed) {
      ncclCommAbort(h->comm);
    } else {
      ncclResult_t r = ncclCommFinalize(h->comm);
      wait_nccl(h->comm, r, 60000);
      ncclCommDestroy(h->comm);
    }
    h->comm = nullptr;
  }
  if (h->comm_stream) cudaStreamSynchronize(h->comm_stream);
  for (auto& sp : h->spans) cudaEventSynchronize(sp.end);
  for (auto& e : h->ev_pool)
    if (e) cudaEventDestroy(e);
  if (h->ev_in) cudaEventDestroy(h->ev_in);
  if (h->ev_comm) cudaEventDestroy(h->ev_comm);
  for (auto& e : h->ev_group)
    if (e) cudaEventDestroy(e);
  for (auto& e : h->ev_step)
    if (e) cudaEventDestroy(e);
  if (h->ev_cur) cudaEventDestroy(h->ev_cur);
  if (h->comm_stream) cudaStreamDestroy(h->comm_stream);
  cudaFree(h->ring);
  cudaFree(h->stage);
  cudaFree(h->cur_k);
  cudaFree(h->cur_v);
  cudaFree(h->ws);
  if (h->h2d_stream) {
    cudaStreamSynchronize(h->h2d_stream);
    cudaStreamSynchronize(h->d2h_stream);
  }
  for (auto& sl : h->slots) {
    cudaFree(sl.q);
    cudaFree(sl.kv);
    cudaFree(sl.out);
    if (sl.loaded) cudaEventDestroy(sl.loaded);
    if (sl.done) cudaEventDestroy(sl.done);
    if (sl.fetched) cudaEventDestroy(sl.fetched);
  }
  if (h->h2d_stream) cudaStreamDestroy(h->h2d_stream);
  if (h->d2h_stream) cudaStreamDestroy(h->d2h_stream);
  delete h;
  return PCP_OK;
}

int pcp_selftest_bounded_wait(int32_t limit_us, int32_t* device_status) {
  if (!device_status || limit_us <= 0) return fail(PCP_ERR_INVALID_ARGUMENT, "bad arguments");
  int* err = nullptr;
  CUDA_TRY(cudaMalloc(&err, sizeof(int)));
  cudaMemset(err, 0, sizeof(int));
  bounded_wait_probe_kernel<<<1, 32>>>(err, static_cast<unsigned long long>(limit_us) * 1000ull);
  cudaError_t e = cudaDeviceSynchronize();
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(err);
  if (e != cudaSuccess) return fail(PCP_ERR_CUDA, "probe: %s", cudaGetErrorString(e));
  *device_status = v;
  return PCP_OK;
}

}  // extern "C"
