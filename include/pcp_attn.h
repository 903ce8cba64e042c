/*
 * C ABI of the B200 prefill context-parallel (PCP) history-attention path.
 *
 * Replaces the reference's device path (HandsomeHow/aws_training_study):
 *   pcp_attention/kernel.py:559-564   wrap_for_native_torch(cfg) -> kernel(q, packed_kv, mask)
 *   pcp_attention/kernel.py:32-556    make_history_attention_kernel(cfg) (the NKI kernel,
 *                                     with its ring collective_permute at kernel.py:276-293)
 *   run_poc.py:200-212                root communicator id exchange
 *   run_poc.py:241-257                host->device copies, compiled call, .cpu()
 *
 * Conventions
 *   - Plain pointers and sizes only; the caller owns every buffer it passes.
 *   - Device pointers are CUDA device memory of the current device; `stream` is a
 *     cudaStream_t (NULL = legacy default stream).  Calls are asynchronous on the
 *     stream unless stated otherwise.
 *   - Every function returns PCP_OK (0) or a pcp_status code; pcp_last_error()
 *     gives a message for the calling thread's last failure.
 *   - Layouts (row-major, innermost last):
 *       q, out      [num_q_heads][local_q_len][head_dim]                  bf16
 *       packed_kv   [blocks][2][num_kv_heads][block_size][head_dim]        e4m3fn or bf16
 *                   (the reference's pack_local_kv ring payload, kernel.py:17-29)
 *       valid_len   int32 per source rank, host memory: valid history tokens in
 *                   that rank's shard (its first valid_len tokens; the rest of the
 *                   blocks is padding and never read).
 */
#ifndef PCP_ATTN_H
#define PCP_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PCP_ATTN_ABI_VERSION 2

enum pcp_kv_dtype {
  PCP_KV_E4M3 = 0, /* float8_e4m3fn, dequantised at unit scale (reference.py:29-31) */
  PCP_KV_BF16 = 1
};

enum pcp_status {
  PCP_OK = 0,
  PCP_ERR_INVALID_ARGUMENT = 1,
  PCP_ERR_UNSUPPORTED = 2,
  PCP_ERR_CUDA = 3,
  PCP_ERR_NCCL = 4,
  PCP_ERR_DEVICE_TIMEOUT = 5,
  PCP_ERR_OUT_OF_MEMORY = 6,
  PCP_ERR_PEER = 7
};

/* Static shape of one PCP rank (the fields of PCPAttentionConfig that fix
 * buffer shapes, pcp_attention/config.py:17-59). */
typedef struct pcp_dims {
  int32_t pcp_size;         /* P: ranks in the ring */
  int32_t local_q_len;      /* current_len / P */
  int32_t max_local_blocks; /* cache blocks per rank in packed_kv */
  int32_t block_size;       /* tokens per cache block */
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;         /* 128 or 256 on the CUDA path */
  int32_t kv_dtype;         /* enum pcp_kv_dtype */
} pcp_dims_t;

/* Measurements accumulated over every pcp_forward since the last
 * pcp_set_profiling(h, 1) (device times, from CUDA events recorded on the
 * stream each kernel is launched on).  With profiling off, the counts and
 * sizes describe the last forward and the times are 0. */
typedef struct pcp_stats {
  double attn_ms;          /* summed duration of the attention kernel launches */
  double unpack_ms;        /* summed duration of the KV unpack launches */
  double combine_ms;       /* summed duration of the split combine launches */
  double comm_ms;          /* summed ring exchange time on the comm stream */
  int32_t kernel_launches; /* kernels of this library launched */
  int32_t attn_launches;   /* of which attention kernels */
  int32_t splits;          /* key splits of the last forward (1 = direct bf16 output) */
  int32_t forwards;        /* forwards accumulated */
  int64_t ring_bytes;      /* bytes this rank sent around the ring */
  int64_t keys;            /* valid history keys attended by the last forward */
  int32_t kv_in_place;     /* 1: the last forward read the cache in place (pcp_set_kv_path) */
  int32_t reserved;
} pcp_stats_t;

typedef struct pcp_handle pcp_handle_t;

/* Message for the calling thread's last failing call ("" if none). */
const char* pcp_last_error(void);
int pcp_abi_version(void);

/* ---- host-only helpers (no GPU needed) --------------------------------- */

/* Valid history tokens owned by `rank` for a global history of `total_len`
 * under the striped map of pcp_attention/layout.py:10-16.  Equals the
 * reference's actual_local_history_len (config.py:45-47) when total_len is a
 * multiple of pcp_size * interleave_size. */
int64_t pcp_source_valid_len(int64_t total_len, int32_t pcp_size, int32_t interleave_size, int32_t rank);

/* Ring schedule of hop `hop` (1..P-1) for `rank`: the source rank whose shard
 * this rank sends to rank+1 and the source rank whose shard it receives from
 * rank-1 (reference.py:68-71 "source_rank = (rank - step) % P", kernel.py:276-293
 * receive-from-predecessor permute; the final hop back to the owner is omitted). */
int pcp_ring_schedule(int32_t rank, int32_t pcp_size, int32_t hop, int32_t* send_source, int32_t* recv_source,
                      int32_t* send_to, int32_t* recv_from);

/* Bytes of an NCCL unique id, and a fresh one (rank 0 creates, all ranks
 * receive it out of band; replaces run_poc.py:200-212). */
int pcp_nccl_unique_id_bytes(void);
int pcp_get_nccl_unique_id(void* out);

/* Host-side view of the stream-K schedule of a history launch (the same
 * arithmetic the kernel runs), for tests and tools.  pcp_stream_k_plan: the
 * CTA pairs and partial slots per unit the planner picks for `units`
 * 256-row units x `key_tiles` 128-key tiles on `sms` SMs within `slot_cap`
 * slots.  pcp_stream_k_segments: the segments pair `pair` of a
 * `grid_pairs` grid walks, 6 int32 each (unit, first tile, end tile, slot,
 * segments of the unit, ends the unit); *count gets the number. */
int pcp_stream_k_plan(int64_t units, int64_t key_tiles, int32_t sms, int32_t slot_cap, int32_t* pairs,
                      int32_t* slots);
int pcp_stream_k_segments(int32_t units, int32_t key_tiles, int32_t grid_pairs, int32_t pair, int32_t* segments,
                          int32_t max_segments, int32_t* count);

/* ---- stateless single-GPU entry ---------------------------------------- */

/* Device workspace bytes needed by pcp_history_attention for `total_valid`
 * history keys on the current device. */
int pcp_history_attention_workspace_size(const pcp_dims_t* dims, int64_t total_valid, size_t* bytes);

/* History attention of one rank whose history is fully resident: the
 * packed shards of `num_sources` ranks laid out back to back
 * ([num_sources][max_local_blocks][payload]) with valid_len[num_sources].
 * For P == 1 this is the whole path (replaces kernel(q, packed_kv, mask) of
 * kernel.py:559-564 with pcp_size 1).  `workspace` is caller-owned device
 * memory of pcp_history_attention_workspace_size bytes. */
int pcp_history_attention(const pcp_dims_t* dims, const void* q, const void* packed_kv, int32_t num_sources,
                          const int32_t* valid_len, void* out, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Synchronises `stream` and reports a device-side wait timeout recorded in
 * `workspace` by the last pcp_history_attention on it (PCP_ERR_DEVICE_TIMEOUT). */
int pcp_history_attention_status(const void* workspace, void* stream);

/* ---- paged KV cache: producer and block-table consumer ------------------ */

/* The paged-cache producer (no device counterpart in the reference, which
 * builds its caches on the host with shard_history + pack_local_kv,
 * layout.py:54-98 and kernel.py:17-29, quantising with
 * tensor.to(torch.float8_e4m3fn) in run_poc.py:81-134).  Writes new tokens'
 * K and V into THIS rank's paged cache, quantised to dims->kv_dtype:
 *   - k_src / v_src: [Hkv][num_tokens][D] bf16 in sequence order (device);
 *     token t sits at absolute history position first_position + t.
 *   - Position p belongs to rank (p / I) % P at local slot
 *     (p / (P * I)) * I + p % I; only this rank's tokens are written (every
 *     rank may pass the same sources).  Slot l lives in logical block l / bs,
 *     row l % bs, and logical block b is pool block block_table[b]
 *     (block_table: DEVICE int32[table_len]).
 *   - cache_pool: [pool_blocks][2 * Hkv * bs * D] in the packed payload
 *     format (per block all K rows of every head, then all V rows).
 *   - e4m3fn: round to nearest even; magnitudes above 464 and NaN/Inf become
 *     NaN (0x7F | sign), as torch's cast does.  bf16 caches are copied.
 *   - device_status: caller-owned DEVICE int32, zeroed here and set to 109 if
 *     a table entry lies outside the pool (that token is skipped).
 *   - interleave_size I must divide block_size. */
int pcp_cache_write(const pcp_dims_t* dims, int32_t interleave_size, int32_t rank, int64_t first_position,
                    int32_t num_tokens, const void* k_src, const void* v_src, const int32_t* block_table,
                    int32_t table_len, void* cache_pool, int64_t pool_blocks, int32_t* device_status, void* stream);

/* pcp_history_attention over paged shards: source s's logical blocks are
 * pool blocks block_tables[s * max_local_blocks + b] (DEVICE int32) of one
 * cache_pool [pool_blocks][payload].  A table entry outside the pool is
 * skipped and reported as code 109 by pcp_history_attention_status.
 * Workspace: pcp_history_attention_workspace_size. */
int pcp_history_attention_paged(const pcp_dims_t* dims, const void* q, const void* cache_pool, int64_t pool_blocks,
                                const int32_t* block_tables, int32_t num_sources, const int32_t* valid_len, void* out,
                                void* workspace, size_t workspace_bytes, void* stream);

/* ---- prefill: history plus causal current-token attention -------------- */

/* The reference leaves current-token attention for later (README.md:17-18):
 * its kernel attends the Q shard to the history only.  These entries add the
 * adjacent step of the same prefill layer: each query also attends, causally,
 * to the current (prefill) tokens of every rank, and the two parts merge
 * through the same (O, log-sum-exp) combine as the history splits.
 *   - Current tokens are striped across ranks exactly like Q (layout.py:34-51,
 *     global position of local token i of rank s is
 *     (i / I) * (P * I) + s * I + i % I); a query at global position g sees
 *     every history key and the current keys at positions <= g.
 *   - k_cur_all / v_cur_all: the current tokens' K and V of ALL ranks,
 *     [pcp_size][Hkv][Qloc][D] bf16, rank s's shard at index s.
 *   - `rank`: which rank's Q shard `q` is.  interleave_size I must divide Qloc.
 *   - Zero history tokens (valid_len all 0, packed_kv may then be NULL) is a
 *     plain causal prefill. */
int pcp_prefill_attention_workspace_size(const pcp_dims_t* dims, int64_t total_valid, size_t* bytes);
int pcp_prefill_attention(const pcp_dims_t* dims, int32_t interleave_size, int32_t rank, const void* q,
                          const void* packed_kv, int32_t num_sources, const int32_t* valid_len, const void* k_cur_all,
                          const void* v_cur_all, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Failure-detection self test: runs one kernel that waits on an mbarrier
 * nothing arrives at, bounded by limit_us of device time, and returns the
 * device error word it recorded (199 when the bound fired) in *device_status.
 * The context stays usable.  Synchronous. */
int pcp_selftest_bounded_wait(int32_t limit_us, int32_t* device_status);

/* ---- allocation-free single-GPU entry ---------------------------------- */

/* No counterpart in the reference: an addition for callers that may not
 * allocate device memory at all -- code running where cudaMalloc is
 * forbidden or unsafe (inside a host framework that owns every byte of
 * device memory, a real-time serving loop that must never hit the allocator,
 * a plugin whose host forbids allocation).  Same computation and arguments as
 * pcp_history_attention, but the scratch (error word, split partials, and
 * for a bf16 cache its dense bf16 copy; an e4m3 cache is read in place) lives
 * in a fixed static device array of
 * PCP_NOALLOC_SCRATCH_BYTES inside this library, which every GPU that loads
 * the library holds until the process exits.  The caller still passes the
 * inputs and the output, plus `device_status`: a caller-owned DEVICE int32
 * that receives the kernel's error word (0, or a wait-timeout code).
 *   - Problems whose scratch does not fit return PCP_ERR_UNSUPPORTED with the
 *     size needed; nothing is launched.
 *   - The call makes no allocation (no cudaMalloc/cudaFree, no library
 *     allocator).  Its first call on a device looks up the array's device
 *     address (cudaGetSymbolAddress) with that device current; make that
 *     first call before any stream capture.
 *   - Every call on a device shares the one array, which keeps the last
 *     call's contents (each call clears what must start at zero).  Calls that
 *     overlap on the GPU (different streams, no ordering between them) race
 *     on it: order them on one stream or serialise them. */
#define PCP_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)
int pcp_history_attention_noalloc(const pcp_dims_t* dims, const void* q, const void* packed_kv, int32_t num_sources,
                                  const int32_t* valid_len, void* out, int32_t* device_status, void* stream);

/* ---- ring entry (one handle per rank) ---------------------------------- */

/* Collective over the P ranks when pcp_size > 1 (every rank calls it with the
 * same dims and unique id).  `device` is the CUDA device of this rank.  For
 * pcp_size == 1, nccl_unique_id may be NULL. */
int pcp_create(const pcp_dims_t* dims, int32_t rank, int32_t device, const void* nccl_unique_id,
               pcp_handle_t** out);

/* One forward of this rank: q and packed_kv are this rank's shard (device),
 * valid_len[P] the valid tokens of every source rank (identical on all ranks),
 * out the bf16 output (device).  The local shard is attended while the other
 * shards travel the ring on an internal high-priority stream; `stream` waits
 * for everything before the call's last kernel writes `out`. */
int pcp_forward(pcp_handle_t* h, const void* q, const void* packed_kv, const int32_t* valid_len, void* out,
                void* stream);

/* Length buckets (README.md:52-54: one artifact per bucket, masked blocks
 * skipped).  pcp_forward whose valid lengths are read ON THE DEVICE from
 * valid_len_dev (DEVICE int32[P]) when the kernels run, while everything the
 * host plans -- NCCL transfer sizes, key regions, split plans, grids -- is
 * sized by bucket_len (HOST int32[P], each source's upper bound).  Recorded
 * into a CUDA graph (stream capture of this call), one graph serves every
 * valid_len <= bucket_len: the caller writes new lengths into valid_len_dev
 * and replays.  Per source: blocks past bucket_len are never sent, unpacked
 * or computed; blocks between valid_len and bucket_len are sent (the bucket's
 * slack) but never unpacked or computed.  A device length above its bound is
 * clamped and reported as code 110 by pcp_device_status.  The total of
 * valid_len_dev must be positive (else the output is unspecified). */
int pcp_forward_bucketed(pcp_handle_t* h, const void* q, const void* packed_kv, const int32_t* valid_len_dev,
                         const int32_t* bucket_len, void* out, void* stream);

/* pcp_forward with this rank's shard in a paged cache: its logical block b is
 * pool block block_table[b] (DEVICE int32[max_local_blocks]) of cache_pool
 * [pool_blocks][payload].  The live blocks are gathered into a contiguous
 * buffer on the ring stream before they are sent; the local part reads the
 * pool directly. */
int pcp_forward_paged(pcp_handle_t* h, const void* q, const void* cache_pool, int64_t pool_blocks,
                      const int32_t* block_table, const int32_t* valid_len, void* out, void* stream);

/* pcp_forward plus causal attention over the current tokens (see
 * pcp_prefill_attention): k_cur / v_cur are THIS rank's current tokens' K and
 * V shard, [Hkv][Qloc][D] bf16 on the device, striped like q.  The shards of
 * all ranks are all-gathered on the ring stream before the history exchange
 * and attended right after the local history shard. */
int pcp_forward_prefill(pcp_handle_t* h, int32_t interleave_size, const void* q, const void* packed_kv,
                        const int32_t* valid_len, const void* k_cur, const void* v_cur, void* out, void* stream);

/* Same as pcp_forward, with HOST buffers (pinned or pageable): copies q and packed_kv in,
 * runs pcp_forward on `stream`, copies out back, and returns when out_host is
 * filled (the end-to-end call of run_poc.py:241-257: host tensors in, .cpu() out). */
int pcp_forward_host(pcp_handle_t* h, const void* q_host, const void* packed_kv_host, const int32_t* valid_len,
                     void* out_host, void* stream);

/* The asynchronous form for a serving loop: enqueues the host->device copies
 * (a copy stream of the handle), pcp_forward on `stream` and the copy of out
 * back (a second copy stream), and returns at once.  The handle alternates
 * two device staging slots, so one call's copies overlap the previous call's
 * forward.  Host buffers should be pinned (pageable ones make the copies
 * synchronous); they must stay valid and unmodified, and out_host must not
 * be read, until pcp_forward_host_wait returns.  Not in the reference, whose
 * driver loop is synchronous (run_poc.py:289-318). */
int pcp_forward_host_async(pcp_handle_t* h, const void* q_host, const void* packed_kv_host,
                           const int32_t* valid_len, void* out_host, void* stream);
/* Waits for every pcp_forward_host_async of the handle (copies included). */
int pcp_forward_host_wait(pcp_handle_t* h);

/* Waits up to timeout_ms for the last forward (compute and ring streams) and
 * reports failures: device-side wait timeouts, CUDA errors, NCCL async errors
 * (a peer that left).  On a timeout the NCCL communicator is aborted. */
int pcp_device_status(pcp_handle_t* h, int32_t timeout_ms);

/* How the shards reach every rank (both send only live blocks and never
 * return a shard to its owner; outputs are identical up to fp rounding):
 *   PCP_EXCHANGE_DIRECT (default) -- one NCCL group per forward: each rank
 *     sends its shard to every peer and receives each peer's shard from its
 *     owner (NVSwitch gives every pair full bandwidth);
 *   PCP_EXCHANGE_RING -- the reference's store-and-forward ring
 *     (kernel.py:276-293): P-1 hops to rank+1, schedule of pcp_ring_schedule;
 *   PCP_EXCHANGE_PIPELINE -- direct sends, one NCCL group per ring step (up
 *     to 7 groups), each step's shard attended as soon as it lands; every
 *     launch but the last leaves pcp_set_comm_sms SMs to the exchange (for
 *     exchanges that take as long as the compute, e.g. bf16 MHA shapes);
 *   PCP_EXCHANGE_ALLGATHER -- one NCCL all-gather of equal slots sized to the
 *     longest live shard (lets NCCL multicast through the switch). */
enum pcp_exchange {
  PCP_EXCHANGE_DIRECT = 0,
  PCP_EXCHANGE_RING = 1,
  PCP_EXCHANGE_ALLGATHER = 2,
  PCP_EXCHANGE_PIPELINE = 3
};
int pcp_set_exchange(pcp_handle_t* h, int32_t mode);

/* SMs left to the direct exchange while the local shard is attended, with
 * pcp_size >= 4 and a local shard whose dense bf16 K/V fits in L2: that
 * launch then runs on a persistent grid of the other SMs and every peer's
 * shard travels in one NCCL group meanwhile (NCCL's kernels need SMs; a
 * launch on all of them would hold them off until it ends).  0 turns it off
 * (the exchange then goes in two groups when the local launch fills the
 * GPU).  Default 16; rounded down to whole SM pairs. */
int pcp_set_comm_sms(pcp_handle_t* h, int32_t sms);

/* How history launches read the KV cache.  No counterpart in the reference
 * (its NKI kernel always loads the fp8 blocks into SBUF and upcasts there,
 * kernel.py:295-339); both paths compute the same attention.
 *   PCP_KV_PATH_DENSE -- the valid tokens are first expanded into a dense
 *     bf16 workspace (one pass per forward), which the attention reads;
 *   PCP_KV_PATH_IN_PLACE -- e4m3 caches with block_size % 64 == 0 are read
 *     straight from their cache blocks (TMA) and upcast to f16 in shared
 *     memory: no extra pass, no dense copy, but each 256-row query unit
 *     converts every key tile again (other caches use the dense path);
 *   PCP_KV_PATH_AUTO (default) -- in place when a KV head has at most 4096
 *     query rows (num_q_heads / num_kv_heads * local_q_len), dense otherwise (the allocation-free entry also reads in
 *     place when the dense copy would not fit its scratch).
 * h == NULL sets the process default, used by the stateless entries and by
 * handles without their own setting.  The stateless entries size their
 * workspace for the path in force when queried: keep the default unchanged
 * between the workspace-size query and the call. */
enum pcp_kv_path {
  PCP_KV_PATH_AUTO = 0,
  PCP_KV_PATH_DENSE = 1,
  PCP_KV_PATH_IN_PLACE = 2
};
int pcp_set_kv_path(pcp_handle_t* h, int32_t mode);

int pcp_set_profiling(pcp_handle_t* h, int32_t enable);
int pcp_get_stats(const pcp_handle_t* h, pcp_stats_t* out);
int pcp_destroy(pcp_handle_t* h);

#ifdef __cplusplus
}
#endif

#endif /* PCP_ATTN_H */
