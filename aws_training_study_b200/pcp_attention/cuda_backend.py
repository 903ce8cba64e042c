"""CUDA backend: one ``HistoryAttention`` object per PCP rank.

It owns the C-ABI handle (workspace, ring receive buffers, NCCL communicator,
high-priority comm stream) and exposes the call the reference makes through
``wrap_for_native_torch`` (``pcp_attention/kernel.py:559-564``):

    out = attn(q, packed_kv, valid_len)

with ``q`` ``[Hq, Qloc, D]`` bf16, ``packed_kv`` ``[max_local_blocks,
2*Hkv*bs*D]`` e4m3fn or bf16 (``pack_local_kv`` format) and ``valid_len`` the
valid history tokens of every source rank.  Output ``[Hq, Qloc, D]`` bf16.
Errors are raised as ``PcpError`` (a ``RuntimeError``); invalid shapes raise
``ValueError`` before any device work, like the reference's build-time checks
(``kernel.py:43-51,111-118``).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _capi
from .config import PCPAttentionConfig

SUPPORTED_HEAD_DIMS = (128, 256)


@dataclass(frozen=True)
class KernelLimits:
    head_dims: tuple = SUPPORTED_HEAD_DIMS
    max_pcp_size: int = 64
    kv_dtypes: tuple = (torch.float8_e4m3fn, torch.bfloat16)


kernel_limits = KernelLimits()


def _kv_code(dtype: torch.dtype) -> int:
    if dtype == torch.float8_e4m3fn:
        return _capi.PCP_KV_E4M3
    if dtype == torch.bfloat16:
        return _capi.PCP_KV_BF16
    raise ValueError(f"KV dtype {dtype} is not supported (float8_e4m3fn or bfloat16)")


def make_dims(config: PCPAttentionConfig, kv_dtype: torch.dtype) -> _capi.PcpDims:
    config.validate()
    if config.head_dim not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim {config.head_dim} unsupported by the CUDA kernel {SUPPORTED_HEAD_DIMS}")
    if config.pcp_size > kernel_limits.max_pcp_size:
        raise ValueError(f"pcp_size above {kernel_limits.max_pcp_size}")
    return _capi.PcpDims(
        config.pcp_size,
        config.local_q_len,
        config.max_local_blocks,
        config.block_size,
        config.num_q_heads,
        config.num_kv_heads,
        config.head_dim,
        _kv_code(kv_dtype),
    )


def payload_elements(config: PCPAttentionConfig) -> int:
    return 2 * config.num_kv_heads * config.block_size * config.head_dim


def _cuda_stream_ptr(stream: torch.cuda.Stream | None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def check_ring_consistency(config: PCPAttentionConfig, valid_len, group=None) -> None:
    """Host-side guard before a device ring: every rank must hold the same
    static shape and the same per-source valid lengths, or the send/recv
    sizes disagree and the ring stalls (the reference's README warns that
    unequal ``actual_history_len`` deadlocks its collective ring).  Uses the
    default (or given) ``torch.distributed`` group; raises ``RuntimeError`` on
    the first mismatch, on every rank."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    mine = (
        config.pcp_size,
        config.current_len,
        config.max_history_len,
        config.block_size,
        config.interleave_size,
        config.num_q_heads,
        config.num_kv_heads,
        config.head_dim,
        tuple(int(v) for v in valid_len),
    )
    world = dist.get_world_size(group)
    gathered = [None] * world
    dist.all_gather_object(gathered, mine, group=group)
    for r, other in enumerate(gathered):
        if other != mine:
            raise RuntimeError(
                f"PCP ring configuration mismatch: rank {r} has {other}, this rank has {mine}"
            )


class HistoryAttention:
    """Per-rank CUDA history attention for one static ``PCPAttentionConfig``.

    ``rank``/``device`` default to ``torch.distributed``'s rank and the current
    CUDA device.  With ``pcp_size > 1`` construction is collective: rank 0
    creates the NCCL id and broadcasts it over ``group`` (any backend; gloo is
    enough), then every rank joins the ring communicator.

    ``exchange`` picks how the shards reach every rank: ``"direct"`` (each
    rank sends its shard to every peer in one NCCL group; the default on
    NVSwitch), ``"ring"`` (the reference's store-and-forward ring),
    ``"allgather"`` (one NCCL all-gather) or ``"pipeline"`` (one group per
    ring step, each step's shard attended as soon as it lands).
    ``comm_sms`` (default 16) is how many SMs the local-shard launch leaves to
    the direct exchange when ``pcp_size >= 4`` (``pcp_set_comm_sms``).
    ``kv_path`` picks how the KV cache is read (``pcp_set_kv_path``):
    ``"dense"`` (a dense bf16 copy per forward), ``"in_place"`` (e4m3 blocks
    read by TMA and upcast in shared memory) or ``"auto"``; None keeps the
    process default (``_capi.set_default_kv_path``).
    """

    def __init__(
        self,
        config: PCPAttentionConfig,
        kv_dtype: torch.dtype = torch.float8_e4m3fn,
        rank: int | None = None,
        device: int | torch.device | None = None,
        group=None,
        exchange: str = "direct",
        comm_sms: int | None = None,
        kv_path: str | None = None,
    ):
        self.config = config
        self.kv_dtype = kv_dtype
        self._dims = make_dims(config, kv_dtype)
        lib = _capi.lib()
        if rank is None:
            import torch.distributed as dist

            rank = dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device if isinstance(device, int) else device.index)
        self.rank = int(rank)
        uid = None
        if config.pcp_size > 1:
            import torch.distributed as dist

            if not dist.is_initialized():
                raise RuntimeError("pcp_size > 1 needs an initialised torch.distributed process group")
            check_ring_consistency(config, config.source_valid_lens(), group)
            nbytes = lib.pcp_nccl_unique_id_bytes()
            box = [None]
            if self.rank == 0:
                buf = ctypes.create_string_buffer(nbytes)
                _capi.check(lib.pcp_get_nccl_unique_id(buf))
                box[0] = bytes(buf.raw)
            dist.broadcast_object_list(box, src=0, group=group)
            uid = ctypes.create_string_buffer(box[0], nbytes)
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _capi.check(lib.pcp_create(ctypes.byref(self._dims), self.rank, self.device.index, uid, ctypes.byref(handle)))
        self._handle = handle
        modes = {"direct": _capi.PCP_EXCHANGE_DIRECT, "ring": _capi.PCP_EXCHANGE_RING,
                 "allgather": _capi.PCP_EXCHANGE_ALLGATHER, "pipeline": _capi.PCP_EXCHANGE_PIPELINE}
        if exchange not in modes:
            self.close()
            raise ValueError(f"exchange must be one of {sorted(modes)}, got {exchange!r}")
        _capi.check(lib.pcp_set_exchange(self._handle, modes[exchange]))
        self.exchange = exchange
        if comm_sms is not None:
            _capi.check(lib.pcp_set_comm_sms(self._handle, int(comm_sms)))
        if kv_path is not None:
            if kv_path not in _capi.KV_PATHS:
                self.close()
                raise ValueError(f"kv_path must be one of {sorted(_capi.KV_PATHS)}, got {kv_path!r}")
            _capi.check(lib.pcp_set_kv_path(self._handle, _capi.KV_PATHS[kv_path]))
        self.kv_path = kv_path or "default"

    # -- calls -------------------------------------------------------------
    def _check_inputs(self, q: torch.Tensor, packed_kv: torch.Tensor) -> None:
        cfg = self.config
        qshape = (cfg.num_q_heads, cfg.local_q_len, cfg.head_dim)
        kvshape = (cfg.max_local_blocks, payload_elements(cfg))
        if tuple(q.shape) != qshape or q.dtype != torch.bfloat16:
            raise ValueError(f"expected Q {qshape} bf16, got {tuple(q.shape)} {q.dtype}")
        if tuple(packed_kv.shape) != kvshape or packed_kv.dtype != self.kv_dtype:
            raise ValueError(f"expected packed KV {kvshape} {self.kv_dtype}, got {tuple(packed_kv.shape)} {packed_kv.dtype}")
        for name, t in (("q", q), ("packed_kv", packed_kv)):
            if t.device != self.device:
                raise ValueError(f"{name} is on {t.device}, expected {self.device}")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")

    def _valid(self, valid_len) -> ctypes.Array:
        if valid_len is None:
            valid_len = self.config.source_valid_lens()
        vals = [int(v) for v in valid_len]
        if len(vals) != self.config.pcp_size:
            raise ValueError(f"valid_len needs {self.config.pcp_size} entries, got {len(vals)}")
        return _capi.int32_array(vals)

    def __call__(self, q: torch.Tensor, packed_kv: torch.Tensor, valid_len=None, out: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        self._check_inputs(q, packed_kv)
        if out is None:
            out = torch.empty_like(q)
        elif tuple(out.shape) != tuple(q.shape) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bf16 tensor shaped like q")
        vals = self._valid(valid_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward(
                    self._handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed_kv.data_ptr()), vals,
                    ctypes.c_void_p(out.data_ptr()), _cuda_stream_ptr(stream)
                )
            )
        return out

    def forward_bucketed(self, q: torch.Tensor, packed_kv: torch.Tensor, valid_dev: torch.Tensor, bucket_len,
                         out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """``__call__`` whose valid lengths are read on the device from
        ``valid_dev`` (int32 ``[P]``) when the kernels run; ``bucket_len`` (P
        ints) bounds them and sizes every transfer and launch.  This is the
        call a length-bucket CUDA graph records (``graphs.BucketGraph``)."""
        self._check_inputs(q, packed_kv)
        if valid_dev.dtype != torch.int32 or valid_dev.numel() != self.config.pcp_size or \
                valid_dev.device != self.device or not valid_dev.is_contiguous():
            raise ValueError(f"valid_dev must be a contiguous int32 [{self.config.pcp_size}] tensor on {self.device}")
        if out is None:
            out = torch.empty_like(q)
        elif tuple(out.shape) != tuple(q.shape) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bf16 tensor shaped like q")
        bounds = self._valid(bucket_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward_bucketed(
                    self._handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed_kv.data_ptr()),
                    ctypes.c_void_p(valid_dev.data_ptr()), bounds, ctypes.c_void_p(out.data_ptr()),
                    _cuda_stream_ptr(stream)
                )
            )
        return out

    def forward_paged(self, q: torch.Tensor, pool: torch.Tensor, block_table: torch.Tensor, valid_len=None,
                      out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """``__call__`` with this rank's history shard in a block pool
        (``[pool_blocks, payload]``, see ``paged.make_pool``): logical block b
        is pool block ``block_table[b]`` (int32 ``[max_local_blocks]`` on the
        device)."""
        cfg = self.config
        if tuple(q.shape) != (cfg.num_q_heads, cfg.local_q_len, cfg.head_dim) or q.dtype != torch.bfloat16:
            raise ValueError("bad Q")
        if pool.dim() != 2 or pool.shape[1] != payload_elements(cfg) or pool.dtype != self.kv_dtype:
            raise ValueError(f"pool must be [blocks, {payload_elements(cfg)}] {self.kv_dtype}")
        if block_table.dtype != torch.int32 or block_table.numel() != cfg.max_local_blocks:
            raise ValueError(f"block_table must be int32 [{cfg.max_local_blocks}]")
        for name, t in (("q", q), ("pool", pool), ("block_table", block_table)):
            if t.device != self.device or not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous on {self.device}")
        if out is None:
            out = torch.empty_like(q)
        vals = self._valid(valid_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward_paged(
                    self._handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(pool.data_ptr()),
                    int(pool.shape[0]), ctypes.c_void_p(block_table.data_ptr()), vals,
                    ctypes.c_void_p(out.data_ptr()), _cuda_stream_ptr(stream)
                )
            )
        return out

    def prefill(self, q: torch.Tensor, packed_kv: torch.Tensor, k_cur: torch.Tensor, v_cur: torch.Tensor,
                valid_len=None, out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """History attention plus causal attention over the current (prefill)
        tokens of every rank, merged by log-sum-exp.  ``k_cur``/``v_cur`` are
        this rank's current tokens' K/V shard ``[Hkv, Qloc, D]`` bf16, striped
        like ``q`` (``shard_query`` layout); a query sees every history key and
        the current keys at global positions up to its own."""
        self._check_inputs(q, packed_kv)
        _check_current(self.config, k_cur, v_cur, False, self.device)
        if out is None:
            out = torch.empty_like(q)
        elif tuple(out.shape) != tuple(q.shape) or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bf16 tensor shaped like q")
        vals = self._valid(valid_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward_prefill(
                    self._handle, self.config.interleave_size, ctypes.c_void_p(q.data_ptr()),
                    ctypes.c_void_p(packed_kv.data_ptr()), vals, ctypes.c_void_p(k_cur.data_ptr()),
                    ctypes.c_void_p(v_cur.data_ptr()), ctypes.c_void_p(out.data_ptr()), _cuda_stream_ptr(stream)
                )
            )
        return out

    def forward_host(self, q: torch.Tensor, packed_kv: torch.Tensor, valid_len=None, out: torch.Tensor | None = None,
                     stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """End-to-end call with host tensors: H2D copies, forward, D2H copy, sync."""
        cfg = self.config
        if q.device.type != "cpu" or packed_kv.device.type != "cpu":
            raise ValueError("forward_host takes CPU tensors")
        if tuple(q.shape) != (cfg.num_q_heads, cfg.local_q_len, cfg.head_dim) or q.dtype != torch.bfloat16:
            raise ValueError("bad Q")
        if tuple(packed_kv.shape) != (cfg.max_local_blocks, payload_elements(cfg)) or packed_kv.dtype != self.kv_dtype:
            raise ValueError("bad packed KV")
        if out is None:
            out = torch.empty_like(q, pin_memory=q.is_pinned())
        vals = self._valid(valid_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward_host(
                    self._handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed_kv.data_ptr()), vals,
                    ctypes.c_void_p(out.data_ptr()), _cuda_stream_ptr(stream)
                )
            )
        return out

    def forward_host_async(self, q: torch.Tensor, packed_kv: torch.Tensor, valid_len=None,
                           out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """``forward_host`` without waiting (``pcp_forward_host_async``): the
        copies and the forward are enqueued and the call returns; one call's
        copies overlap the previous call's forward.  ``q``, ``packed_kv`` and
        ``out`` should be pinned; keep them unmodified (and do not read ``out``)
        until ``forward_host_wait``."""
        cfg = self.config
        if q.device.type != "cpu" or packed_kv.device.type != "cpu":
            raise ValueError("forward_host_async takes CPU tensors")
        if tuple(q.shape) != (cfg.num_q_heads, cfg.local_q_len, cfg.head_dim) or q.dtype != torch.bfloat16:
            raise ValueError("bad Q")
        if tuple(packed_kv.shape) != (cfg.max_local_blocks, payload_elements(cfg)) or packed_kv.dtype != self.kv_dtype:
            raise ValueError("bad packed KV")
        if out is None:
            out = torch.empty_like(q, pin_memory=True)
        vals = self._valid(valid_len)
        with torch.cuda.device(self.device):
            _capi.check(
                _capi.lib().pcp_forward_host_async(
                    self._handle, ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed_kv.data_ptr()), vals,
                    ctypes.c_void_p(out.data_ptr()), _cuda_stream_ptr(stream)
                )
            )
        return out

    def forward_host_wait(self) -> None:
        """Waits for every ``forward_host_async`` of this handle."""
        _capi.check(_capi.lib().pcp_forward_host_wait(self._handle))

    def status(self, timeout_ms: int = 60000) -> None:
        """Wait for the last call and raise on device timeouts / ring failures."""
        _capi.check(_capi.lib().pcp_device_status(self._handle, int(timeout_ms)))

    def set_profiling(self, enable: bool) -> None:
        _capi.check(_capi.lib().pcp_set_profiling(self._handle, 1 if enable else 0))

    def stats(self) -> dict:
        st = _capi.PcpStats()
        _capi.check(_capi.lib().pcp_get_stats(self._handle, ctypes.byref(st)))
        return {name: getattr(st, name) for name, _ in _capi.PcpStats._fields_}

    def _register_graph(self, graph) -> None:
        import weakref

        if not hasattr(self, "_graphs"):
            self._graphs = weakref.WeakSet()
        self._graphs.add(graph)

    def close(self) -> None:
        # Graphs that recorded this handle's NCCL calls go before the communicator.
        for g in list(getattr(self, "_graphs", ())):
            g.reset()
        if getattr(self, "_handle", None) is not None and self._handle.value:
            _capi.lib().pcp_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _check_current(config: PCPAttentionConfig, k_cur: torch.Tensor, v_cur: torch.Tensor, all_ranks: bool,
                   device: torch.device | None) -> None:
    shape = (config.num_kv_heads, config.local_q_len, config.head_dim)
    if all_ranks:
        shape = (config.pcp_size,) + shape
    for name, t in (("k_cur", k_cur), ("v_cur", v_cur)):
        if tuple(t.shape) != shape or t.dtype != torch.bfloat16:
            raise ValueError(f"expected {name} {shape} bf16, got {tuple(t.shape)} {t.dtype}")
        if not t.is_cuda or not t.is_contiguous() or (device is not None and t.device != device):
            raise ValueError(f"{name} must be a contiguous CUDA tensor on {device}")
    if config.local_q_len % config.interleave_size:
        raise ValueError("interleave_size must divide local_q_len")


def prefill_attention_single(q: torch.Tensor, packed_kv: torch.Tensor | None, valid_len, k_cur_all: torch.Tensor,
                             v_cur_all: torch.Tensor, config: PCPAttentionConfig, rank: int,
                             kv_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
                             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Stateless single-GPU prefill (``pcp_prefill_attention``): rank
    ``rank``'s Q shard against ``len(valid_len)`` resident history shards
    (as in ``history_attention_single``) and, causally, the current tokens of
    all ``pcp_size`` ranks, ``k_cur_all``/``v_cur_all`` ``[P, Hkv, Qloc, D]``
    bf16 (rank s's striped shard at index s)."""
    vals = [int(v) for v in valid_len]
    nsrc = len(vals)
    if packed_kv is None:
        if any(vals):
            raise ValueError("history tokens given without packed_kv")
        kv_dtype = kv_dtype or torch.float8_e4m3fn
    else:
        kv_dtype = kv_dtype or packed_kv.dtype
        if tuple(packed_kv.shape) != (nsrc * config.max_local_blocks, payload_elements(config)):
            raise ValueError(f"packed KV must be [{nsrc * config.max_local_blocks}, {payload_elements(config)}]")
        if not (packed_kv.is_cuda and packed_kv.is_contiguous()):
            raise ValueError("packed_kv must be a contiguous CUDA tensor")
    dims = make_dims(config, kv_dtype)
    if q.dtype != torch.bfloat16 or tuple(q.shape) != (config.num_q_heads, config.local_q_len, config.head_dim):
        raise ValueError("bad Q")
    if not (q.is_cuda and q.is_contiguous()):
        raise ValueError("q must be a contiguous CUDA tensor")
    _check_current(config, k_cur_all, v_cur_all, True, q.device)
    if not 0 <= rank < config.pcp_size:
        raise ValueError(f"rank {rank} outside [0, {config.pcp_size})")
    lib = _capi.lib()
    nbytes = ctypes.c_size_t()
    _capi.check(lib.pcp_prefill_attention_workspace_size(ctypes.byref(dims), sum(vals), ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty_like(q)
    kv_ptr = packed_kv.data_ptr() if packed_kv is not None else 0
    with torch.cuda.device(q.device):
        _capi.check(
            lib.pcp_prefill_attention(
                ctypes.byref(dims), config.interleave_size, rank, ctypes.c_void_p(q.data_ptr()),
                ctypes.c_void_p(kv_ptr), nsrc, _capi.int32_array(vals) if nsrc else None,
                ctypes.c_void_p(k_cur_all.data_ptr()), ctypes.c_void_p(v_cur_all.data_ptr()),
                ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes.value,
                _cuda_stream_ptr(stream)
            )
        )
        _capi.check(lib.pcp_history_attention_status(ctypes.c_void_p(ws.data_ptr()), _cuda_stream_ptr(stream)))
    return out


def history_attention_single(q: torch.Tensor, packed_kv: torch.Tensor, valid_len, config: PCPAttentionConfig,
                             kv_dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
                             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Stateless single-GPU entry (``pcp_history_attention``): ``packed_kv`` holds
    ``len(valid_len)`` source shards back to back, ``[sources * max_local_blocks,
    payload]``; workspace is allocated here from torch's caching allocator."""
    kv_dtype = kv_dtype or packed_kv.dtype
    dims = make_dims(config, kv_dtype)
    vals = [int(v) for v in valid_len]
    nsrc = len(vals)
    if tuple(packed_kv.shape) != (nsrc * config.max_local_blocks, payload_elements(config)):
        raise ValueError(f"packed KV must be [{nsrc * config.max_local_blocks}, {payload_elements(config)}]")
    if q.dtype != torch.bfloat16 or tuple(q.shape) != (config.num_q_heads, config.local_q_len, config.head_dim):
        raise ValueError("bad Q")
    if not (q.is_cuda and packed_kv.is_cuda and q.is_contiguous() and packed_kv.is_contiguous()):
        raise ValueError("q and packed_kv must be contiguous CUDA tensors")
    lib = _capi.lib()
    nbytes = ctypes.c_size_t()
    _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(dims), sum(vals), ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty_like(q)
    with torch.cuda.device(q.device):
        _capi.check(
            lib.pcp_history_attention(
                ctypes.byref(dims), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed_kv.data_ptr()), nsrc,
                _capi.int32_array(vals), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                nbytes.value, _cuda_stream_ptr(stream)
            )
        )
        _capi.check(lib.pcp_history_attention_status(ctypes.c_void_p(ws.data_ptr()), _cuda_stream_ptr(stream)))
    return out
