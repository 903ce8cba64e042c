"""Paged KV cache on the device: the producer that writes new tokens into a
rank's block pool, and the history attention that reads a pool through block
tables.

The reference builds each rank's cache on the host: ``shard_history``
(``pcp_attention/layout.py:54-98``) stripes a global K/V over the ranks and
reshapes each shard to ``[blocks, Hkv, bs, D]``; ``pack_local_kv``
(``pcp_attention/kernel.py:17-29``) packs a block's K then V into the ring
payload; FP8 comes from ``tensor.to(torch.float8_e4m3fn)`` (``run_poc.py:81-134``).
Here the same cache is produced by a CUDA kernel, token by token, into a pool
of physical blocks addressed through a block table (logical local block b of
this rank -> pool block ``block_table[b]``), so a serving loop can append the
tokens of each prefill without host copies and without contiguous shards.

Pool layout: ``[pool_blocks, 2 * Hkv * bs * D]`` in the cache dtype (e4m3fn or
bf16) -- the packed payload format, one block per row.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _capi
from .config import PCPAttentionConfig
from .cuda_backend import _cuda_stream_ptr, make_dims, payload_elements


def make_pool(config: PCPAttentionConfig, pool_blocks: int, kv_dtype: torch.dtype = torch.float8_e4m3fn,
              device: int | torch.device | str = "cuda") -> torch.Tensor:
    """A zeroed block pool ``[pool_blocks, payload]``."""
    if pool_blocks <= 0:
        raise ValueError("pool_blocks must be positive")
    return torch.zeros((pool_blocks, payload_elements(config)), dtype=kv_dtype, device=device)


def local_blocks_needed(config: PCPAttentionConfig, rank: int, total_len: int) -> int:
    """Logical blocks rank ``rank`` needs to hold its share of positions
    ``[0, total_len)``."""
    return -(-config_source_len(config, rank, total_len) // config.block_size)


def config_source_len(config: PCPAttentionConfig, rank: int, total_len: int) -> int:
    """Positions of ``[0, total_len)`` that rank ``rank`` owns (stripe layout,
    ``layout.py:10-31``)."""
    stride = config.pcp_size * config.interleave_size
    return (total_len // stride) * config.interleave_size + min(
        max(total_len % stride - rank * config.interleave_size, 0), config.interleave_size
    )


def _check_pool(config: PCPAttentionConfig, pool: torch.Tensor, kv_dtype: torch.dtype) -> None:
    if pool.dim() != 2 or pool.shape[1] != payload_elements(config) or pool.dtype != kv_dtype:
        raise ValueError(f"pool must be [blocks, {payload_elements(config)}] {kv_dtype}, got "
                         f"{tuple(pool.shape)} {pool.dtype}")
    if not (pool.is_cuda and pool.is_contiguous()):
        raise ValueError("pool must be a contiguous CUDA tensor")


def _check_table(table: torch.Tensor, device: torch.device) -> None:
    if table.dtype != torch.int32 or not table.is_contiguous() or table.device != device:
        raise ValueError(f"block table must be a contiguous int32 tensor on {device}")


def cache_write(config: PCPAttentionConfig, rank: int, first_position: int, k_src: torch.Tensor,
                v_src: torch.Tensor, block_table: torch.Tensor, pool: torch.Tensor,
                status: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Write the tokens of ``k_src``/``v_src`` (``[Hkv, T, D]`` bf16, sequence
    order, token t at absolute position ``first_position + t``) that rank
    ``rank`` owns into its pool, quantised to the pool's dtype.  Returns the
    device int32 status word (0, or 109 when a table entry lies outside the
    pool; that token is skipped).  Asynchronous on ``stream``."""
    kv_dtype = pool.dtype
    dims = make_dims(config, kv_dtype)
    _check_pool(config, pool, kv_dtype)
    _check_table(block_table, pool.device)
    shape = (config.num_kv_heads, k_src.shape[1] if k_src.dim() == 3 else -1, config.head_dim)
    for name, t in (("k_src", k_src), ("v_src", v_src)):
        if t.dim() != 3 or tuple(t.shape) != shape or t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be [Hkv, T, D] bf16 {shape}, got {tuple(t.shape)} {t.dtype}")
        if not t.is_contiguous() or t.device != pool.device:
            raise ValueError(f"{name} must be contiguous on {pool.device}")
    if status is None:
        status = torch.empty(1, dtype=torch.int32, device=pool.device)
    with torch.cuda.device(pool.device):
        _capi.check(
            _capi.lib().pcp_cache_write(
                ctypes.byref(dims), config.interleave_size, rank, int(first_position), int(k_src.shape[1]),
                ctypes.c_void_p(k_src.data_ptr()), ctypes.c_void_p(v_src.data_ptr()),
                ctypes.c_void_p(block_table.data_ptr()), int(block_table.numel()), ctypes.c_void_p(pool.data_ptr()),
                int(pool.shape[0]), ctypes.c_void_p(status.data_ptr()), _cuda_stream_ptr(stream)
            )
        )
    return status


def history_attention_paged_single(q: torch.Tensor, pool: torch.Tensor, block_tables: torch.Tensor, valid_len,
                                   config: PCPAttentionConfig, out: torch.Tensor | None = None,
                                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """``history_attention_single`` over paged shards: source s's logical
    blocks are pool blocks ``block_tables[s]`` (``[sources, max_local_blocks]``
    int32 on the device)."""
    kv_dtype = pool.dtype
    dims = make_dims(config, kv_dtype)
    _check_pool(config, pool, kv_dtype)
    vals = [int(v) for v in valid_len]
    nsrc = len(vals)
    _check_table(block_tables, pool.device)
    if tuple(block_tables.shape) != (nsrc, config.max_local_blocks):
        raise ValueError(f"block_tables must be [{nsrc}, {config.max_local_blocks}]")
    if q.dtype != torch.bfloat16 or tuple(q.shape) != (config.num_q_heads, config.local_q_len, config.head_dim):
        raise ValueError("bad Q")
    if not (q.is_cuda and q.is_contiguous()):
        raise ValueError("q must be a contiguous CUDA tensor")
    lib = _capi.lib()
    nbytes = ctypes.c_size_t()
    _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(dims), sum(vals), ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty_like(q)
    with torch.cuda.device(q.device):
        _capi.check(
            lib.pcp_history_attention_paged(
                ctypes.byref(dims), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(pool.data_ptr()),
                int(pool.shape[0]), ctypes.c_void_p(block_tables.data_ptr()), nsrc, _capi.int32_array(vals),
                ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes.value,
                _cuda_stream_ptr(stream)
            )
        )
        _capi.check(lib.pcp_history_attention_status(ctypes.c_void_p(ws.data_ptr()), _cuda_stream_ptr(stream)))
    return out
