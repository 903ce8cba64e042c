"""Striped token ownership and host-side shard/gather helpers.

Same functions, argument meaning, shapes and errors as the reference's
``pcp_attention/layout.py:10-132``; results are bit-exact with it whenever the
reference accepts the input.  For an ``actual_history_len`` that is not a
multiple of ``pcp_size * interleave_size`` (which the reference rejects),
positions are taken from the aligned superset and truncated at the actual
length, so each rank's shard holds exactly ``config.source_valid_len(rank)``
tokens, zero-padded to ``config.local_cache_blocks`` blocks.

For a global position ``p``::

    chunk       = p // interleave_size
    owner_rank  = chunk % pcp_size
    local_pos   = (chunk // pcp_size) * interleave_size + p % interleave_size
"""

from __future__ import annotations

import torch

from .config import PCPAttentionConfig


def owner_and_local_position(
    global_position: int, pcp_size: int, interleave_size: int
) -> tuple[int, int]:
    """Owner rank and local position of one global token (``layout.py:10-16``)."""
    chunk, within_chunk = divmod(global_position, interleave_size)
    return chunk % pcp_size, (chunk // pcp_size) * interleave_size + within_chunk


def global_positions_for_rank(
    total_len: int, rank: int, pcp_size: int, interleave_size: int
) -> torch.Tensor:
    """int64 global positions owned by ``rank``, in local order (``layout.py:19-31``).

    Raises like the reference when ``total_len`` does not divide evenly across
    the striped ranks; ``_positions_upto`` is the ragged variant.
    """
    if not 0 <= rank < pcp_size:
        raise ValueError(f"rank {rank} is outside [0, {pcp_size})")
    if total_len % (pcp_size * interleave_size):
        raise ValueError("total_len must divide evenly across striped ranks")
    return _positions_upto(total_len, rank, pcp_size, interleave_size)


def _positions_upto(total_len: int, rank: int, pcp_size: int, interleave_size: int) -> torch.Tensor:
    stride = pcp_size * interleave_size
    chunks = -(-total_len // stride)
    base = (torch.arange(chunks, dtype=torch.int64) * pcp_size + rank) * interleave_size
    within = torch.arange(interleave_size, dtype=torch.int64)
    positions = (base[:, None] + within[None, :]).reshape(-1)
    if total_len % stride:
        positions = positions[positions < total_len]
    return positions


def shard_query(q: torch.Tensor, config: PCPAttentionConfig) -> list[torch.Tensor]:
    """Shard global ``[Hq, current_len, D]`` Q by striped ownership (``layout.py:34-51``).

    Ownership is computed on positions relative to the current segment, as in
    the reference.  History-only attention treats every query row
    independently, so this choice moves rows between ranks but never changes
    a row's result.
    """
    config.validate()
    expected = (config.num_q_heads, config.current_len, config.head_dim)
    if tuple(q.shape) != expected:
        raise ValueError(f"expected Q shape {expected}, got {tuple(q.shape)}")
    return [
        q[:, global_positions_for_rank(
            config.current_len, rank, config.pcp_size, config.interleave_size
        ).to(q.device), :].contiguous()
        for rank in range(config.pcp_size)
    ]


def shard_history(
    k: torch.Tensor, v: torch.Tensor, config: PCPAttentionConfig
) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    """Shard global history into per-rank paged caches (``layout.py:54-98``).

    Input K/V ``[Hkv, actual_history_len, D]``; output per rank
    ``[local_cache_blocks, Hkv, block_size, D]`` with the unused tail of the
    last block zeroed.
    """
    config.validate()
    expected = (config.num_kv_heads, config.actual_history_len, config.head_dim)
    if tuple(k.shape) != expected or tuple(v.shape) != expected:
        raise ValueError(
            f"expected K/V shape {expected}, got {tuple(k.shape)} and {tuple(v.shape)}"
        )
    blocks = config.local_cache_blocks
    k_shards: list[torch.Tensor] = []
    v_shards: list[torch.Tensor] = []
    for rank in range(config.pcp_size):
        positions = _positions_upto(
            config.actual_history_len, rank, config.pcp_size, config.interleave_size
        ).to(k.device)

        def to_cache_layout(tensor: torch.Tensor) -> torch.Tensor:
            padded = torch.zeros(
                (config.num_kv_heads, blocks * config.block_size, config.head_dim),
                dtype=tensor.dtype,
                device=tensor.device,
            )
            padded[:, : positions.numel(), :] = tensor[:, positions, :]
            return padded.reshape(
                config.num_kv_heads, blocks, config.block_size, config.head_dim
            ).permute(1, 0, 2, 3).contiguous()

        k_shards.append(to_cache_layout(k))
        v_shards.append(to_cache_layout(v))
    return k_shards, v_shards


def gather_history(shards: list[torch.Tensor], config: PCPAttentionConfig) -> torch.Tensor:
    """Invert ``shard_history`` for one of K or V (``layout.py:101-132``)."""
    config.validate()
    if len(shards) != config.pcp_size:
        raise ValueError(f"expected {config.pcp_size} shards, got {len(shards)}")
    sample = shards[0]
    result = torch.empty(
        (config.num_kv_heads, config.actual_history_len, config.head_dim),
        dtype=sample.dtype,
        device=sample.device,
    )
    expected = (
        config.local_cache_blocks,
        config.num_kv_heads,
        config.block_size,
        config.head_dim,
    )
    for rank, shard in enumerate(shards):
        if tuple(shard.shape) != expected:
            raise ValueError(f"rank {rank}: expected {expected}, got {tuple(shard.shape)}")
        positions = _positions_upto(
            config.actual_history_len, rank, config.pcp_size, config.interleave_size
        ).to(shard.device)
        local = shard.permute(1, 0, 2, 3).reshape(config.num_kv_heads, -1, config.head_dim)
        result[:, positions, :] = local[:, : positions.numel(), :]
    return result
