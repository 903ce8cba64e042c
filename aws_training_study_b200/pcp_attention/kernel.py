"""Drop-in for the reference's ``pcp_attention/kernel.py``.

* ``pack_local_kv`` -- identical ring payload format (``kernel.py:17-29``).
* ``make_history_attention_kernel(config)`` -- returns the CUDA
  ``HistoryAttention`` for this rank instead of an NKI kernel
  (``kernel.py:32-556``).
* ``wrap_for_native_torch(config)`` -- returns ``kernel(q, packed_kv,
  block_valid_mask) -> out`` with the reference's signature
  (``kernel.py:559-564``).  The additive mask of ``run_poc.py:137-153`` is
  turned into the valid-token count it encodes (it is the same for every
  source rank in the reference), so existing callers need no change.
"""

from __future__ import annotations

from typing import Any

import torch

from .config import PCPAttentionConfig


def pack_local_kv(k: Any, v: Any) -> Any:
    """Pack ``[blocks, Hkv, block_size, D]`` K and V into the ring payload
    ``[blocks, 2 * Hkv * block_size * D]`` with all K before all V per block."""
    if k.shape != v.shape or k.ndim != 4:
        raise ValueError("K and V must have equal [blocks, Hkv, block, D] shapes")
    if k.dtype in (torch.float8_e4m3fn, torch.float8_e5m2) and k.dtype == v.dtype:
        # Byte copy: stacking works on every device for uint8 storage.
        packed = torch.stack((k.view(torch.uint8), v.view(torch.uint8)), dim=1)
        return packed.reshape(k.shape[0], -1).contiguous().view(k.dtype)
    return torch.stack((k, v), dim=1).reshape(k.shape[0], -1).contiguous()


def valid_tokens_from_mask(block_valid_mask: torch.Tensor, config: PCPAttentionConfig) -> int:
    """Valid tokens encoded by a ``[max_local_blocks, bs/128, 1, 128]`` additive
    bias (0 = valid, -9984 = masked), as built by ``make_block_valid_mask``."""
    expected = (config.max_local_blocks, config.block_size // 128, 1, 128)
    if tuple(block_valid_mask.shape) != expected:
        raise ValueError(f"expected mask shape {expected}, got {tuple(block_valid_mask.shape)}")
    valid = (block_valid_mask.reshape(config.max_local_blocks, -1) == 0)
    counts = valid.sum(dim=1).tolist()
    total = 0
    for b, c in enumerate(counts):
        # Valid tokens form a prefix of the shard: full blocks, then one partial.
        if c and total != b * config.block_size:
            raise ValueError("block_valid_mask does not describe a prefix of valid tokens")
        total += int(c)
    return total


def make_history_attention_kernel(config: PCPAttentionConfig, kv_dtype: torch.dtype = torch.float8_e4m3fn,
                                  rank: int | None = None, group=None):
    """CUDA history attention for every field of ``config`` (the handle sizes
    its buffers for ``max_local_blocks``; ``valid_len`` varies per call)."""
    from .cuda_backend import HistoryAttention

    return HistoryAttention(config, kv_dtype=kv_dtype, rank=rank, group=group)


def wrap_for_native_torch(config: PCPAttentionConfig, kv_dtype: torch.dtype = torch.float8_e4m3fn):
    """``kernel(q, packed_kv, block_valid_mask) -> out`` like the reference."""
    attn = make_history_attention_kernel(config, kv_dtype=kv_dtype)

    def kernel(q: torch.Tensor, packed_kv: torch.Tensor, block_valid_mask: torch.Tensor) -> torch.Tensor:
        valid = valid_tokens_from_mask(block_valid_mask, config)
        return attn(q, packed_kv, [valid] * config.pcp_size)

    kernel.history_attention = attn
    return kernel
