"""Prefill context-parallel history attention, B200 CUDA backend.

Same public names as the reference package ``pcp_attention``
(``pcp_attention/__init__.py``) for the config and layout API; the NKI kernel
is replaced by the CUDA ``HistoryAttention``.  There is no CPU compute path.
"""

from .config import PCPAttentionConfig, get_preset
from .layout import (
    gather_history,
    global_positions_for_rank,
    owner_and_local_position,
    shard_history,
    shard_query,
)
from .kernel import pack_local_kv, wrap_for_native_torch, make_history_attention_kernel

__all__ = [
    "PCPAttentionConfig",
    "gather_history",
    "get_preset",
    "global_positions_for_rank",
    "make_history_attention_kernel",
    "owner_and_local_position",
    "pack_local_kv",
    "shard_history",
    "shard_query",
    "wrap_for_native_torch",
]
