"""Seeded synthetic inputs and the additive block-valid mask.

``make_inputs`` / ``make_local_inputs`` / ``make_block_valid_mask`` reproduce
``run_poc.py:81-153`` of the reference bit for bit (same torch generator,
draw order and dtypes).  ``make_baseline_inputs`` draws the benchmark
distributions: Q bf16 ~ N(0,1); K/V ~ 0.5 * N(0,1) cast to e4m3fn (or kept
bf16), optionally with a fraction of K/V entries scaled x8 before the cast.
"""

from __future__ import annotations

import torch

from .config import PCPAttentionConfig


def make_inputs(cfg: PCPAttentionConfig, seed: int):
    """Global Q ``[Hq, current_len, D]`` bf16 and K/V ``[Hkv, A, D]`` e4m3fn (run_poc.py:81-104)."""
    generator = torch.Generator().manual_seed(seed)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=generator, dtype=torch.bfloat16)
    k = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=generator,
                    dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    v = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=generator,
                    dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    return q, k, v


def make_local_inputs(cfg: PCPAttentionConfig, seed: int, rank: int):
    """One rank's Q shard and paged K/V cache (run_poc.py:107-134)."""
    generator = torch.Generator().manual_seed(seed + 104729 * rank)
    q = torch.randn(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, generator=generator, dtype=torch.bfloat16)
    cache_shape = (cfg.actual_local_blocks, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    k = torch.randn(*cache_shape, generator=generator, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    v = torch.randn(*cache_shape, generator=generator, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    return q, k, v


def make_block_valid_mask(cfg: PCPAttentionConfig) -> torch.Tensor:
    """Additive score bias ``[max_local_blocks, bs/128, 1, 128]`` bf16: 0 for the
    first ``actual_local_history_len`` tokens, -9984 after (run_poc.py:137-153)."""
    kv_tiles = cfg.block_size // 128
    mask = torch.full((cfg.max_local_blocks, kv_tiles, 1, 128), fill_value=-9984.0, dtype=torch.bfloat16)
    remaining = cfg.actual_local_history_len
    for block in range(cfg.actual_local_blocks):
        valid_in_block = min(cfg.block_size, remaining)
        for tile in range(kv_tiles):
            valid_in_tile = min(128, max(0, valid_in_block - tile * 128))
            mask[block, tile, 0, :valid_in_tile] = 0
        remaining -= valid_in_block
    return mask


def make_baseline_inputs(cfg: PCPAttentionConfig, seed: int, kv_dtype: torch.dtype = torch.float8_e4m3fn,
                         kv_scale: float = 0.5, outlier_frac: float = 0.0, outlier_mult: float = 8.0,
                         device: torch.device | str = "cpu"):
    """Global Q ``[Hq, current_len, D]`` bf16 and K/V ``[Hkv, A, D]`` in ``kv_dtype``."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=g, device=device,
                    dtype=torch.float32).to(torch.bfloat16)
    kv = []
    for _ in range(2):
        t = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g, device=device,
                        dtype=torch.float32) * kv_scale
        if outlier_frac > 0:
            sel = torch.rand(t.shape, generator=g, device=device) < outlier_frac
            t = torch.where(sel, t * outlier_mult, t)
        kv.append(t.to(kv_dtype))
    return q, kv[0], kv[1]


def make_local_baseline_inputs(cfg: PCPAttentionConfig, seed: int, rank: int,
                               kv_dtype: torch.dtype = torch.float8_e4m3fn, kv_scale: float = 0.5,
                               outlier_frac: float = 0.0, outlier_mult: float = 8.0,
                               device: torch.device | str = "cpu"):
    """One rank's Q shard ``[Hq, Qloc, D]`` and packed KV ``[max_local_blocks,
    payload]`` (live blocks drawn, padding zero), drawn directly on ``device``
    with the benchmark distributions (no global tensors: memory-safe at full size)."""
    from .kernel import pack_local_kv

    g = torch.Generator(device=device).manual_seed(seed + 104729 * rank)
    q = torch.randn(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, generator=g, device=device,
                    dtype=torch.float32).to(torch.bfloat16)
    valid = cfg.source_valid_len(rank)
    shape = (cfg.max_local_blocks, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    parts = []
    for _ in range(2):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * kv_scale
        if outlier_frac > 0:
            sel = torch.rand(shape, generator=g, device=device) < outlier_frac
            t = torch.where(sel, t * outlier_mult, t)
        # zero the padding past this rank's valid tokens
        tok = torch.arange(cfg.max_local_blocks * cfg.block_size, device=device).reshape(cfg.max_local_blocks, 1,
                                                                                        cfg.block_size, 1)
        t = torch.where(tok < valid, t, torch.zeros((), device=device))
        parts.append(t.to(kv_dtype))
    return q, pack_local_kv(parts[0], parts[1])
