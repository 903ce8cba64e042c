"""Shared helpers of the parity tests: seeded inputs, the oracle's expected
output for one rank, and the error metrics with their bounds.

Bounds on the bf16 output (written here, used by every GPU parity test):
  * max-abs <= 2e-2 and mean-abs <= 2e-3 (the BASELINE tolerance),
  * relative L2 error <= 1e-2, because at long history |O| shrinks like
    1/sqrt(hist) and an all-zero output would pass the absolute bounds,
  * the output is not trivially small: ||O|| >= 0.25 ||O_ref||.
"""

from __future__ import annotations

import numpy as np
import torch

from aws_training_study_b200.pcp_attention import (
    PCPAttentionConfig,
    global_positions_for_rank,
    pack_local_kv,
    shard_history,
    shard_query,
)
from aws_training_study_b200.pcp_attention.inputs import make_baseline_inputs
from oracle import pcp_oracle as orc

MAX_ABS = 2e-2
MEAN_ABS = 2e-3
REL_L2 = 1e-2


def oracle_config(cfg: PCPAttentionConfig) -> orc.OracleConfig:
    return orc.OracleConfig(
        pcp_size=cfg.pcp_size,
        current_len=cfg.current_len,
        max_history_len=cfg.max_history_len,
        actual_history_len=cfg.actual_history_len,
        block_size=cfg.block_size,
        interleave_size=cfg.interleave_size,
        num_q_heads=cfg.num_q_heads,
        num_kv_heads=cfg.num_kv_heads,
        head_dim=cfg.head_dim,
    )


def to_numpy_f32(t: torch.Tensor) -> np.ndarray:
    """Exact fp32 values of bf16 / e4m3fn / fp32 tensors, decoded by the oracle."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        return orc.e4m3fn_decode(t.view(torch.uint8).numpy())
    if t.dtype == torch.bfloat16:
        return orc.bf16_bits_to_float32(t.view(torch.int16).numpy().view(np.uint16))
    return t.float().numpy()


def make_case(cfg: PCPAttentionConfig, seed: int, kv_dtype=torch.float8_e4m3fn, outlier_frac: float = 0.0):
    """Global inputs drawn on the CPU and sharded with the product layout."""
    q, k, v = make_baseline_inputs(cfg, seed, kv_dtype=kv_dtype, outlier_frac=outlier_frac)
    q_shards = shard_query(q, cfg)
    k_shards, v_shards = shard_history(k, v, cfg)
    return q, k, v, q_shards, k_shards, v_shards


def packed_shards(cfg: PCPAttentionConfig, k_shards, v_shards) -> list[torch.Tensor]:
    """Per-rank ring payload padded to ``max_local_blocks`` (run_poc.py:231-237)."""
    out = []
    for ks, vs in zip(k_shards, v_shards):
        packed = pack_local_kv(ks, vs)
        if packed.shape[0] < cfg.max_local_blocks:
            padded = torch.zeros((cfg.max_local_blocks, packed.shape[1]), dtype=packed.dtype)
            padded[: packed.shape[0]] = packed
            packed = padded
        out.append(packed)
    return out


def expected_rank_output(cfg: PCPAttentionConfig, q, k, v, rank: int) -> np.ndarray:
    """Oracle output of one rank: dense fp32 attention of its Q shard over the
    whole (dequantised) history."""
    oc = oracle_config(cfg)
    qn = to_numpy_f32(q)
    q_shard = orc.shard_query(qn, oc)[rank]
    return orc.dense_history_attention(q_shard, to_numpy_f32(k), to_numpy_f32(v), oc.softmax_scale)


def error_metrics(actual: torch.Tensor, expected: np.ndarray) -> dict:
    a = to_numpy_f32(actual).astype(np.float64)
    e = expected.astype(np.float64)
    diff = np.abs(a - e)
    return {
        "max_abs": float(diff.max()),
        "mean_abs": float(diff.mean()),
        "rel_l2": float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)),
        "norm_ratio": float(np.linalg.norm(a) / max(np.linalg.norm(e), 1e-30)),
        "finite": bool(np.isfinite(a).all()),
    }


def assert_parity(actual: torch.Tensor, expected: np.ndarray, label: str = "") -> dict:
    m = error_metrics(actual, expected)
    assert m["finite"], f"{label}: non-finite output"
    assert m["max_abs"] <= MAX_ABS, f"{label}: max-abs {m}"
    assert m["mean_abs"] <= MEAN_ABS, f"{label}: mean-abs {m}"
    assert m["rel_l2"] <= REL_L2, f"{label}: rel-L2 {m}"
    assert m["norm_ratio"] >= 0.25, f"{label}: output trivially small {m}"
    return m


def make_current(cfg: PCPAttentionConfig, seed: int, scale: float = 0.5):
    """Current (prefill) tokens' K/V in sequence order ``[Hkv, current_len, D]``
    bf16 (seeded N(0, scale^2)) and their striped per-rank shards (the
    ``shard_query`` layout)."""
    g = torch.Generator().manual_seed(seed + 7919)
    shape = (cfg.num_kv_heads, cfg.current_len, cfg.head_dim)
    k_cur = (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)
    v_cur = (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)
    pos = [global_positions_for_rank(cfg.current_len, r, cfg.pcp_size, cfg.interleave_size) for r in range(cfg.pcp_size)]
    return k_cur, v_cur, [k_cur[:, p].contiguous() for p in pos], [v_cur[:, p].contiguous() for p in pos]


def expected_prefill_output(cfg: PCPAttentionConfig, q, k, v, k_cur, v_cur, rank: int) -> np.ndarray:
    """Oracle prefill output of one rank: its Q shard over the whole history
    and, causally, the current tokens."""
    oc = oracle_config(cfg)
    q_shard = orc.shard_query(to_numpy_f32(q), oc)[rank]
    return orc.prefill_attention(q_shard, to_numpy_f32(k), to_numpy_f32(v), to_numpy_f32(k_cur),
                                 to_numpy_f32(v_cur), oc, rank)
