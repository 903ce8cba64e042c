"""CPU checks of the fp32 checker used by bench.py's parity record, run_poc's
check and the full-size GPU tests: it must equal the oracle's dense attention
(pinned to the reference) and rebuild the history from packed shards."""

from __future__ import annotations

import numpy as np
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.check import compare, dense_reference, history_from_packed, within_bounds
from oracle import pcp_oracle as orc

from parity import make_case, oracle_config, packed_shards, to_numpy_f32


def test_dense_reference_equals_oracle_in_chunks():
    cfg = PCPAttentionConfig(2, 256, 2048, 1500, 512, 64, 8, 2, 128)
    q, k, v, q_shards, _, _ = make_case(cfg, seed=5)
    oc = oracle_config(cfg)
    want = orc.dense_history_attention(to_numpy_f32(q_shards[1]), to_numpy_f32(k), to_numpy_f32(v), oc.softmax_scale)
    # A tiny score budget forces many row chunks, including a ragged last one.
    got = dense_reference(q_shards[1], k, v, cfg.softmax_scale, score_bytes=4 * 1500 * 37)
    assert np.abs(got.numpy() - want).max() < 2e-6


def test_history_from_packed_rebuilds_the_valid_tokens():
    cfg = PCPAttentionConfig(4, 256, 4096, 3001, 512, 64, 8, 2, 128)
    for kv_dtype in (torch.float8_e4m3fn, torch.bfloat16):
        _, k, v, _, k_shards, v_shards = make_case(cfg, seed=9, kv_dtype=kv_dtype)
        packed = packed_shards(cfg, k_shards, v_shards)
        valid = cfg.source_valid_lens()
        kk, vv = history_from_packed(cfg, packed, valid)
        assert kk.dtype == kv_dtype and tuple(kk.shape) == (cfg.num_kv_heads, sum(valid), cfg.head_dim)
        # Same multiset of tokens as the global history (order: shard by shard).
        kg = to_numpy_f32(k).reshape(-1, cfg.head_dim)
        kr = to_numpy_f32(kk).reshape(-1, cfg.head_dim)
        assert np.array_equal(np.sort(kg, axis=0), np.sort(kr, axis=0))
        vg = to_numpy_f32(v).reshape(-1, cfg.head_dim)
        vr = to_numpy_f32(vv).reshape(-1, cfg.head_dim)
        assert np.array_equal(np.sort(vg, axis=0), np.sort(vr, axis=0))


def test_compare_flags_a_zero_output():
    ref = torch.randn(4, 64, 128) * 1e-3
    assert within_bounds(compare(ref.to(torch.bfloat16), ref))
    assert not within_bounds(compare(torch.zeros_like(ref), ref))
