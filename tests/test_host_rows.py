"""Host-side logic of the prefill, paged-cache and bucket APIs, on the CPU:
stripe arithmetic against the oracle, and argument checks that must reject
bad calls before any device work."""

from __future__ import annotations

import random

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import prefill_attention_single
from aws_training_study_b200.pcp_attention.paged import cache_write, config_source_len, local_blocks_needed
from oracle import pcp_oracle as orc


def test_owned_positions_match_the_oracle():
    rng = random.Random(3)
    for _ in range(300):
        P = rng.randint(1, 9)
        I = rng.choice([1, 8, 16, 64])
        cfg = PCPAttentionConfig(P, P * I, P * I * 64, P * I * 64, I * 8, I, 4, 2, 128)
        total = rng.randint(0, P * I * 64)
        for r in range(P):
            assert config_source_len(cfg, r, total) == orc.source_valid_len(total, P, I, r)
            assert local_blocks_needed(cfg, r, total) == -(-orc.source_valid_len(total, P, I, r) // cfg.block_size)


CFG = PCPAttentionConfig(2, 256, 2048, 2048, 512, 64, 4, 2, 128)


def _cpu(*shape, dtype=torch.bfloat16):
    return torch.zeros(shape, dtype=dtype)


def test_prefill_rejects_bad_shapes_before_device_work():
    q = _cpu(4, 128, 128)
    kc = _cpu(2, 2, 128, 128)
    with pytest.raises(ValueError):  # CPU tensors
        prefill_attention_single(q, None, [], kc, kc, CFG, 0)
    with pytest.raises(ValueError):  # history lengths without a history
        prefill_attention_single(q, None, [5, 0], kc, kc, CFG, 0)
    with pytest.raises(ValueError):  # current K/V without the rank axis
        prefill_attention_single(q, None, [], kc[0], kc[0], CFG, 0)


def test_cache_write_rejects_bad_arguments_before_device_work():
    pool = _cpu(4, 2 * 2 * 512 * 128, dtype=torch.float8_e4m3fn)
    table = torch.zeros(4, dtype=torch.int32)
    k = _cpu(2, 100, 128)
    with pytest.raises(ValueError):  # pool on the CPU
        cache_write(CFG, 0, 0, k, k, table, pool)
    with pytest.raises(ValueError):  # wrong payload width
        cache_write(CFG, 0, 0, k, k, table, _cpu(4, 7, dtype=torch.float8_e4m3fn))
    with pytest.raises(ValueError):  # K/V not [Hkv, T, D] bf16
        cache_write(CFG, 0, 0, _cpu(2, 100, 64), k, table, pool)
