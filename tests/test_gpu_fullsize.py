"""Parity at BASELINE sizes over EVERY output row (needs a B200).

The CUDA path runs the whole single-GPU workload; every query row of every
head is compared with the reference's dense attention restated in torch fp32
(``pcp_attention.check.dense_reference``: softmax(q K^T / sqrt(D)) V over the
full dequantised history, TF32 off, chunked over rows), computed on the GPU
because the CPU oracle would take minutes at these sizes.  Same bounds as
tests/parity.py.
"""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.check import compare, dense_reference, history_from_packed
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
from aws_training_study_b200.pcp_attention.inputs import make_local_baseline_inputs

from parity import MAX_ABS, MEAN_ABS, REL_L2

pytestmark = pytest.mark.gpu


def _check(cfg: PCPAttentionConfig, kv_dtype, outliers: float) -> dict:
    dev = torch.device("cuda", 0)
    q, packed = make_local_baseline_inputs(cfg, 77, 0, kv_dtype=kv_dtype, outlier_frac=outliers, device=dev)
    attn = HistoryAttention(cfg, kv_dtype=kv_dtype, rank=0, device=0)
    out = attn(q, packed, [cfg.actual_history_len])
    attn.status()
    attn.close()
    k, v = history_from_packed(cfg, [packed], [cfg.actual_history_len])
    ref = dense_reference(q, k, v, cfg.softmax_scale)
    m = compare(out, ref)
    # Per head as well: a fault confined to some units must not hide in the total.
    for h in range(cfg.num_q_heads):
        mh = compare(out[h], ref[h])
        assert mh["finite"] and mh["rel_l2"] <= REL_L2 and mh["norm_ratio"] >= 0.25, (h, mh)
    assert m["finite"], m
    assert m["max_abs"] <= MAX_ABS and m["mean_abs"] <= MEAN_ABS and m["rel_l2"] <= REL_L2, m
    assert m["norm_ratio"] >= 0.25, m
    return m


def test_configs3_qwen_full_history_fp8(kv_path):
    """BASELINE configs[3] at one GPU: 32/2 heads, D=256, Q=4096, 131072 history."""
    _check(PCPAttentionConfig(1, 4096, 131072, 131072, 512, 64, 32, 2, 256), torch.float8_e4m3fn, 0.0)


def test_configs4_long_gqa_outliers_unaligned(kv_path):
    """BASELINE configs[4] shape at one GPU: 64/8 heads, D=128, Q=8192,
    500000 of 524288 history tokens, 1 % of K/V entries x8."""
    _check(PCPAttentionConfig(1, 8192, 524288, 500000, 512, 64, 64, 8, 128), torch.float8_e4m3fn, 0.01)


def test_configs2_bf16_masked_full():
    """BASELINE configs[2] shape at one GPU: BF16 K/V, 30001 of 32768 history."""
    _check(PCPAttentionConfig(1, 2048, 32768, 30001, 512, 64, 32, 2, 256), torch.bfloat16, 0.0)
