"""Parity at BASELINE sizes (needs a B200).

The CUDA path runs the whole single-GPU workload; sampled query rows of
sampled heads are compared with a plain torch fp32 reference of the same op
(softmax(q K^T / sqrt(D)) V over the full dequantised history, TF32 off),
computed on the GPU because the CPU oracle would take minutes at these
sizes.  Same bounds as tests/parity.py.
"""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
from aws_training_study_b200.pcp_attention.inputs import make_local_baseline_inputs

from parity import MAX_ABS, MEAN_ABS, REL_L2

pytestmark = pytest.mark.gpu


def _dense_rows(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        s = torch.matmul(q_rows.float(), k.float().T) * scale
        return torch.matmul(torch.softmax(s, dim=-1), v.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _check(cfg: PCPAttentionConfig, kv_dtype, outliers: float, heads, row_starts, nrows=256):
    dev = torch.device("cuda", 0)
    q, packed = make_local_baseline_inputs(cfg, 77, 0, kv_dtype=kv_dtype, outlier_frac=outliers, device=dev)
    attn = HistoryAttention(cfg, kv_dtype=kv_dtype, rank=0, device=0)
    out = attn(q, packed, [cfg.actual_history_len])
    attn.status()
    A = cfg.actual_history_len
    blk = packed.view(torch.uint8) if kv_dtype == torch.float8_e4m3fn else packed
    blk = blk.reshape(cfg.max_local_blocks, 2, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    if kv_dtype == torch.float8_e4m3fn:
        blk = blk.view(torch.float8_e4m3fn)
    group = cfg.q_heads_per_kv_head
    worst = {"max_abs": 0.0, "mean_abs": 0.0, "rel_l2": 0.0}
    for h in heads:
        g = h // group
        k = blk[:, 0, g].reshape(-1, cfg.head_dim)[:A]
        v = blk[:, 1, g].reshape(-1, cfg.head_dim)[:A]
        for r0 in row_starts:
            ref = _dense_rows(q[h, r0 : r0 + nrows], k, v, cfg.softmax_scale)
            got = out[h, r0 : r0 + nrows].float()
            assert torch.isfinite(got).all()
            d = (got - ref).abs()
            rel = (torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref)).item()
            worst["max_abs"] = max(worst["max_abs"], d.max().item())
            worst["mean_abs"] = max(worst["mean_abs"], d.mean().item())
            worst["rel_l2"] = max(worst["rel_l2"], rel)
            assert torch.linalg.vector_norm(got) >= 0.25 * torch.linalg.vector_norm(ref)
    attn.close()
    assert worst["max_abs"] <= MAX_ABS and worst["mean_abs"] <= MEAN_ABS and worst["rel_l2"] <= REL_L2, worst
    return worst


def test_configs3_qwen_full_history_fp8():
    """BASELINE configs[3] at one GPU: 32/2 heads, D=256, Q=4096, 131072 history."""
    cfg = PCPAttentionConfig(1, 4096, 131072, 131072, 512, 64, 32, 2, 256)
    _check(cfg, torch.float8_e4m3fn, 0.0, heads=(0, 17, 31), row_starts=(0, 2048, 3840))


def test_configs4_long_gqa_outliers_unaligned():
    """BASELINE configs[4] shape at one GPU: 64/8 heads, D=128, Q=8192,
    500000 of 524288 history tokens, 1 % of K/V entries x8."""
    cfg = PCPAttentionConfig(1, 8192, 524288, 500000, 512, 64, 64, 8, 128)
    _check(cfg, torch.float8_e4m3fn, 0.01, heads=(0, 9, 63), row_starts=(0, 8192 - 256))


def test_configs2_bf16_masked_full():
    """BASELINE configs[2] shape at one GPU: BF16 K/V, 30001 of 32768 history."""
    cfg = PCPAttentionConfig(1, 2048, 32768, 30001, 512, 64, 32, 2, 256)
    _check(cfg, torch.bfloat16, 0.0, heads=(0, 31), row_starts=(0, 1792))
