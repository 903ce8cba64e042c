"""The multi-GPU path: one process per GPU, the NCCL send/recv ring inside
the C ABI, each rank's bf16 output compared with the oracle (needs 2 GPUs;
skipped on a 1-GPU box).  NVLS is off in these tests."""

from __future__ import annotations

import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu

CASES = {
    # P, current, max hist, actual hist, bs, I, Hq, Hkv, D, kv dtype
    "qwen_d256_fp8": (2, 512, 8192, 8192, 512, 64, 32, 2, 256, "e4m3"),
    "ragged_d128_bf16": (2, 512, 8192, 6001, 512, 64, 16, 4, 128, "bf16"),
}


def _ring_body(rank, world, name, exchange="direct"):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from parity import assert_parity, expected_rank_output, make_case, packed_shards

    P, cur, mh, ah, bs, I, hq, hkv, d, kv = CASES[name]
    cfg = PCPAttentionConfig(P, cur, mh, ah, bs, I, hq, hkv, d).validate()
    kv_dtype = torch.float8_e4m3fn if kv == "e4m3" else torch.bfloat16
    torch.cuda.set_device(rank)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=11, kv_dtype=kv_dtype)
    packed = packed_shards(cfg, k_shards, v_shards)
    attn = HistoryAttention(cfg, kv_dtype=kv_dtype, rank=rank, device=rank, exchange=exchange)
    qd, kvd = q_shards[rank].cuda(), packed[rank].cuda()
    for _ in range(3):  # repeated calls reuse the ring buffers
        out = attn(qd, kvd)
    attn.status(120000)
    st = attn.stats()
    m = assert_parity(out, expected_rank_output(cfg, q, k, v, rank), f"{name} rank {rank}")
    attn.close()
    return {"metrics": m, "ring_bytes": st["ring_bytes"], "attn_launches": st["attn_launches"]}


def ring_qwen(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8")


def ring_ragged(rank, world):
    return _ring_body(rank, world, "ragged_d128_bf16")


def ring_qwen_storeforward(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8", exchange="ring")


def ring_ragged_allgather(rank, world):
    return _ring_body(rank, world, "ragged_d128_bf16", exchange="allgather")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fn", ["ring_qwen", "ring_ragged", "ring_qwen_storeforward", "ring_ragged_allgather"])
def test_two_rank_ring_matches_oracle(fn):
    res = run_ranks("test_gpu_ring", fn, 2, timeout=600, backend="gloo", env={"NCCL_NVLS_ENABLE": "0"})
    assert len(res) == 2, res
    for rank, (status, payload) in res.items():
        assert status == "ok", payload
        assert payload["ring_bytes"] > 0 and payload["attn_launches"] == 2
