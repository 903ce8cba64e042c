"""The exchange paths that only exist at 4+ ranks (needs 4 or more GPUs;
skipped otherwise): the local shard attended on a grid that leaves SMs to
NCCL with one exchange group, the two-group fallback (comm_sms 0, a local
launch that fills the GPU), and the pipelined exchange with one group per
ring step.  Every rank's output against the oracle.  NVLS is off."""

from __future__ import annotations

import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu

WORLD = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0

# (world) -> current, max hist, actual hist, bs, I, Hq, Hkv, D
SHAPES = {
    # local shard small (fits L2): SM reservation for the exchange
    "small": lambda world: (1024, 8192, 8192, 512, 64, 32, 2, 256),
    # Qloc 1024 with 32/2 heads = 128 units of 256 rows: the wave-scheduled
    # local launch fills the 74 SM pairs, so without reservation the peers
    # go in two groups
    "fill": lambda world: (1024 * world, 8192, 8192, 512, 64, 32, 2, 256),
}


def _body(rank, world, shape, exchange, comm_sms):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from parity import assert_parity, expected_rank_output, make_case, packed_shards

    cur, mh, ah, bs, I, hq, hkv, d = SHAPES[shape](world)
    cfg = PCPAttentionConfig(world, cur, mh, ah, bs, I, hq, hkv, d).validate()
    torch.cuda.set_device(rank)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=23)
    packed = packed_shards(cfg, k_shards, v_shards)
    attn = HistoryAttention(cfg, rank=rank, device=rank, exchange=exchange, comm_sms=comm_sms)
    qd, kvd = q_shards[rank].cuda(), packed[rank].cuda()
    for _ in range(2):
        out = attn(qd, kvd)
    attn.status(120000)
    st = attn.stats()
    m = None
    if rank in (0, world - 1):  # the oracle is CPU work: two ranks are enough
        m = assert_parity(out, expected_rank_output(cfg, q, k, v, rank), f"{shape}/{exchange} rank {rank}")
    attn.close()
    return {"metrics": m, "attn_launches": st["attn_launches"]}


def small_direct_reserved(rank, world):
    return _body(rank, world, "small", "direct", 16)


def fill_direct_two_groups(rank, world):
    return _body(rank, world, "fill", "direct", 0)


def small_pipeline(rank, world):
    return _body(rank, world, "small", "pipeline", 16)


@pytest.mark.skipif(WORLD < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("fn,launches", [("small_direct_reserved", 2), ("fill_direct_two_groups", 3),
                                         ("small_pipeline", None)])
def test_wide_exchange_matches_oracle(fn, launches):
    res = run_ranks("test_gpu_ring_wide", fn, WORLD, timeout=900, backend="gloo", env={"NCCL_NVLS_ENABLE": "0"})
    assert len(res) == WORLD, res
    for rank, (status, payload) in res.items():
        assert status == "ok", payload
        expected = launches if launches is not None else min(WORLD, 8)  # local + one launch per step chunk
        assert payload["attn_launches"] == expected, (rank, payload)
