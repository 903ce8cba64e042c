"""CUDA path vs the CPU oracle on the same seeded inputs (needs a B200).

Each case builds global Q/K/V, shards them with the product layout, runs the
CUDA path for one or more ranks and compares each rank's bf16 output with the
oracle's fp32 dense attention of that rank's Q shard over the whole history
(``oracle.pcp_oracle.dense_history_attention``, pinned to the reference's
``dense_history_attention`` by tests/test_oracle_golden.py).  Bounds are in
tests/parity.py.
"""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention, history_attention_single

from parity import assert_parity, expected_rank_output, make_case, packed_shards

pytestmark = pytest.mark.gpu


def _run_gathered(cfg, q_shards, packed, rank, kv_dtype):
    """What one rank computes after the ring: its Q shard against every
    source's shard, through the stateless C-ABI entry."""
    dev = torch.device("cuda", 0)
    allkv = torch.cat([packed[(rank - s) % cfg.pcp_size] for s in range(cfg.pcp_size)]).to(dev)
    valid = [cfg.source_valid_len((rank - s) % cfg.pcp_size) for s in range(cfg.pcp_size)]
    return history_attention_single(q_shards[rank].to(dev), allkv, valid, cfg, kv_dtype=kv_dtype)


CASES = [
    # name, config, kv dtype, ranks to check
    ("ref_tiny_d128", PCPAttentionConfig(4, 256, 2048, 2048, 512, 64, 4, 2, 128), torch.float8_e4m3fn, [0, 3]),
    ("qwen_small_d256", PCPAttentionConfig(8, 1024, 8192, 8192, 512, 64, 32, 2, 256), torch.float8_e4m3fn, [0, 5]),
    ("masked_bf16_d256", PCPAttentionConfig(8, 2048, 32768, 30001, 512, 64, 32, 2, 256), torch.bfloat16, [0, 4, 7]),
    ("gqa8_d128_ragged", PCPAttentionConfig(4, 1024, 8192, 5000, 512, 64, 16, 4, 128), torch.float8_e4m3fn, [0, 2]),
    # multi-head (no GQA), the official-ring benchmark's shape at small size
    ("mha_d128_bf16", PCPAttentionConfig(2, 1024, 2048, 2048, 512, 64, 8, 8, 128), torch.bfloat16, [0, 1]),
    # BASELINE configs[0]'s shape (64-token blocks): in place, the two 64-key
    # halves of a V tile come from two cache blocks
    ("cfg1_bs64_d128", PCPAttentionConfig(4, 256, 1024, 1024, 64, 16, 8, 2, 128), torch.float8_e4m3fn, [0, 3]),
    # ragged sources with 64-token blocks: partial key tiles at every source,
    # some of them one key half only
    ("ragged_bs64_d256", PCPAttentionConfig(4, 256, 2048, 1001, 64, 16, 8, 2, 256), torch.float8_e4m3fn,
     [0, 1, 2, 3]),
    # an e4m3 block size that is no multiple of 64: the dense unpack path
    ("e4m3_bs32_unpack", PCPAttentionConfig(2, 256, 1024, 1000, 32, 16, 8, 2, 128), torch.float8_e4m3fn, [0, 1]),
]


@pytest.mark.parametrize("name,cfg,kv_dtype,ranks", CASES, ids=[c[0] for c in CASES])
def test_rank_matches_oracle(name, cfg, kv_dtype, ranks, kv_path):
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=1234, kv_dtype=kv_dtype)
    packed = packed_shards(cfg, k_shards, v_shards)
    for rank in ranks:
        out = _run_gathered(cfg, q_shards, packed, rank, kv_dtype)
        assert_parity(out, expected_rank_output(cfg, q, k, v, rank), f"{name} rank {rank}")


def test_single_rank_handle_direct_output(kv_path):
    """P = 1 through the handle: one stream-K attention launch writes every
    unit one segment covers as bf16 output; the combine merges the rest."""
    cfg = PCPAttentionConfig(1, 1024, 4096, 4096, 512, 64, 32, 2, 256)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=7)
    packed = packed_shards(cfg, k_shards, v_shards)[0].cuda()
    attn = HistoryAttention(cfg, rank=0, device=0)
    out = attn(q_shards[0].cuda(), packed)
    attn.status()
    st = attn.stats()
    # unpack (dense path only), attention, combine
    assert st["attn_launches"] == 1 and st["kernel_launches"] <= (2 if kv_path == "in_place" else 3)
    assert st["kv_in_place"] == (kv_path == "in_place")
    assert_parity(out, expected_rank_output(cfg, q, k, v, 0), "p1 direct")
    attn.close()


def test_bounded_wait_reports_timeout():
    """A device wait that nothing satisfies gives up by itself and reports
    its error code; the context stays usable afterwards."""
    import ctypes

    from aws_training_study_b200 import _capi

    status = ctypes.c_int32(-1)
    _capi.check(_capi.lib().pcp_selftest_bounded_wait(2000, ctypes.byref(status)))
    assert status.value == 199
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0
