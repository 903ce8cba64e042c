"""Prefill on the GPU: history attention plus causal attention over the
current tokens of every rank, merged by log-sum-exp, against the oracle's
``prefill_attention`` (needs a B200).  Bounds are in tests/parity.py."""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention, prefill_attention_single

from parity import assert_parity, expected_prefill_output, make_case, make_current, packed_shards

pytestmark = pytest.mark.gpu

CASES = [
    # name, config, kv dtype, ranks to check
    ("qwen_d256_p1", PCPAttentionConfig(1, 1024, 4096, 4096, 512, 64, 32, 2, 256), torch.float8_e4m3fn, [0]),
    ("gqa_d128_p4_ragged", PCPAttentionConfig(4, 1024, 8192, 5000, 512, 64, 16, 4, 128), torch.float8_e4m3fn,
     [0, 3]),
    # Qloc 192: 256-row pair tiles wrap from one Q head into the next
    ("wrap_d256_p2_bf16", PCPAttentionConfig(2, 384, 2048, 1000, 512, 64, 8, 2, 256), torch.bfloat16, [0, 1]),
    ("mha_d128_p2", PCPAttentionConfig(2, 1024, 2048, 2048, 512, 64, 8, 8, 128), torch.bfloat16, [1]),
]


def _stateless(cfg, q_shards, packed, kc_shards, vc_shards, rank, kv_dtype, with_history=True):
    dev = torch.device("cuda", 0)
    kc_all = torch.stack(kc_shards).contiguous().to(dev)
    vc_all = torch.stack(vc_shards).contiguous().to(dev)
    if not with_history:
        return prefill_attention_single(q_shards[rank].to(dev), None, [], kc_all, vc_all, cfg, rank)
    allkv = torch.cat([packed[(rank - s) % cfg.pcp_size] for s in range(cfg.pcp_size)]).to(dev)
    valid = [cfg.source_valid_len((rank - s) % cfg.pcp_size) for s in range(cfg.pcp_size)]
    return prefill_attention_single(q_shards[rank].to(dev), allkv, valid, kc_all, vc_all, cfg, rank, kv_dtype)


@pytest.mark.parametrize("name,cfg,kv_dtype,ranks", CASES, ids=[c[0] for c in CASES])
def test_prefill_matches_oracle(name, cfg, kv_dtype, ranks, kv_path):
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=21, kv_dtype=kv_dtype)
    k_cur, v_cur, kc_shards, vc_shards = make_current(cfg, seed=21)
    packed = packed_shards(cfg, k_shards, v_shards)
    for rank in ranks:
        out = _stateless(cfg, q_shards, packed, kc_shards, vc_shards, rank, kv_dtype)
        assert_parity(out, expected_prefill_output(cfg, q, k, v, k_cur, v_cur, rank), f"{name} rank {rank}")


def test_causal_only_without_history():
    """No history tokens: a plain causal prefill over the striped sequence."""
    cfg = PCPAttentionConfig(4, 2048, 2048, 2048, 512, 64, 16, 2, 128)
    q, k, v, q_shards, _, _ = make_case(cfg, seed=5)
    k_cur, v_cur, kc_shards, vc_shards = make_current(cfg, seed=5)
    for rank in (0, 2):
        out = _stateless(cfg, q_shards, None, kc_shards, vc_shards, rank, None, with_history=False)
        assert_parity(out, expected_prefill_output(cfg, q, k[:, :0], v[:, :0], k_cur, v_cur, rank),
                      f"causal-only rank {rank}")


def test_handle_prefill_single_rank(kv_path):
    cfg = CASES[0][1]
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=8)
    k_cur, v_cur, kc_shards, vc_shards = make_current(cfg, seed=8)
    packed = packed_shards(cfg, k_shards, v_shards)[0].cuda()
    attn = HistoryAttention(cfg, rank=0, device=0)
    out = attn.prefill(q_shards[0].cuda(), packed, kc_shards[0].cuda(), vc_shards[0].cuda())
    attn.status()
    st = attn.stats()
    assert st["attn_launches"] == 2 and st["splits"] >= 2
    assert_parity(out, expected_prefill_output(cfg, q, k, v, k_cur, v_cur, 0), "handle prefill")
    # the plain forward on the same handle is unaffected
    plain = attn(q_shards[0].cuda(), packed)
    attn.status()
    assert attn.stats()["attn_launches"] == 1
    assert not torch.equal(plain, out)
    attn.close()
