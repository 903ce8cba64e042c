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


def _ring_body(rank, world, name, exchange="direct", kv_path=None):
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
    attn = HistoryAttention(cfg, kv_dtype=kv_dtype, rank=rank, device=rank, exchange=exchange, kv_path=kv_path)
    qd, kvd = q_shards[rank].cuda(), packed[rank].cuda()
    for _ in range(3):  # repeated calls reuse the ring buffers
        out = attn(qd, kvd)
    attn.status(120000)
    st = attn.stats()
    assert kv_path is None or st["kv_in_place"] == (kv_path == "in_place")
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


def ring_qwen_pipeline(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8", exchange="pipeline")


# The e4m3 cache read in place from the receive slots (pcp_set_kv_path).
def ring_qwen_inplace(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8", kv_path="in_place")


def ring_qwen_storeforward_inplace(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8", exchange="ring", kv_path="in_place")


def ring_qwen_pipeline_inplace(rank, world):
    return _ring_body(rank, world, "qwen_d256_fp8", exchange="pipeline", kv_path="in_place")


def prefill_ragged(rank, world):
    """History plus causal current tokens through the handle: the current
    K/V shards are all-gathered inside the C ABI."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from parity import assert_parity, expected_prefill_output, make_case, make_current, packed_shards

    P, cur, mh, ah, bs, I, hq, hkv, d, kv = CASES["ragged_d128_bf16"]
    cfg = PCPAttentionConfig(P, cur, mh, ah, bs, I, hq, hkv, d).validate()
    torch.cuda.set_device(rank)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=13, kv_dtype=torch.bfloat16)
    k_cur, v_cur, kc_shards, vc_shards = make_current(cfg, seed=13)
    packed = packed_shards(cfg, k_shards, v_shards)
    attn = HistoryAttention(cfg, kv_dtype=torch.bfloat16, rank=rank, device=rank)
    qd, kvd = q_shards[rank].cuda(), packed[rank].cuda()
    kcd, vcd = kc_shards[rank].cuda(), vc_shards[rank].cuda()
    for _ in range(2):
        out = attn.prefill(qd, kvd, kcd, vcd)
    attn.status(120000)
    st = attn.stats()
    m = assert_parity(out, expected_prefill_output(cfg, q, k, v, k_cur, v_cur, rank), f"prefill rank {rank}")
    attn.close()
    return {"metrics": m, "ring_bytes": st["ring_bytes"], "attn_launches": st["attn_launches"]}


def ring_paged(rank, world, kv_path=None):
    """Each rank's cache written by the GPU producer into a pool through a
    permuted block table, then attended through the handle's paged entry
    (its live blocks are gathered before the exchange)."""
    import sys
    from pathlib import Path

    import numpy as np

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from aws_training_study_b200.pcp_attention.paged import cache_write, make_pool
    from oracle import pcp_oracle as orc
    from parity import assert_parity, oracle_config, to_numpy_f32

    P, cur, mh, ah, bs, I, hq, hkv, d, kv = CASES["qwen_d256_fp8"]
    ah = 7000  # ragged: the ranks hold different block counts
    cfg = PCPAttentionConfig(P, cur, mh, ah, bs, I, hq, hkv, d).validate()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    g = torch.Generator().manual_seed(17)
    q = torch.randn(hq, cur, d, generator=g).to(torch.bfloat16)
    k = (torch.randn(hkv, ah, d, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(hkv, ah, d, generator=g) * 0.5).to(torch.bfloat16)
    nb = cfg.max_local_blocks
    table = torch.from_numpy(np.random.default_rng(rank).permutation(nb + 4)[:nb].astype(np.int32)).to(dev)
    pool = make_pool(cfg, nb + 4, torch.float8_e4m3fn, dev)
    st = cache_write(cfg, rank, 0, k.to(dev), v.to(dev), table, pool)
    assert int(st.item()) == 0
    oc = oracle_config(cfg)
    q_shard = torch.from_numpy(orc.shard_query(to_numpy_f32(q), oc)[rank]).to(torch.bfloat16).to(dev)
    attn = HistoryAttention(cfg, rank=rank, device=rank, kv_path=kv_path)
    for _ in range(2):
        out = attn.forward_paged(q_shard, pool, table)
    attn.status(120000)
    stats = attn.stats()
    kq = orc.e4m3fn_decode(orc.e4m3fn_encode(to_numpy_f32(k)))
    vq = orc.e4m3fn_decode(orc.e4m3fn_encode(to_numpy_f32(v)))
    want = orc.dense_history_attention(to_numpy_f32(q_shard), kq, vq, oc.softmax_scale)
    m = assert_parity(out, want, f"paged rank {rank}")
    attn.close()
    return {"metrics": m, "ring_bytes": stats["ring_bytes"], "attn_launches": stats["attn_launches"]}


def ring_graph(rank, world, kv_path=None):
    """A length-bucket CUDA graph that records the NCCL exchange, replayed
    for several history lengths inside its bucket."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from aws_training_study_b200.pcp_attention.graphs import BucketGraph, bucket_for
    from oracle import pcp_oracle as orc
    from parity import assert_parity, make_case, oracle_config, packed_shards, to_numpy_f32

    P, cur, mh, ah, bs, I, hq, hkv, d, kv = CASES["qwen_d256_fp8"]
    cfg = PCPAttentionConfig(P, cur, mh, ah, bs, I, hq, hkv, d).validate()
    torch.cuda.set_device(rank)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=19)
    packed = packed_shards(cfg, k_shards, v_shards)
    attn = HistoryAttention(cfg, rank=rank, device=rank, kv_path=kv_path)
    qd, kvd = q_shards[rank].cuda(), packed[rank].cuda()
    lens = {h: [orc.source_valid_len(h, P, I, s) for s in range(P)] for h in (6000, 5121, 4100)}
    bucket = bucket_for(cfg, lens[6000], granularity_blocks=2)
    g = BucketGraph(attn, bucket, qd, kvd)
    oc = oracle_config(cfg)
    q_shard = orc.shard_query(to_numpy_f32(q), oc)[rank]
    worst = {}
    for hist, vl in lens.items():
        out = g.replay(vl).clone()
        attn.status(120000)
        want = orc.dense_history_attention(q_shard, to_numpy_f32(k[:, :hist]), to_numpy_f32(v[:, :hist]),
                                           oc.softmax_scale)
        worst[hist] = assert_parity(out, want, f"graph rank {rank} hist {hist}")
    stats = attn.stats()
    attn.close()
    return {"metrics": worst, "ring_bytes": stats["ring_bytes"], "attn_launches": stats["attn_launches"]}


def ring_host_async(rank, world):
    """The serving-loop host entry at two ranks: pinned host inputs, several
    asynchronous steps, every output against the oracle."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
    from parity import assert_parity, expected_rank_output, make_case, packed_shards

    P, cur, mh, ah, bs, I, hq, hkv, d, kv = CASES["qwen_d256_fp8"]
    cfg = PCPAttentionConfig(P, cur, mh, ah, bs, I, hq, hkv, d).validate()
    torch.cuda.set_device(rank)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=29)
    packed = packed_shards(cfg, k_shards, v_shards)
    attn = HistoryAttention(cfg, rank=rank, device=rank)
    qh = q_shards[rank].pin_memory()
    kvh = packed[rank].view(torch.uint8).pin_memory().view(packed[rank].dtype)
    outs = [torch.empty_like(qh).pin_memory() for _ in range(4)]
    for o in outs:
        attn.forward_host_async(qh, kvh, out=o)
    attn.forward_host_wait()
    attn.status(120000)
    want = expected_rank_output(cfg, q, k, v, rank)
    m = [assert_parity(o, want, f"host async rank {rank} step {i}") for i, o in enumerate(outs)]
    st = attn.stats()
    attn.close()
    return {"metrics": m, "ring_bytes": st["ring_bytes"], "attn_launches": st["attn_launches"]}


def ring_paged_inplace(rank, world):
    return ring_paged(rank, world, kv_path="in_place")


def ring_graph_inplace(rank, world):
    return ring_graph(rank, world, kv_path="in_place")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fn", ["ring_qwen", "ring_ragged", "ring_qwen_storeforward", "ring_ragged_allgather",
                                "prefill_ragged", "ring_paged", "ring_graph", "ring_qwen_pipeline",
                                "ring_qwen_inplace", "ring_qwen_storeforward_inplace", "ring_qwen_pipeline_inplace",
                                "ring_paged_inplace", "ring_graph_inplace", "ring_host_async"])
def test_two_rank_ring_matches_oracle(fn):
    res = run_ranks("test_gpu_ring", fn, 2, timeout=600, backend="gloo", env={"NCCL_NVLS_ENABLE": "0"})
    assert len(res) == 2, res
    for rank, (status, payload) in res.items():
        assert status == "ok", payload
        # local shard, remote shard (+ the causal current-token launch)
        assert payload["ring_bytes"] > 0 and payload["attn_launches"] == (3 if fn == "prefill_ragged" else 2)
