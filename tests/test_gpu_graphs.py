"""Length-bucket CUDA graphs on the GPU (needs a B200): lengths read on the
device inside a bucket give the same result as the host-planned call, a
recorded graph replays correctly for several lengths in its bucket, and a
length above its bucket is clamped and reported, not faulted."""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention
from aws_training_study_b200 import _capi
from aws_training_study_b200.pcp_attention.graphs import BucketedHistoryAttention, BucketGraph, bucket_for
from oracle import pcp_oracle as orc

from parity import assert_parity, make_case, oracle_config, packed_shards, to_numpy_f32

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CFG = PCPAttentionConfig(1, 1024, 8192, 8192, 512, 64, 32, 2, 256)


@pytest.fixture(scope="module")
def case():
    q, k, v, q_shards, k_shards, v_shards = make_case(CFG, seed=31)
    packed = packed_shards(CFG, k_shards, v_shards)[0].to(DEV)
    return q, k, v, q_shards[0].to(DEV), packed


def _expected(q, k, v, hist):
    oc = oracle_config(CFG)
    return orc.dense_history_attention(to_numpy_f32(q), to_numpy_f32(k[:, :hist]), to_numpy_f32(v[:, :hist]),
                                       oc.softmax_scale)


def test_device_lengths_equal_host_lengths_at_the_bound(case, kv_path):
    q, k, v, qd, packed = case
    attn = HistoryAttention(CFG, rank=0, device=0)
    for hist in (8192, 3000):
        vd = torch.tensor([hist], dtype=torch.int32, device=DEV)
        a = attn.forward_bucketed(qd, packed, vd, [hist])
        b = attn(qd, packed, [hist])
        attn.status()
        assert torch.equal(a, b), hist
    attn.close()


def test_device_lengths_below_the_bound(case, kv_path):
    q, k, v, qd, packed = case
    attn = HistoryAttention(CFG, rank=0, device=0)
    for hist in (1, 700, 4096, 6145):
        vd = torch.tensor([hist], dtype=torch.int32, device=DEV)
        out = attn.forward_bucketed(qd, packed, vd, [8192])
        attn.status()
        assert_parity(out, _expected(q, k, v, hist), f"bucket 8192 len {hist}")
    attn.close()


def test_graph_replays_every_length_in_its_bucket(case, kv_path):
    q, k, v, qd, packed = case
    attn = HistoryAttention(CFG, rank=0, device=0)
    g = BucketGraph(attn, [6144], qd, packed)
    for hist in (6144, 5000, 4097, 333):
        out = g.replay([hist]).clone()
        attn.status()
        assert_parity(out, _expected(q, k, v, hist), f"graph len {hist}")
        eager = attn.forward_bucketed(qd, packed, torch.tensor([hist], dtype=torch.int32, device=DEV), [6144])
        attn.status()
        assert torch.equal(out, eager)
    attn.close()
    assert g.graph is None  # released with the handle


def test_bucketed_wrapper_records_one_graph_per_bucket(case, kv_path):
    q, k, v, qd, packed = case
    attn = HistoryAttention(CFG, rank=0, device=0)
    b = BucketedHistoryAttention(attn, qd, packed, granularity_blocks=4)
    for hist in (1000, 2048, 2049, 8192):
        out = b([hist])
        attn.status()
        assert_parity(out, _expected(q, k, v, hist), f"bucketed len {hist}")
    assert sorted(b.graphs) == [(2048,), (4096,), (8192,)]
    assert bucket_for(CFG, [1000], 4) == (2048,)
    b.close()
    attn.close()


def test_length_above_bucket_is_reported(case, kv_path):
    q, k, v, qd, packed = case
    attn = HistoryAttention(CFG, rank=0, device=0)
    vd = torch.tensor([5000], dtype=torch.int32, device=DEV)
    attn.forward_bucketed(qd, packed, vd, [4096])
    with pytest.raises(_capi.PcpError, match="code 110"):
        attn.status()
    attn.close()


def test_device_lengths_at_head_dim_128(kv_path):
    """Device-length mode through the head-dim-128 kernels (the two-query-tile
    ping-pong kernel on the dense path, the in-place kernel otherwise):
    lengths below the bound and a recorded graph replayed inside it."""
    cfg = PCPAttentionConfig(1, 1024, 8192, 8192, 512, 64, 16, 4, 128)
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=37)
    qd, packed = q_shards[0].to(DEV), packed_shards(cfg, k_shards, v_shards)[0].to(DEV)
    oc = oracle_config(cfg)

    def expected(hist):
        return orc.dense_history_attention(to_numpy_f32(q), to_numpy_f32(k[:, :hist]), to_numpy_f32(v[:, :hist]),
                                           oc.softmax_scale)

    attn = HistoryAttention(cfg, rank=0, device=0)
    for hist in (1, 2000, 8192):
        out = attn.forward_bucketed(qd, packed, torch.tensor([hist], dtype=torch.int32, device=DEV), [8192])
        attn.status()
        assert_parity(out, expected(hist), f"d128 bucket 8192 len {hist}")
    g = BucketGraph(attn, [4096], qd, packed)
    for hist in (4096, 2500):
        out = g.replay([hist]).clone()
        attn.status()
        assert_parity(out, expected(hist), f"d128 graph len {hist}")
    attn.close()
