"""Multi-rank host logic on CPU ranks (gloo, world size 2 and 3): the ring
schedule exported by the C ABI moves every shard to every rank with the
byte counts the CUDA path uses, the per-rank result equals the oracle, and
configuration mismatches or a missing rank surface as host exceptions before
any device ring starts."""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist

from mp_util import run_ranks


# -------------------------------------------------------------- rank bodies --
def _ring_cfg(world):
    from aws_training_study_b200.pcp_attention import PCPAttentionConfig

    # ragged history so the ranks hold different numbers of live blocks
    return PCPAttentionConfig(world, 64 * world, 64 * 16 * world, 64 * 9 * world + 37, 64, 16, 4, 2, 32).validate()


def ring_exchange_body(rank, world):
    """Move the packed shards with the C-ABI schedule over gloo and compute
    this rank's result with the oracle from what arrived."""
    from aws_training_study_b200 import _capi
    from aws_training_study_b200.pcp_attention import pack_local_kv, shard_history, shard_query
    from oracle import pcp_oracle as orc

    cfg = _ring_cfg(world)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=g)
    k = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g)
    v = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g)
    ks, vs = shard_history(k, v, cfg)
    payload = 2 * cfg.num_kv_heads * cfg.block_size * cfg.head_dim
    valid = cfg.source_valid_lens()
    mine = pack_local_kv(ks[rank], vs[rank])  # [blocks, payload] fp32
    have = {rank: mine}
    lib = _capi.lib()
    for hop in range(1, world):
        ss, rs, to, frm = (ctypes.c_int32() for _ in range(4))
        _capi.check(lib.pcp_ring_schedule(rank, world, hop, ctypes.byref(ss), ctypes.byref(rs), ctypes.byref(to),
                                          ctypes.byref(frm)))
        live_send = -(-valid[ss.value] // cfg.block_size)
        live_recv = -(-valid[rs.value] // cfg.block_size)
        send = have[ss.value][:live_send].contiguous()
        recv = torch.zeros((live_recv, payload))
        ops = [dist.P2POp(dist.isend, send, to.value), dist.P2POp(dist.irecv, recv, frm.value)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        have[rs.value] = recv
    assert sorted(have) == list(range(world))
    # unpack what arrived: source s contributes its first valid[s] tokens
    kd, vd = [], []
    for s in range(world):
        blk = have[s].reshape(-1, 2, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
        kd.append(blk[:, 0].permute(1, 0, 2, 3).reshape(cfg.num_kv_heads, -1, cfg.head_dim)[:, : valid[s]])
        vd.append(blk[:, 1].permute(1, 0, 2, 3).reshape(cfg.num_kv_heads, -1, cfg.head_dim)[:, : valid[s]])
    kc, vc = torch.cat(kd, 1).numpy(), torch.cat(vd, 1).numpy()
    qs = shard_query(q, cfg)[rank].numpy()
    got = orc.dense_history_attention(qs, kc, vc, cfg.softmax_scale)
    want = orc.dense_history_attention(qs, k.numpy(), v.numpy(), cfg.softmax_scale)
    np.testing.assert_allclose(got, want, atol=2e-5, rtol=2e-5)
    return {"live_blocks": [-(-x // cfg.block_size) for x in valid]}


def mismatch_body(rank, world):
    from aws_training_study_b200.pcp_attention.cuda_backend import check_ring_consistency

    cfg = _ring_cfg(world)
    if rank == world - 1:  # this rank was launched with another history length
        cfg = cfg.with_overrides(actual_history_len=cfg.actual_history_len - 64)
    try:
        check_ring_consistency(cfg, cfg.source_valid_lens())
    except RuntimeError as exc:
        return str(exc)
    return None


def missing_rank_body(rank, world):
    from aws_training_study_b200.pcp_attention.cuda_backend import check_ring_consistency

    cfg = _ring_cfg(world)
    if rank == world - 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        check_ring_consistency(cfg, cfg.source_valid_lens())
    except Exception as exc:  # gloo reports the lost peer / timeout
        return f"{type(exc).__name__}"
    return None


# ------------------------------------------------------------------- tests --
@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_delivers_every_shard(world):
    res = run_ranks("test_ring_gloo", "ring_exchange_body", world)
    assert all(s == "ok" for s, _ in res.values()), res


def test_config_mismatch_is_caught_on_every_rank():
    res = run_ranks("test_ring_gloo", "mismatch_body", 2)
    for rank, (status, payload) in res.items():
        assert status == "ok", payload
        assert payload and "mismatch" in payload, (rank, payload)


def test_missing_rank_surfaces_as_host_exception():
    res = run_ranks("test_ring_gloo", "missing_rank_body", 2, timeout=90)
    status, payload = res[0]
    assert status == "ok" and payload is not None, res
