"""Paged KV cache on the GPU (needs a B200): the producer kernel is bit-exact
with the oracle's restatement of the reference's cache construction, its
e4m3 rounding matches ``e4m3fn_encode`` on every bf16 bit pattern, and
attention read through block tables equals the contiguous path bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention, history_attention_single
from aws_training_study_b200.pcp_attention.paged import cache_write, history_attention_paged_single, make_pool
from oracle import pcp_oracle as orc

from parity import assert_parity, oracle_config, to_numpy_f32

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _history_bf16(cfg, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    shape = (cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16), \
        (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)


def _gpu_pools(cfg, k, v, kv_dtype, seed, cuts=None):
    """Every rank's pool written by the GPU producer through a permuted table,
    in appends at `cuts`; returns pools, tables and the oracle's pools."""
    rng = np.random.default_rng(seed)
    oc = oracle_config(cfg)
    bf16 = kv_dtype == torch.bfloat16
    A = cfg.actual_history_len
    cuts = cuts or [0, A]
    kd, vd = k.to(DEV), v.to(DEV)
    kn, vn = to_numpy_f32(k), to_numpy_f32(v)
    pools, tables, expected = [], [], []
    for rank in range(cfg.pcp_size):
        nb = cfg.max_local_blocks
        extra = 3
        perm = rng.permutation(nb + extra)[:nb].astype(np.int32)
        table = torch.from_numpy(perm).to(DEV)
        pool = make_pool(cfg, nb + extra, kv_dtype, DEV)
        for a, b in zip(cuts[:-1], cuts[1:]):
            st = cache_write(cfg, rank, a, kd[:, a:b].contiguous(), vd[:, a:b].contiguous(), table, pool)
            assert int(st.item()) == 0
        ref = np.zeros((nb + extra, pool.shape[1] * pool.element_size()), dtype=np.uint8)
        orc.cache_write(ref, perm, kn, vn, 0, oc, rank, bf16)
        pools.append(pool)
        tables.append(table)
        expected.append(ref)
    return pools, tables, expected


@pytest.mark.parametrize("kv_dtype", [torch.float8_e4m3fn, torch.bfloat16], ids=["e4m3", "bf16"])
@pytest.mark.parametrize("cfg", [
    PCPAttentionConfig(4, 1024, 8192, 5000, 512, 64, 16, 2, 256),
    PCPAttentionConfig(3, 384, 2304, 1111, 128, 32, 4, 2, 128),
], ids=["p4_bs512", "p3_bs128"])
def test_cache_write_bit_exact(cfg, kv_dtype):
    A = cfg.actual_history_len
    k, v = _history_bf16(cfg, seed=3)
    pools, _, expected = _gpu_pools(cfg, k, v, kv_dtype, seed=4, cuts=sorted({0, 1, 77, 640, A // 2, A}))
    for rank, (pool, ref) in enumerate(zip(pools, expected)):
        got = pool.view(torch.uint8).cpu().numpy().reshape(ref.shape)
        np.testing.assert_array_equal(got, ref, err_msg=f"rank {rank}")


def test_e4m3_rounding_on_every_bf16_pattern():
    """All 65536 bf16 bit patterns (zeros, subnormals, ties, 448..464, beyond,
    Inf, NaN) through the producer's e4m3 conversion."""
    cfg = PCPAttentionConfig(1, 64, 512, 512, 512, 64, 1, 1, 128)
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    k = bits.reshape(1, 512, 128).contiguous()
    v = torch.zeros_like(k)
    pool = make_pool(cfg, 1, torch.float8_e4m3fn, DEV)
    table = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert int(cache_write(cfg, 0, 0, k.to(DEV), v.to(DEV), table, pool).item()) == 0
    got = pool.view(torch.uint8).cpu().numpy()[0, : 512 * 128]
    want = orc.e4m3fn_encode(to_numpy_f32(k).reshape(-1))
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first bf16 bits {bad[:8]}: got {got[bad[:8]]} want {want[bad[:8]]}"


def test_out_of_pool_table_entry_is_reported_not_written():
    cfg = PCPAttentionConfig(1, 64, 1024, 1024, 512, 64, 1, 1, 128)
    k, v = _history_bf16(cfg, seed=1)
    pool = make_pool(cfg, 2, torch.float8_e4m3fn, DEV)
    table = torch.tensor([1, 2], dtype=torch.int32, device=DEV)  # block 1 -> pool block 2: outside
    st = cache_write(cfg, 0, 0, k.to(DEV), v.to(DEV), table, pool)
    assert int(st.item()) == 109
    assert torch.count_nonzero(pool[0].view(torch.uint8)) == 0  # pool block 0 untouched
    assert torch.count_nonzero(pool[1].view(torch.uint8)) > 0   # logical block 0 written


@pytest.mark.parametrize("kv_dtype", [torch.float8_e4m3fn, torch.bfloat16], ids=["e4m3", "bf16"])
def test_paged_attention_equals_contiguous_and_oracle(kv_dtype, kv_path):
    cfg = PCPAttentionConfig(4, 1024, 8192, 5000, 512, 64, 16, 2, 256)
    oc = oracle_config(cfg)
    k, v = _history_bf16(cfg, seed=9)
    pools, tables, expected = _gpu_pools(cfg, k, v, kv_dtype, seed=10)
    gq = torch.Generator().manual_seed(11)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=gq).to(torch.bfloat16)
    rank = 2
    q_shard = torch.from_numpy(orc.shard_query(to_numpy_f32(q), oc)[rank]).to(torch.bfloat16).to(DEV)
    srcs = [(rank - s) % cfg.pcp_size for s in range(cfg.pcp_size)]
    valid = [cfg.source_valid_len(s) for s in srcs]
    # paged: one pool holding every source's blocks, tables offset per source
    nb = pools[0].shape[0]
    pool = torch.cat([pools[s] for s in srcs]).contiguous()
    tables_all = torch.stack([tables[s] + i * nb for i, s in enumerate(srcs)]).contiguous()
    paged = history_attention_paged_single(q_shard, pool, tables_all, valid, cfg)
    # contiguous: the oracle's pools read in table order
    packed = []
    for s in srcs:
        raw = torch.from_numpy(expected[s][tables[s].cpu().numpy()]).view(kv_dtype)
        packed.append(raw.reshape(cfg.max_local_blocks, -1))
    contiguous = history_attention_single(q_shard, torch.cat(packed).to(DEV), valid, cfg, kv_dtype=kv_dtype)
    assert torch.equal(paged, contiguous)
    kq = k if kv_dtype == torch.bfloat16 else torch.from_numpy(orc.e4m3fn_encode(to_numpy_f32(k))).view(kv_dtype)
    vq = v if kv_dtype == torch.bfloat16 else torch.from_numpy(orc.e4m3fn_encode(to_numpy_f32(v))).view(kv_dtype)
    want = orc.dense_history_attention(to_numpy_f32(q_shard), to_numpy_f32(kq), to_numpy_f32(vq), oc.softmax_scale)
    assert_parity(paged, want, "paged")


def test_handle_forward_paged_single_rank_equals_forward(kv_path):
    cfg = PCPAttentionConfig(1, 1024, 4096, 3333, 512, 64, 32, 2, 256)
    k, v = _history_bf16(cfg, seed=5)
    pools, tables, expected = _gpu_pools(cfg, k, v, torch.float8_e4m3fn, seed=6)
    packed = torch.from_numpy(expected[0][tables[0].cpu().numpy()]).view(torch.float8_e4m3fn)
    packed = packed.reshape(cfg.max_local_blocks, -1).to(DEV)
    q = torch.randn(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, device=DEV).to(torch.bfloat16)
    attn = HistoryAttention(cfg, rank=0, device=0)
    a = attn.forward_paged(q, pools[0], tables[0])
    b = attn(q, packed)
    attn.status()
    assert torch.equal(a, b)
    attn.close()


@pytest.mark.parametrize("kv_dtype", [torch.float8_e4m3fn, torch.bfloat16], ids=["e4m3", "bf16"])
def test_attention_table_entry_outside_pool_is_reported(kv_dtype, kv_path):
    """A block-table entry outside the pool is reported as code 109 (device
    status) and never read: the e4m3 path loads an in-pool block in its place,
    the bf16 unpack skips it."""
    from aws_training_study_b200._capi import PcpError

    cfg = PCPAttentionConfig(1, 256, 2048, 2048, 512, 64, 8, 2, 128)
    k, v = _history_bf16(cfg, seed=3)
    pools, tables, _ = _gpu_pools(cfg, k, v, kv_dtype, seed=4)
    bad = tables[0].clone().reshape(1, -1)
    bad[0, 1] = pools[0].shape[0] + 5
    q = torch.randn(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, device=DEV).to(torch.bfloat16)
    with pytest.raises(PcpError, match="code 109"):
        history_attention_paged_single(q, pools[0], bad.contiguous(), [2048], cfg)
    # the context is still usable
    good = history_attention_paged_single(q, pools[0], tables[0].reshape(1, -1).contiguous(), [2048], cfg)
    assert torch.isfinite(good.float()).all()
