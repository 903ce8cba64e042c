"""Randomised equivalence of the product's layout functions with the oracle's
restatement of ``pcp_attention/layout.py`` (which is pinned to the reference's
own outputs), over many shapes including ragged histories: every result must
be bit-exact."""

from __future__ import annotations

import numpy as np
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from aws_training_study_b200.pcp_attention import (
    PCPAttentionConfig,
    gather_history,
    owner_and_local_position,
    pack_local_kv,
    shard_history,
    shard_query,
)
from oracle import pcp_oracle as orc


@st.composite
def configs(draw):
    P = draw(st.integers(1, 6))
    I = draw(st.sampled_from([1, 2, 4, 8, 16]))
    bs = I * draw(st.integers(1, 4))
    stride = P * I
    cur = stride * draw(st.integers(1, 3))
    max_hist = stride * draw(st.integers(1, 12))
    actual = draw(st.integers(1, max_hist))
    hkv = draw(st.integers(1, 2))
    hq = hkv * draw(st.integers(1, 3))
    return PCPAttentionConfig(P, cur, max_hist, actual, bs, I, hq, hkv, 4)


def _oc(cfg):
    return orc.OracleConfig(cfg.pcp_size, cfg.current_len, cfg.max_history_len, cfg.actual_history_len,
                            cfg.block_size, cfg.interleave_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)


@settings(max_examples=150, deadline=None)
@given(configs(), st.integers(0, 2**31 - 1))
def test_layout_matches_oracle(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=g)
    k = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g)
    v = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g)
    oc = _oc(cfg)
    for mine, ref in zip(shard_query(q, cfg), orc.shard_query(q.numpy(), oc)):
        np.testing.assert_array_equal(mine.numpy(), ref)
    ks, vs = shard_history(k, v, cfg)
    rks, rvs = orc.shard_history(k.numpy(), v.numpy(), oc, num_blocks=ks[0].shape[0])
    for a, b in zip(ks + vs, rks + rvs):
        np.testing.assert_array_equal(a.numpy(), b)
    np.testing.assert_array_equal(gather_history(ks, cfg).numpy(), k.numpy())
    for a, b, rk, rv in zip(ks, vs, rks, rvs):
        np.testing.assert_array_equal(pack_local_kv(a, b).numpy(), orc.pack_local_kv(rk, rv))


@settings(max_examples=300, deadline=None)
@given(st.integers(0, 10**6), st.integers(1, 16), st.sampled_from([1, 8, 64]))
def test_owner_matches_oracle(p, P, I):
    assert owner_and_local_position(p, P, I) == orc.owner_and_local_position(p, P, I)
