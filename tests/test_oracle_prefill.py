"""The oracle's prefill attention (history plus causal current tokens),
checked three independent ways on the CPU:

* against torch's fp32 ``scaled_dot_product_attention`` with an explicit
  boolean mask, on un-striped (P = 1) inputs;
* stripe consistency: every rank's output equals its rows of the P = 1
  computation over the whole sequence (the position arithmetic of the stripe
  layout, ``layout.py:19-51``);
* the log-sum-exp merge of history-only (``dense_history_attention``, pinned
  to the reference) and causal-current-only attention reproduces it -- the
  decomposition the CUDA path computes.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import pcp_oracle as orc


def _inputs(hq, hkv, a, cur, d, seed):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    return f(hq, cur, d), f(hkv, a, d) * 0.5, f(hkv, a, d) * 0.5, f(hkv, cur, d) * 0.5, f(hkv, cur, d) * 0.5


def _merge(o1, l1, o2, l2):
    m = np.maximum(l1, l2)
    w1, w2 = np.exp(l1 - m), np.exp(l2 - m)
    return (o1 * w1[..., None] + o2 * w2[..., None]) / (w1 + w2)[..., None]


def _attn_lse(q, k, v, mask=None):
    s = np.einsum("hqd,hkd->hqk", q, k) / math.sqrt(q.shape[-1])
    if mask is not None:
        s = np.where(mask, s, -np.inf)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    return (p @ v) / p.sum(-1, keepdims=True), (m[..., 0] + np.log(p.sum(-1)))


@pytest.mark.parametrize("a", [0, 96])
def test_matches_torch_sdpa_unstriped(a):
    hq, hkv, cur, d = 4, 2, 48, 32
    q, kh, vh, kc, vc = _inputs(hq, hkv, a, cur, d, seed=3)
    cfg = orc.OracleConfig(1, cur, max(a, 1), a, 16, cur, hq, hkv, d)
    got = orc.prefill_attention(q, kh, vh, kc, vc, cfg, rank=0)
    g = hq // hkv
    keys = torch.from_numpy(np.concatenate([kh, kc], 1)).repeat_interleave(g, 0)
    vals = torch.from_numpy(np.concatenate([vh, vc], 1)).repeat_interleave(g, 0)
    mask = torch.ones(cur, a + cur, dtype=torch.bool)
    mask[:, a:] = torch.tril(torch.ones(cur, cur, dtype=torch.bool))
    ref = torch.nn.functional.scaled_dot_product_attention(torch.from_numpy(q), keys, vals, attn_mask=mask)
    np.testing.assert_allclose(got, ref.numpy(), atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("P,I", [(4, 8), (3, 16), (2, 32)])
def test_striped_ranks_equal_rows_of_global_causal(P, I):
    hq, hkv, a, d = 4, 2, 40, 16
    cur = P * I * 2
    q, kh, vh, kc, vc = _inputs(hq, hkv, a, cur, d, seed=11)
    whole = orc.prefill_attention(q, kh, vh, kc, vc, orc.OracleConfig(1, cur, a, a, 8, cur, hq, hkv, d), 0)
    cfg = orc.OracleConfig(P, cur, a, a, 8, I, hq, hkv, d)
    for rank in range(P):
        pos = orc.global_positions_for_rank(cur, rank, P, I)
        q_shard = orc.shard_query(q, cfg)[rank]
        got = orc.prefill_attention(q_shard, kh, vh, kc, vc, cfg, rank)
        np.testing.assert_allclose(got, whole[:, pos], atol=2e-6, rtol=1e-5)


def test_lse_merge_of_history_and_current_parts():
    hq, hkv, a, d, P, I = 4, 1, 64, 32, 2, 16
    cur = P * I * 2
    q, kh, vh, kc, vc = _inputs(hq, hkv, a, cur, d, seed=5)
    cfg = orc.OracleConfig(P, cur, a, a, 16, I, hq, hkv, d)
    rank = 1
    q_shard = orc.shard_query(q, cfg)[rank]
    got = orc.prefill_attention(q_shard, kh, vh, kc, vc, cfg, rank)
    hist = orc.dense_history_attention(q_shard, kh, vh, cfg.softmax_scale)
    g = hq // hkv
    _, l_hist = _attn_lse(q_shard, np.repeat(kh, g, 0), np.repeat(vh, g, 0))
    pos = orc.global_positions_for_rank(cur, rank, P, I)
    mask = np.arange(cur)[None, None, :] <= pos[None, :, None]
    o_cur, l_cur = _attn_lse(q_shard, np.repeat(kc, g, 0), np.repeat(vc, g, 0), mask)
    np.testing.assert_allclose(got, _merge(hist, l_hist, o_cur, l_cur), atol=2e-6, rtol=1e-5)


def test_flops_count_visible_pairs_only():
    cfg = orc.OracleConfig(2, 8, 4, 4, 4, 2, 1, 1, 1)
    # rank 0 holds positions 0,1,4,5 -> visible current keys 1+2+5+6 = 14
    assert orc.prefill_flops(cfg, 0) == 4.0 * (4 * 4 + 14)
