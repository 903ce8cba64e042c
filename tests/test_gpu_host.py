"""The host-buffer entries (needs a B200): ``forward_host`` and the
double-buffered ``forward_host_async`` / ``forward_host_wait`` serving loop
give the same output as the device-buffer call on the same inputs, step
after step, with inputs that change between steps (a slot reused too early
would show the previous step's data)."""

from __future__ import annotations

import pytest
import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention

from parity import assert_parity, expected_rank_output, make_case, packed_shards

pytestmark = pytest.mark.gpu


def test_host_entries_equal_device_call_over_a_stream_of_steps():
    cfg = PCPAttentionConfig(1, 1024, 4096, 3001, 512, 64, 32, 2, 256)
    attn = HistoryAttention(cfg, rank=0, device=0)
    cases = []
    for seed in (1, 2, 3):
        q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=seed)
        kv = packed_shards(cfg, k_shards, v_shards)[0]
        want = attn(q_shards[0].cuda(), kv.cuda()).cpu()
        cases.append((q_shards[0].pin_memory(), kv.view(torch.uint8).pin_memory().view(kv.dtype), want,
                      expected_rank_output(cfg, q, k, v, 0)))
    attn.status()
    order = [0, 1, 2, 0, 2, 1, 1]
    outs = [torch.empty_like(cases[0][0]).pin_memory() for _ in order]
    for i, c in enumerate(order):
        attn.forward_host_async(cases[c][0], cases[c][1], out=outs[i])
    attn.forward_host_wait()
    attn.status()
    for i, c in enumerate(order):
        assert torch.equal(outs[i], cases[c][2]), f"step {i} (case {c})"
    sync_out = attn.forward_host(cases[1][0], cases[1][1])
    assert torch.equal(sync_out, cases[1][2])
    assert_parity(sync_out, cases[1][3], "forward_host")
    attn.close()
