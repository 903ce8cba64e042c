"""The allocation-free entry point ``pcp_history_attention_noalloc``.

It exists for callers that may not allocate device memory (a host framework
that owns all device memory, a serving loop that must never reach the
allocator, a plugin whose host forbids allocation): its scratch is a fixed
static device array inside the library.  This file is collected last on
purpose, so that a failure here (e.g. run with -x) comes after every other
test has run.  It also passes alone in a fresh process.

The check: two calls in a row through the C ABI -- a long history, then a
shorter one, so stale scratch contents from the first call must not leak into
the second -- each compared with the existing workspace entry
``pcp_history_attention`` on the same inputs, within the parity bounds of
tests/parity.py, and the device status word must stay 0.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from aws_training_study_b200 import _capi
from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import history_attention_single, make_dims

from parity import MAX_ABS, MEAN_ABS, REL_L2, make_case, packed_shards

pytestmark = pytest.mark.gpu


def _noalloc(cfg, q, allkv, valid, kv_dtype, out, status):
    dims = make_dims(cfg, kv_dtype)
    _capi.check(
        _capi.lib().pcp_history_attention_noalloc(
            ctypes.byref(dims), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(allkv.data_ptr()), len(valid),
            _capi.int32_array(valid), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
        )
    )


def _close(a: torch.Tensor, b: torch.Tensor) -> None:
    a, b = a.float(), b.float()
    diff = (a - b).abs()
    assert torch.isfinite(a).all()
    assert diff.max().item() <= MAX_ABS
    assert diff.mean().item() <= MEAN_ABS
    assert (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item() <= REL_L2


def test_noalloc_matches_workspace_entry_twice_in_a_row():
    dev = torch.device("cuda", 0)
    cases = [
        # first call: long history; second: shorter ragged history, other shape
        (PCPAttentionConfig(4, 1024, 16384, 16384, 512, 64, 32, 2, 256), torch.float8_e4m3fn, 3),
        (PCPAttentionConfig(4, 512, 8192, 5001, 512, 64, 16, 4, 128), torch.bfloat16, 4),
    ]
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    for cfg, kv_dtype, seed in cases:
        _, _, _, q_shards, k_shards, v_shards = make_case(cfg, seed=seed, kv_dtype=kv_dtype)
        packed = packed_shards(cfg, k_shards, v_shards)
        rank = 1
        order = [(rank - s) % cfg.pcp_size for s in range(cfg.pcp_size)]
        allkv = torch.cat([packed[s] for s in order]).to(dev)
        valid = [cfg.source_valid_len(s) for s in order]
        q = q_shards[rank].to(dev)
        want = history_attention_single(q, allkv, valid, cfg, kv_dtype=kv_dtype)
        got = torch.full_like(q, float("nan"))
        _noalloc(cfg, q, allkv, valid, kv_dtype, got, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        _close(got, want)


def test_noalloc_rejects_oversized_problems():
    cfg = PCPAttentionConfig(1, 4096, 131072, 131072, 512, 64, 32, 2, 256)
    dims = make_dims(cfg, torch.float8_e4m3fn)
    status = _capi.lib().pcp_history_attention_noalloc(
        ctypes.byref(dims), ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 20), 1, _capi.int32_array([131072]),
        ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 20), None,
    )
    assert status == 2  # PCP_ERR_UNSUPPORTED, nothing launched
    assert b"scratch bytes" in _capi.lib().pcp_last_error()
