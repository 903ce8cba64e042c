"""The allocation-free entry point ``pcp_history_attention_noalloc``.

It exists for callers that may not allocate device memory (a host framework
that owns all device memory, a serving loop that must never reach the
allocator, a plugin whose host forbids allocation): its scratch is a fixed
static device array inside the library.  This file is collected last on
purpose, so that a failure here (e.g. run with -x) comes after every other
test has run.  It also passes alone in a fresh process.

The checks, all through the C ABI:
  * two calls in a row -- a long history, then a shorter ragged one of
    another shape, so stale scratch contents from the first call must not
    leak into the second -- each compared with the CPU oracle (dense fp32
    attention of the reference, pinned to its outputs) and with the existing
    workspace entry ``pcp_history_attention`` on the same inputs, within the
    parity bounds of tests/parity.py; the device status word stays 0;
  * a problem whose split partials cannot fit the scratch runs as one split
    (compared with a torch fp32 reference on the GPU);
  * repeated calls change neither torch's reserved memory nor the device's
    free memory;
  * an oversized problem is rejected before anything is launched (real
    device buffers of the stated shapes, so a regression cannot touch
    unmapped memory).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from aws_training_study_b200 import _capi
from aws_training_study_b200.pcp_attention import PCPAttentionConfig
from aws_training_study_b200.pcp_attention.cuda_backend import history_attention_single, make_dims, payload_elements

from parity import MAX_ABS, MEAN_ABS, REL_L2, assert_parity, expected_rank_output, make_case, packed_shards

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


# first call: long history; second: shorter ragged history, other shape
CASES = [
    (PCPAttentionConfig(4, 1024, 16384, 16384, 512, 64, 32, 2, 256), torch.float8_e4m3fn, 3),
    (PCPAttentionConfig(4, 512, 8192, 5001, 512, 64, 16, 4, 128), torch.bfloat16, 4),
]


def _inputs(cfg, kv_dtype, seed, dev, rank=1):
    q, k, v, q_shards, k_shards, v_shards = make_case(cfg, seed=seed, kv_dtype=kv_dtype)
    packed = packed_shards(cfg, k_shards, v_shards)
    order = [(rank - s) % cfg.pcp_size for s in range(cfg.pcp_size)]
    allkv = torch.cat([packed[s] for s in order]).to(dev)
    valid = [cfg.source_valid_len(s) for s in order]
    expected = expected_rank_output(cfg, q, k, v, rank)
    return q_shards[rank].to(dev), allkv, valid, expected


def test_noalloc_matches_oracle_and_workspace_entry_twice_in_a_row():
    dev = torch.device("cuda", 0)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    for cfg, kv_dtype, seed in CASES:
        q, allkv, valid, expected = _inputs(cfg, kv_dtype, seed, dev)
        want = history_attention_single(q, allkv, valid, cfg, kv_dtype=kv_dtype)
        got = torch.full_like(q, float("nan"))
        _noalloc(cfg, q, allkv, valid, kv_dtype, got, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_parity(got, expected, f"noalloc vs oracle {cfg}")
        _close(got, want)


def test_noalloc_one_split_when_partials_do_not_fit():
    # 32 x 4096 query rows: one split's fp32 partials alone (128 MiB) exceed
    # the 64 MiB scratch (the e4m3 cache itself is read in place), so the
    # launch runs as one split writing the output directly.
    dev = torch.device("cuda", 0)
    cfg = PCPAttentionConfig(1, 4096, 16384, 16384, 512, 64, 32, 2, 256)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, generator=g, device=dev).to(torch.bfloat16)
    kv = (torch.randn(cfg.max_local_blocks, 2, cfg.num_kv_heads, cfg.block_size, cfg.head_dim, generator=g,
                      device=dev) * 0.5).to(torch.float8_e4m3fn)
    packed = kv.reshape(cfg.max_local_blocks, -1).contiguous()
    out = torch.full_like(q, float("nan"))
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    _noalloc(cfg, q, packed, [16384], torch.float8_e4m3fn, out, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        group = cfg.q_heads_per_kv_head
        for h in (0, 15, 31):
            k = kv[:, 0, h // group].reshape(-1, cfg.head_dim).float()
            v = kv[:, 1, h // group].reshape(-1, cfg.head_dim).float()
            ref = torch.softmax(q[h].float() @ k.T * cfg.softmax_scale, dim=-1) @ v
            _close(out[h], ref)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_noalloc_allocates_nothing():
    dev = torch.device("cuda", 0)
    status = torch.full((1,), -1, dtype=torch.int32, device=dev)
    prepared = []
    for cfg, kv_dtype, seed in CASES:
        q, allkv, valid, _ = _inputs(cfg, kv_dtype, seed, dev)
        prepared.append((cfg, kv_dtype, q, allkv, valid, torch.empty_like(q)))
    # Warm-up: every kernel these shapes use is loaded once.
    for cfg, kv_dtype, q, allkv, valid, out in prepared:
        _noalloc(cfg, q, allkv, valid, kv_dtype, out, status)
    torch.cuda.synchronize()
    reserved = torch.cuda.memory_reserved(dev)
    free = torch.cuda.mem_get_info(dev)[0]
    for _ in range(3):
        for cfg, kv_dtype, q, allkv, valid, out in prepared:
            _noalloc(cfg, q, allkv, valid, kv_dtype, out, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.cuda.memory_reserved(dev) == reserved
    assert torch.cuda.mem_get_info(dev)[0] == free


def test_noalloc_rejects_oversized_problems():
    # A bf16 cache is attended from a dense bf16 copy in the scratch: 256 MiB
    # here, four times the array.  (An e4m3 cache is read in place and needs
    # scratch only for split partials.)
    dev = torch.device("cuda", 0)
    cfg = PCPAttentionConfig(1, 4096, 131072, 131072, 512, 64, 32, 2, 256)
    dims = make_dims(cfg, torch.bfloat16)
    q = torch.zeros(cfg.num_q_heads, cfg.local_q_len, cfg.head_dim, dtype=torch.bfloat16, device=dev)
    packed = torch.zeros(cfg.max_local_blocks, payload_elements(cfg), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    dstatus = torch.zeros(1, dtype=torch.int32, device=dev)
    status = _capi.lib().pcp_history_attention_noalloc(
        ctypes.byref(dims), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(packed.data_ptr()), 1,
        _capi.int32_array([131072]), ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(dstatus.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
    )
    assert status == 2  # PCP_ERR_UNSUPPORTED, nothing launched
    assert b"scratch bytes" in _capi.lib().pcp_last_error()
