"""Host API of the product (config, striped layout, KV packing, mask, inputs):
the reference's own host tests (tests/test_config.py, test_layout.py,
test_kernel_pack.py, test_runner.py) restated against this package, plus
bit-exact comparisons with the golden vectors and with the oracle."""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from aws_training_study_b200.pcp_attention import (
    PCPAttentionConfig,
    gather_history,
    get_preset,
    global_positions_for_rank,
    owner_and_local_position,
    pack_local_kv,
    shard_history,
    shard_query,
)
from aws_training_study_b200.pcp_attention.inputs import make_block_valid_mask, make_inputs, make_local_inputs
from aws_training_study_b200.pcp_attention.kernel import valid_tokens_from_mask
from oracle import pcp_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


# -- config (reference tests/test_config.py:6-44) ------------------------------
def test_full_shape_math():
    cfg = get_preset("full")
    assert cfg.local_q_len == 64
    assert cfg.actual_local_history_len == 2048
    assert cfg.actual_local_blocks == 4
    assert cfg.softmax_scale == 1 / 16


def test_rejects_unequal_striped_shards():
    with pytest.raises(ValueError, match=r"pcp_size \* interleave_size"):
        get_preset("tiny").with_overrides(current_len=320)


def test_partial_last_local_cache_block():
    cfg = get_preset("tiny").with_overrides(max_history_len=2048, actual_history_len=1024)
    assert cfg.actual_local_history_len == 256
    assert cfg.actual_local_blocks == 1


def test_accepts_multiple_local_q_tiles():
    cfg = get_preset("full").with_overrides(pcp_size=16, current_len=4096, max_history_len=8192,
                                            actual_history_len=8192)
    assert cfg.local_q_len == 256


def test_relaxed_trainium_checks():
    """Shapes only the NKI kernel rejected are valid here (local Q 192,
    block 64, D 64, odd KV head counts, unaligned history)."""
    get_preset("full").with_overrides(pcp_size=16, current_len=3072)
    PCPAttentionConfig(4, 256, 1024, 1024, 64, 16, 8, 2, 128).validate()
    PCPAttentionConfig(4, 256, 1024, 1024, 64, 16, 6, 3, 64).validate()
    cfg = PCPAttentionConfig(8, 2048, 32768, 30001, 512, 64, 32, 2, 256).validate()
    assert cfg.source_valid_lens() == [3776] * 4 + [3761] + [3712] * 3
    assert cfg.local_cache_blocks == 8


@pytest.mark.parametrize("bad,match", [
    (dict(actual_history_len=4096), "must not exceed"),
    (dict(num_q_heads=3), "divisible by num_kv_heads"),
    (dict(block_size=96), "divisible by interleave_size"),
    (dict(max_history_len=2100), r"pcp_size \* interleave_size"),
    (dict(pcp_size=0), "positive"),
])
def test_semantic_checks_kept(bad, match):
    with pytest.raises(ValueError, match=match):
        get_preset("tiny").with_overrides(**bad)


def test_config_matches_oracle_math():
    for cfg in (get_preset("tiny"), get_preset("full"), PCPAttentionConfig(8, 8192, 524288, 500000, 512, 64, 64, 8, 128)):
        oc = orc.OracleConfig(cfg.pcp_size, cfg.current_len, cfg.max_history_len, cfg.actual_history_len,
                              cfg.block_size, cfg.interleave_size, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim)
        for name in ("softmax_scale", "q_heads_per_kv_head", "local_q_len", "max_local_history_len",
                     "actual_local_history_len", "max_local_blocks", "actual_local_blocks", "rank_stride"):
            assert getattr(cfg, name) == getattr(oc, name), name
        assert cfg.source_valid_lens() == [oc.source_valid_len(r) for r in range(cfg.pcp_size)]


# -- layout (reference tests/test_layout.py:12-40) -------------------------------
def test_owner_round_trip():
    for rank in range(4):
        positions = global_positions_for_rank(2048, rank, 4, 64)
        for local_position, global_position in enumerate(positions.tolist()):
            assert owner_and_local_position(global_position, 4, 64) == (rank, local_position)


def test_history_shard_and_gather_are_inverse():
    cfg = get_preset("tiny")
    shape = (cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim)
    k = torch.arange(int(np.prod(shape)), dtype=torch.float32).reshape(shape)
    ks, vs = shard_history(k, -k, cfg)
    torch.testing.assert_close(gather_history(ks, cfg), k)
    torch.testing.assert_close(gather_history(vs, cfg), -k)


def test_partial_cache_block_shard_and_gather_are_inverse():
    cfg = get_preset("tiny").with_overrides(actual_history_len=1024)
    shape = (cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim)
    k = torch.arange(int(np.prod(shape)), dtype=torch.float32).reshape(shape)
    ks, _ = shard_history(k, -k, cfg)
    assert ks[0].shape[0] == 1
    assert torch.count_nonzero(ks[0][:, :, 256:, :]) == 0
    torch.testing.assert_close(gather_history(ks, cfg), k)


def test_layout_bit_exact_with_reference_golden():
    g = np.load(GOLDEN / "layout.npz")
    for total, P, I in ((2048, 4, 64), (1024, 4, 16), (8192, 8, 64), (131072, 8, 64)):
        for r in range(P):
            np.testing.assert_array_equal(global_positions_for_rank(total, r, P, I).numpy(),
                                          g[f"pos_{total}_{P}_{I}_{r}"])
    samples = g["owner_samples"]
    np.testing.assert_array_equal(np.array([owner_and_local_position(int(p), 8, 64) for p in samples]),
                                  g["owner_8_64"])
    for tag, cfg in (("tiny", get_preset("tiny")), ("partial", get_preset("tiny").with_overrides(actual_history_len=1024))):
        shape = (cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim)
        kk = torch.arange(int(np.prod(shape)), dtype=torch.float32).reshape(shape)
        ks, _ = shard_history(kk, -kk, cfg)
        for r, t in enumerate(ks):
            assert tuple(t.shape) == tuple(g[f"shard_{tag}_{r}_shape"])
            assert sha(t) == str(g[f"shard_{tag}_{r}_sha"])


def test_ragged_layout_matches_oracle():
    """Unaligned history (rejected by the reference): product == oracle, and
    every rank holds exactly source_valid_len tokens, then zeros."""
    cfg = PCPAttentionConfig(4, 128, 1024, 1001, 64, 16, 4, 2, 32).validate()
    oc = orc.OracleConfig(4, 128, 1024, 1001, 64, 16, 4, 2, 32)
    k = torch.randn(2, 1001, 32)
    q = torch.randn(4, 128, 32)
    ks, _ = shard_history(k, -k, cfg)
    oks, _ = orc.shard_history(k.numpy(), -k.numpy(), oc)
    for r in range(4):
        np.testing.assert_array_equal(ks[r].numpy(), oks[r])
        flat = ks[r].permute(1, 0, 2, 3).reshape(2, -1, 32)
        assert torch.count_nonzero(flat[:, cfg.source_valid_len(r):]) == 0
    torch.testing.assert_close(gather_history(ks, cfg), k)
    for r, (a, b) in enumerate(zip(shard_query(q, cfg), orc.shard_query(q.numpy(), oc))):
        np.testing.assert_array_equal(a.numpy(), b)


# -- packing (reference tests/test_kernel_pack.py:6-28) ----------------------------
def test_pack_local_kv_order():
    k = torch.arange(2 * 2 * 4 * 8).reshape(2, 2, 4, 8)
    packed = pack_local_kv(k, -k)
    restored = packed.reshape(2, 2, 2, 4, 8)
    torch.testing.assert_close(restored[:, 0], k)
    torch.testing.assert_close(restored[:, 1], -k)
    g = np.load(GOLDEN / "layout.npz")
    kp = torch.from_numpy(g["pack_in"])
    np.testing.assert_array_equal(pack_local_kv(kp, -kp).numpy(), g["pack_out"])


def test_pack_local_kv_preserves_fp8_storage():
    k = torch.randn(1, 2, 4, 8, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    v = torch.randn(1, 2, 4, 8, dtype=torch.bfloat16).to(torch.float8_e4m3fn)
    packed = pack_local_kv(k, v)
    assert packed.dtype == torch.float8_e4m3fn and packed.element_size() == 1
    restored = packed.reshape(1, 2, 2, 4, 8)
    torch.testing.assert_close(restored[:, 0].float(), k.float())
    torch.testing.assert_close(restored[:, 1].float(), v.float())


# -- runner helpers (reference tests/test_runner.py:7-22) --------------------------
def test_partial_block_valid_mask():
    cfg = get_preset("tiny").with_overrides(actual_history_len=1024)
    mask = make_block_valid_mask(cfg)
    assert mask.shape == (1, 4, 1, 128)
    assert mask.dtype == torch.bfloat16
    assert torch.all(mask[0, :2] == 0)
    assert torch.all(mask[0, 2:] == -9984)
    assert valid_tokens_from_mask(mask, cfg) == 256


@pytest.mark.parametrize("name,cfg", [
    ("tiny", get_preset("tiny")),
    ("tiny_partial", get_preset("tiny").with_overrides(actual_history_len=1024)),
    ("full", get_preset("full")),
    ("full_short", get_preset("full").with_overrides(actual_history_len=65536)),
])
def test_block_valid_mask_matches_reference_golden(name, cfg):
    g = np.load(GOLDEN / "layout.npz")
    np.testing.assert_array_equal(make_block_valid_mask(cfg).float().numpy(), g[f"mask_{name}"])
    assert valid_tokens_from_mask(make_block_valid_mask(cfg), cfg) == cfg.actual_local_history_len


def test_local_kv_inputs_use_final_fp8_storage():
    _, k, v = make_local_inputs(get_preset("tiny"), seed=1234, rank=0)
    assert k.dtype == torch.float8_e4m3fn and v.dtype == torch.float8_e4m3fn


def test_input_generators_bit_exact_with_reference():
    g = np.load(GOLDEN / "layout.npz")
    tiny = get_preset("tiny")
    assert [sha(t) for t in make_inputs(tiny, 1234)] == [str(x) for x in g["make_inputs_sha"]]
    assert [sha(t) for t in make_local_inputs(tiny, 1234, 1)] == [str(x) for x in g["make_local_inputs_sha"]]


def test_bucket_for_rounds_up_to_block_groups_and_caps():
    from aws_training_study_b200.pcp_attention.graphs import bucket_for

    cfg = PCPAttentionConfig(2, 256, 8192, 8192, 512, 64, 4, 2, 128)  # 8 blocks per shard
    assert bucket_for(cfg, [0, 1], 2) == (0, 1024)
    assert bucket_for(cfg, [1024, 1025], 2) == (1024, 2048)
    assert bucket_for(cfg, [4000, 4096], 3) == (4096, 4096)  # capped at the shard capacity
    with pytest.raises(ValueError):
        bucket_for(cfg, [4097, 0], 1)
    with pytest.raises(ValueError):
        bucket_for(cfg, [1, 1], 0)
