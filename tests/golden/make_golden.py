"""Generate the golden fixtures in this folder by running the REFERENCE itself.

    python tests/golden/make_golden.py --reference <checkout of HandsomeHow/aws_training_study>

Imports the reference's own ``pcp_attention`` package and ``run_poc.py``
(pure Python/torch, runnable on a CPU) and records their outputs on seeded
inputs.  Inputs are regenerated from the seeds by the tests with the same
torch generator calls, and their SHA-256 digests are stored so a test can
prove it rebuilt the very same inputs.  Fixtures:

* ``ref_tests.npz``     -- the reference's own pins (tests/test_reference.py:8-56):
                          ring vs dense on the ``tiny`` preset with Hq=4, Hkv=2,
                          D=128, seeds 1234 (full blocks) and 7 (partial block).
* ``baseline_cfg1.npz`` -- BASELINE config 1 (P=4, 8/2/128, Q=256, hist=1024,
                          bs=64, I=16; Q, K/V ~ 0.5 N(0,1), K/V via e4m3fn),
                          ring model with the Trainium-only validation bypassed.
* ``unaligned.npz``     -- a ragged history (A=1001 at P=4, I=16): the
                          reference's dense_history_attention per rank on
                          k[:, :A] (its ring model cannot express this case).
* ``layout.npz``        -- positions, owner/local pairs, shard/gather
                          results, block-valid masks, input-generator digests.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bfloat16):
        t = t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def randn_inputs(cfg, seed, scale=1.0):
    """torch.randn fp32 Q, K, V in the order of tests/test_reference.py:13-21."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(cfg.num_q_heads, cfg.current_len, cfg.head_dim, generator=g) * scale
    k = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g) * scale
    v = torch.randn(cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim, generator=g) * scale
    return q, k, v


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a checkout of the reference repository")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from pcp_attention.config import PCPAttentionConfig, get_preset
    from pcp_attention.kernel import pack_local_kv
    from pcp_attention.layout import (
        gather_history,
        global_positions_for_rank,
        owner_and_local_position,
        shard_history,
        shard_query,
    )
    from pcp_attention.reference import dense_history_attention, ring_history_attention
    from run_poc import make_block_valid_mask, make_inputs, make_local_inputs

    # -- the reference's own test pins -------------------------------------
    out = {}
    for tag, seed, overrides in (
        ("full", 1234, dict(num_q_heads=4, num_kv_heads=2, head_dim=128)),
        ("partial", 7, dict(actual_history_len=1024, num_q_heads=4, num_kv_heads=2, head_dim=128)),
    ):
        cfg = get_preset("tiny").with_overrides(**overrides)
        q, k, v = randn_inputs(cfg, seed)
        qs = shard_query(q, cfg)
        ks, vs = shard_history(k, v, cfg)
        ring = ring_history_attention(qs, ks, vs, cfg)
        dk, dv = gather_history(ks, cfg), gather_history(vs, cfg)
        dense = [dense_history_attention(qs[r], dk, dv, cfg.softmax_scale) for r in range(cfg.pcp_size)]
        out[f"{tag}_seed"] = np.int64(seed)
        out[f"{tag}_actual"] = np.int64(cfg.actual_history_len)
        out[f"{tag}_sha_q"] = sha(q)
        out[f"{tag}_sha_k"] = sha(k)
        out[f"{tag}_sha_v"] = sha(v)
        out[f"{tag}_ring"] = np.stack([t.numpy() for t in ring])
        out[f"{tag}_ring_vs_dense"] = np.float64(max((a - b).abs().max().item() for a, b in zip(ring, dense)))
    np.savez_compressed(HERE / "ref_tests.npz", **out)

    # -- BASELINE config 1 (ring model, validate bypassed) -----------------
    PCPAttentionConfig.validate = lambda self: self  # bs=64 is rejected only by a Trainium check
    cfg = PCPAttentionConfig(
        pcp_size=4, current_len=256, max_history_len=1024, actual_history_len=1024,
        block_size=64, interleave_size=16, num_q_heads=8, num_kv_heads=2, head_dim=128,
    )
    g = torch.Generator().manual_seed(2024)
    q = torch.randn(8, 256, 128, generator=g) * 0.5
    k8 = (torch.randn(2, 1024, 128, generator=g) * 0.5).to(torch.float8_e4m3fn)
    v8 = (torch.randn(2, 1024, 128, generator=g) * 0.5).to(torch.float8_e4m3fn)
    qs = shard_query(q, cfg)
    ks, vs = shard_history(k8, v8, cfg)
    ring = ring_history_attention(qs, ks, vs, cfg)
    dense = [dense_history_attention(qs[r], k8, v8, cfg.softmax_scale) for r in range(4)]
    np.savez_compressed(
        HERE / "baseline_cfg1.npz",
        seed=np.int64(2024), sha_q=sha(q), sha_k=sha(k8), sha_v=sha(v8),
        ring=np.stack([t.numpy() for t in ring]),
        ring_vs_dense=np.float64(max((a - b).abs().max().item() for a, b in zip(ring, dense))),
    )

    # -- ragged history: dense reference on k[:, :A] ------------------------
    A = 1001
    cfg_u = PCPAttentionConfig(
        pcp_size=4, current_len=128, max_history_len=1024, actual_history_len=A,
        block_size=64, interleave_size=16, num_q_heads=4, num_kv_heads=2, head_dim=128,
    )
    g = torch.Generator().manual_seed(31)
    q = torch.randn(4, 128, 128, generator=g).to(torch.bfloat16)
    k = (torch.randn(2, A, 128, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(2, A, 128, generator=g) * 0.5).to(torch.bfloat16)
    qs = shard_query(q, cfg_u)
    dense = [dense_history_attention(qs[r], k, v, cfg_u.softmax_scale) for r in range(4)]
    np.savez_compressed(
        HERE / "unaligned.npz",
        seed=np.int64(31), actual=np.int64(A), sha_q=sha(q), sha_k=sha(k), sha_v=sha(v),
        dense=np.stack([t.numpy() for t in dense]),
    )

    # -- layout, masks, input generators -----------------------------------
    del PCPAttentionConfig.validate  # restore the class's own method
    import importlib

    import pcp_attention.config as refcfg

    importlib.reload(refcfg)
    from pcp_attention.config import get_preset as gp

    lay = {}
    for total, P, I in ((2048, 4, 64), (1024, 4, 16), (8192, 8, 64), (131072, 8, 64)):
        for r in range(P):
            lay[f"pos_{total}_{P}_{I}_{r}"] = global_positions_for_rank(total, r, P, I).numpy()
    samples = np.arange(0, 8192, 37)
    lay["owner_samples"] = samples
    lay["owner_8_64"] = np.array([owner_and_local_position(int(p), 8, 64) for p in samples])
    lay["owner_4_16"] = np.array([owner_and_local_position(int(p), 4, 16) for p in samples])
    tiny = gp("tiny")
    shape = (tiny.num_kv_heads, tiny.actual_history_len, tiny.head_dim)
    kk = torch.arange(int(np.prod(shape)), dtype=torch.float32).reshape(shape)
    ksh, _ = shard_history(kk, -kk, tiny)
    for r, t in enumerate(ksh):
        lay[f"shard_tiny_{r}_shape"] = np.array(t.shape)
        lay[f"shard_tiny_{r}_sha"] = sha(t)
    part = tiny.with_overrides(actual_history_len=1024)
    shape = (part.num_kv_heads, part.actual_history_len, part.head_dim)
    kk = torch.arange(int(np.prod(shape)), dtype=torch.float32).reshape(shape)
    ksh, _ = shard_history(kk, -kk, part)
    for r, t in enumerate(ksh):
        lay[f"shard_partial_{r}_shape"] = np.array(t.shape)
        lay[f"shard_partial_{r}_sha"] = sha(t)
    kp = torch.arange(2 * 2 * 4 * 8, dtype=torch.float32).reshape(2, 2, 4, 8)
    lay["pack_in"] = kp.numpy()
    lay["pack_out"] = pack_local_kv(kp, -kp).numpy()
    for name, c in (
        ("tiny", gp("tiny")),
        ("tiny_partial", gp("tiny").with_overrides(actual_history_len=1024)),
        ("full", gp("full")),
        ("full_short", gp("full").with_overrides(actual_history_len=65536)),
    ):
        lay[f"mask_{name}"] = make_block_valid_mask(c).float().numpy()
    q, k, v = make_inputs(tiny, 1234)
    lay["make_inputs_sha"] = np.array([sha(q), sha(k), sha(v)])
    q, k, v = make_local_inputs(tiny, 1234, 1)
    lay["make_local_inputs_sha"] = np.array([sha(q), sha(k), sha(v)])
    np.savez_compressed(HERE / "layout.npz", **lay)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
