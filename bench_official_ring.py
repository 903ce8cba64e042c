#!/usr/bin/env python3
"""The reference's ``bench_official_ring.py`` workload on B200s, through the
same CUDA history-attention path.

    torchrun --nproc-per-node 8 bench_official_ring.py [--local-seqlen 2048 --heads 32 --head-dim 128]

The reference times the nkilib ``ring_attention_spmd_fwd`` kernel on its
own shape (``bench_official_ring.py:1-8,68-166``): every rank holds equal
local Q/K/V ``[1, heads, local_seqlen, head_dim]`` bf16 (seeded with
``seed + 104729 * rank``), multi-head (no GQA), non-causal, and every rank's
queries attend to all ranks' keys.  Non-causal ring self-attention is exactly
history attention whose history is the whole sequence, so here each rank's
K/V becomes its packed cache shard, the shards are exchanged over NVLink and
the CTA-pair kernel attends Q to all of them.

Reported like the reference (min/median/mean/p90/max over iterations of the
per-iteration max over ranks; ``effective_tflops = 4*H*D*S^2 / mean``), for
DEVICE time (CUDA events on the launching stream) and, as the reference
measures, host wall-clock with a one-element device-to-host completion marker.
"""

from __future__ import annotations

import argparse
import os
import statistics
import sys
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))


def parse_args() -> argparse.Namespace:
    parser = argparse.ArgumentParser()
    parser.add_argument("--local-seqlen", type=int, default=2048)
    parser.add_argument("--heads", type=int, default=32)
    parser.add_argument("--head-dim", type=int, default=128)
    parser.add_argument("--block-size", type=int, default=512)
    parser.add_argument("--warmups", type=int, default=3)
    parser.add_argument("--iterations", type=int, default=20)
    parser.add_argument("--seed", type=int, default=20260907)
    parser.add_argument("--exchange", choices=("direct", "ring", "allgather", "pipeline"), default="direct")
    parser.add_argument("--phases", action="store_true",
                        help="after timing, profile a few calls and print rank 0's per-phase device time")
    return parser.parse_args()


def percentile_nearest_rank(samples: list[float], percentile: float) -> float:
    ordered = sorted(samples)
    index = max(0, int((percentile * len(ordered) + 0.999999)) - 1)
    return ordered[min(index, len(ordered) - 1)]


def main() -> int:
    args = parse_args()
    if args.warmups < 1 or args.iterations < 1:
        raise ValueError("warmups and iterations must both be positive")
    import torch.distributed as dist

    from aws_training_study_b200.pcp_attention import PCPAttentionConfig, pack_local_kv
    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() in ("VERSION", ""):
        os.environ["NCCL_DEBUG"] = "WARN"
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("gloo")
    L, H, D = args.local_seqlen, args.heads, args.head_dim
    if L % args.block_size:
        raise ValueError("--local-seqlen must be a multiple of --block-size")
    S = L * world
    cfg = PCPAttentionConfig(pcp_size=world, current_len=S, max_history_len=S, actual_history_len=S,
                             block_size=args.block_size, interleave_size=min(64, args.block_size),
                             num_q_heads=H, num_kv_heads=H, head_dim=D).validate()
    generator = torch.Generator().manual_seed(args.seed + 104729 * rank)
    shape = (1, H, L, D)
    q = torch.randn(shape, dtype=torch.bfloat16, generator=generator)
    k = torch.randn(shape, dtype=torch.bfloat16, generator=generator)
    v = torch.randn(shape, dtype=torch.bfloat16, generator=generator)
    blocks = L // args.block_size

    def cache(t):  # [1, H, L, D] -> [blocks, H, bs, D]
        return t[0].reshape(H, blocks, args.block_size, D).permute(1, 0, 2, 3).contiguous()

    packed = pack_local_kv(cache(k), cache(v))
    if packed.shape[0] < cfg.max_local_blocks:
        padded = torch.zeros((cfg.max_local_blocks, packed.shape[1]), dtype=packed.dtype)
        padded[: packed.shape[0]] = packed
        packed = padded
    attn = HistoryAttention(cfg, kv_dtype=torch.bfloat16, rank=rank, device=local_rank, exchange=args.exchange)
    q_dev, kv_dev = q[0].contiguous().to(dev), packed.to(dev)
    valid = [L] * world
    stream = torch.cuda.current_stream()
    for _ in range(args.warmups):
        attn(q_dev, kv_dev, valid).reshape(-1)[:1].cpu()
    attn.status()
    if world > 1:
        dist.monitored_barrier()
    dev_ms, host_ms = [], []
    for _ in range(args.iterations):
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        s_ev.record(stream)
        out = attn(q_dev, kv_dev, valid)
        e_ev.record(stream)
        marker = out.reshape(-1)[:1].cpu()
        host_ms.append((time.perf_counter() - t0) * 1e3)
        dev_ms.append(s_ev.elapsed_time(e_ev))
        _ = marker[0].item()
    samples = [(dev_ms, host_ms)]
    if world > 1:
        samples = [None] * world
        dist.all_gather_object(samples, (dev_ms, host_ms))
    phases = None
    if args.phases:
        attn.set_profiling(True)
        for _ in range(5):
            attn(q_dev, kv_dev, valid)
        attn.status()
        st = attn.stats()
        attn.set_profiling(False)
        phases = {k: (st[k] / st["forwards"] if k.endswith("_ms") else st[k]) for k in st}
    if rank == 0:
        useful_flops = 4 * H * D * S * S
        if phases:
            print(f"official_ring_benchmark[phases rank0]: {phases}", flush=True)
        for label, idx in (("device", 0), ("host", 1)):
            per_iter = [max(r[idx][i] for r in samples) for i in range(args.iterations)]
            mean_ms = statistics.fmean(per_iter)
            print(
                f"official_ring_benchmark[{label}]: "
                f"world_size={world}, exchange={args.exchange}, "
                f"local_shape={shape}, global_seqlen={S}, "
                f"warmups={args.warmups}, iterations={args.iterations}, "
                f"min_ms={min(per_iter):.3f}, "
                f"median_ms={statistics.median(per_iter):.3f}, "
                f"mean_ms={mean_ms:.3f}, "
                f"p90_ms={percentile_nearest_rank(per_iter, 0.9):.3f}, "
                f"max_ms={max(per_iter):.3f}, "
                f"effective_tflops={useful_flops / (mean_ms / 1000.0) / 1e12:.3f}",
                flush=True,
            )
    attn.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
