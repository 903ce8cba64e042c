#!/usr/bin/env python3
"""Run PCP history attention on B200s -- the ``--backend cuda`` twin of the
reference's ``run_poc.py`` (same presets, overrides, seeds, input
construction, checks and benchmark report).

    python run_poc.py --preset tiny --pcp-size 1
    torchrun --standalone --nproc-per-node 8 run_poc.py --preset b200x8 --check none \
        --benchmark-iterations 30 --benchmark-warmups 3

Differences from the reference (``run_poc.py:22-353``):
* ``--backend cuda`` replaces ``neuron``; there is no CPU compute backend.
* ``--kv-dtype bf16`` runs BF16 K/V; default e4m3fn.
* ``actual_history_len`` may be unaligned; each source rank then holds
  ``config.source_valid_len(rank)`` tokens.
* Benchmark times are DEVICE times (CUDA events around each call on the
  launching stream), max over ranks per iteration, as BASELINE asks; the
  reference's host wall-clock with a 1-element D2H marker is also printed.
* The ``--check`` oracle is the reference's dense attention restated in torch
  fp32 (TF32 off), run per head on the GPU because at full size the CPU would
  take minutes.
"""

from __future__ import annotations

import argparse
import os
import statistics
import sys
import time
from dataclasses import asdict

import torch

from aws_training_study_b200.pcp_attention import PCPAttentionConfig, get_preset, pack_local_kv, shard_history, shard_query
from aws_training_study_b200.pcp_attention.inputs import make_inputs, make_local_inputs


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--backend", choices=("cuda",), default="cuda")
    p.add_argument("--preset", choices=("tiny", "full", "b200x8"), default="tiny")
    p.add_argument("--pcp-size", type=int)
    p.add_argument("--current-len", type=int)
    p.add_argument("--max-history-len", type=int)
    p.add_argument("--actual-history-len", "--start-offset", dest="actual_history_len", type=int,
                   help="runtime historical-token count; also the new-token start offset")
    p.add_argument("--block-size", type=int)
    p.add_argument("--interleave-size", type=int)
    p.add_argument("--num-q-heads", type=int)
    p.add_argument("--num-kv-heads", type=int)
    p.add_argument("--head-dim", type=int)
    p.add_argument("--kv-dtype", choices=("e4m3", "bf16"), default="e4m3")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--check", choices=("full", "sampled", "none"), default="full")
    p.add_argument("--benchmark-iterations", type=int, default=0)
    p.add_argument("--benchmark-warmups", type=int, default=1)
    return p.parse_args(argv)


def make_config(args: argparse.Namespace) -> PCPAttentionConfig:
    cfg = get_preset(args.preset)
    names = ("pcp_size", "current_len", "max_history_len", "actual_history_len", "block_size",
             "interleave_size", "num_q_heads", "num_kv_heads", "head_dim")
    return cfg.with_overrides(**{n: getattr(args, n) for n in names if getattr(args, n) is not None})


def dense_check_gpu(q_local: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """fp32 GQA attention softmax(Q K^T scale) V per head on the GPU (the
    reference's dense_history_attention, reference.py:16-32)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        hq, hkv = q_local.shape[0], k.shape[0]
        group = hq // hkv
        out = torch.empty(q_local.shape, dtype=torch.float32, device=q_local.device)
        for h in range(hq):
            kf, vf = k[h // group].float(), v[h // group].float()
            s = torch.matmul(q_local[h].float(), kf.T) * scale
            out[h] = torch.matmul(torch.softmax(s, dim=-1), vf)
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def run_cuda(cfg: PCPAttentionConfig, seed: int, check: str, kv_dtype: torch.dtype,
             benchmark_iterations: int = 0, benchmark_warmups: int = 1) -> None:
    import torch.distributed as dist

    from aws_training_study_b200.pcp_attention.cuda_backend import HistoryAttention

    if benchmark_iterations < 0 or benchmark_warmups < 0:
        raise ValueError("benchmark counts must be non-negative")
    if benchmark_iterations and benchmark_warmups == 0:
        raise ValueError("benchmark_warmups must be at least one")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != cfg.pcp_size:
        raise RuntimeError(f"torchrun WORLD_SIZE={world}, but pcp_size={cfg.pcp_size}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("gloo")

    if check == "none":
        q_local, k_local, v_local = make_local_inputs(cfg, seed, rank)
        k = v = None
        if kv_dtype != torch.float8_e4m3fn:
            k_local, v_local = k_local.to(kv_dtype), v_local.to(kv_dtype)
    else:
        q, k, v = make_inputs(cfg, seed)
        if kv_dtype != torch.float8_e4m3fn:
            k, v = k.float().to(kv_dtype), v.float().to(kv_dtype)
        q_local = shard_query(q, cfg)[rank]
        ks, vs = shard_history(k, v, cfg)
        k_local, v_local = ks[rank], vs[rank]
    packed = pack_local_kv(k_local, v_local)
    if packed.shape[0] < cfg.max_local_blocks:
        padded = torch.zeros((cfg.max_local_blocks, packed.shape[1]), dtype=packed.dtype)
        padded[: packed.shape[0]] = packed
        packed = padded
    valid = cfg.source_valid_lens()
    attn = HistoryAttention(cfg, kv_dtype=kv_dtype, rank=rank, device=local_rank)
    q_dev, kv_dev = q_local.to(dev), packed.to(dev)

    if check != "none" or benchmark_iterations == 0:
        actual = attn(q_dev, kv_dev, valid)
        attn.status()
        if check != "none":
            expected = dense_check_gpu(q_dev, k.to(dev), v.to(dev), cfg.softmax_scale)
            a = actual.float()
            if check == "sampled":
                a, expected = a[:, :1, :], expected[:, :1, :]
            torch.testing.assert_close(a, expected, atol=6e-2, rtol=6e-2)
            rel = (torch.linalg.vector_norm(a - expected) / torch.linalg.vector_norm(expected)).item()
            print(f"rank={rank}: CUDA output OK (max_abs={(a - expected).abs().max().item():.3e}, rel_l2={rel:.3e})",
                  flush=True)
        else:
            print(f"rank={rank}: CUDA run completed", flush=True)

    if benchmark_iterations:
        stream = torch.cuda.current_stream()
        for _ in range(benchmark_warmups):
            attn(q_dev, kv_dev, valid).reshape(-1)[:1].cpu()
        if dist.is_initialized():
            dist.barrier()
        dev_ms, host_ms = [], []
        for _ in range(benchmark_iterations):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            s.record(stream)
            out = attn(q_dev, kv_dev, valid)
            e.record(stream)
            marker = out.reshape(-1)[:1].cpu()
            host_ms.append((time.perf_counter() - t0) * 1e3)
            dev_ms.append(s.elapsed_time(e))
            _ = marker[0].item()
        samples = [(dev_ms, host_ms)]
        if dist.is_initialized():
            samples = [None] * world
            dist.all_gather_object(samples, (dev_ms, host_ms))
        if rank == 0:
            for label, idx in (("device", 0), ("host", 1)):
                per_iter = [max(r[idx][i] for r in samples) for i in range(benchmark_iterations)]
                srt = sorted(per_iter)
                p90 = srt[max(0, (9 * len(srt) + 9) // 10 - 1)]
                mean = statistics.fmean(per_iter)
                flops = 4.0 * cfg.num_q_heads * cfg.current_len * cfg.actual_history_len * cfg.head_dim
                print(
                    f"benchmark[{label}]: mode=cuda_c_abi, kv_dtype={kv_dtype}, iterations={benchmark_iterations}, "
                    f"warmups={benchmark_warmups}, min_ms={min(per_iter):.3f}, "
                    f"median_ms={statistics.median(per_iter):.3f}, mean_ms={mean:.3f}, p90_ms={p90:.3f}, "
                    f"max_ms={max(per_iter):.3f}, global_current_tokens_per_s={cfg.current_len / (mean / 1e3):.1f}, "
                    f"tflops_median={flops / (statistics.median(per_iter) / 1e3) / 1e12:.1f}",
                    flush=True,
                )
    attn.close()
    if dist.is_initialized():
        dist.destroy_process_group()


def main(argv=None) -> int:
    args = parse_args(argv)
    cfg = make_config(args)
    kv_dtype = torch.float8_e4m3fn if args.kv_dtype == "e4m3" else torch.bfloat16
    if int(os.environ.get("RANK", "0")) == 0:
        print("configuration:")
        for name, value in asdict(cfg).items():
            print(f"  {name}={value}")
        print(f"  local_q_len={cfg.local_q_len}")
        print(f"  source_valid_lens={cfg.source_valid_lens()}")
        print(f"  kv_dtype={args.kv_dtype}")
    run_cuda(cfg, args.seed, args.check, kv_dtype, args.benchmark_iterations, args.benchmark_warmups)
    return 0


if __name__ == "__main__":
    sys.exit(main())
