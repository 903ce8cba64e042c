"""Length-bucket CUDA graphs of the history attention.

The reference compiles its kernel once per static config and masks the
unused history at run time (``pcp_attention/kernel.py:32-40``; its README,
``README.md:52-54``, lists "skip masked blocks' transfer and compute entirely
and graph-capture one artifact per bucket" as the next step).  Here one CUDA
graph is recorded per *bucket* -- an upper bound on every source rank's valid
history -- through ``HistoryAttention.forward_bucketed``: the NCCL exchange,
key regions, split plan and grids are fixed by the bucket, while the kernels
read the actual lengths from a device buffer when the graph runs.  A replay
therefore serves any lengths up to the bucket, never computes a tile past
them, and never touches blocks past the bucket at all.

Graphs record fixed addresses: ``q``, ``packed_kv`` and ``out`` are static
buffers the caller refills before each replay.
"""

from __future__ import annotations

import torch

from .config import PCPAttentionConfig


def bucket_for(config: PCPAttentionConfig, valid_len, granularity_blocks: int = 4) -> tuple[int, ...]:
    """The bucket of ``valid_len``: every source's length rounded up to a
    whole number of ``granularity_blocks`` cache blocks, at most its shard
    capacity (``max_local_blocks * block_size``)."""
    if granularity_blocks <= 0:
        raise ValueError("granularity_blocks must be positive")
    step = granularity_blocks * config.block_size
    cap = config.max_local_blocks * config.block_size
    out = []
    for v in valid_len:
        v = int(v)
        if not 0 <= v <= cap:
            raise ValueError(f"valid length {v} outside [0, {cap}]")
        out.append(min(cap, -(-v // step) * step))
    return tuple(out)


class BucketGraph:
    """One recorded forward for one bucket over static buffers.

    ``replay(valid_len)`` writes the lengths into the graph's device buffer
    (an asynchronous copy on the current stream, ordered before the replay)
    and launches the graph on the current stream; the result lands in
    ``out``.  ``HistoryAttention.status()`` watches the streams of its own
    calls, not replays: synchronise the replay's stream (or consume ``out``
    on it) before calling it to read a replay's device status."""

    def __init__(self, attn, bucket_len, q: torch.Tensor, packed_kv: torch.Tensor, out: torch.Tensor | None = None,
                 warmup: int = 1):
        self.attn = attn
        self.bucket = tuple(int(b) for b in bucket_len)
        if len(self.bucket) != attn.config.pcp_size:
            raise ValueError(f"bucket needs {attn.config.pcp_size} entries")
        self.q, self.packed_kv = q, packed_kv
        self.out = out if out is not None else torch.empty_like(q)
        dev = attn.device
        self.valid_dev = torch.tensor(self.bucket, dtype=torch.int32, device=dev)
        # Warm-up outside the capture: one-time kernel attributes and NCCL's
        # lazy peer connections must not happen while recording.
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                attn.forward_bucketed(q, packed_kv, self.valid_dev, self.bucket, self.out)
        torch.cuda.current_stream(dev).wait_stream(side)
        attn.status()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.device(dev), torch.cuda.graph(self.graph):
            attn.forward_bucketed(q, packed_kv, self.valid_dev, self.bucket, self.out)
        attn._register_graph(self)

    def replay(self, valid_len) -> torch.Tensor:
        vals = [int(v) for v in valid_len]
        if len(vals) != len(self.bucket) or any(v < 0 or v > b for v, b in zip(vals, self.bucket)):
            raise ValueError(f"valid_len {vals} outside bucket {self.bucket}")
        self.valid_dev.copy_(torch.tensor(vals, dtype=torch.int32), non_blocking=True)
        self.graph.replay()
        return self.out

    def reset(self) -> None:
        if getattr(self, "graph", None) is not None:
            self.graph.reset()
            self.graph = None


class BucketedHistoryAttention:
    """``HistoryAttention`` with one CUDA graph per length bucket, recorded on
    first use: ``__call__(valid_len)`` runs the bucket's graph over the static
    ``q`` / ``packed_kv`` buffers (refilled by the caller) and returns ``out``."""

    def __init__(self, attn, q: torch.Tensor, packed_kv: torch.Tensor, granularity_blocks: int = 4):
        self.attn, self.q, self.packed_kv = attn, q, packed_kv
        self.granularity_blocks = granularity_blocks
        self.out = torch.empty_like(q)
        self.graphs: dict[tuple[int, ...], BucketGraph] = {}

    def __call__(self, valid_len=None) -> torch.Tensor:
        if valid_len is None:
            valid_len = self.attn.config.source_valid_lens()
        bucket = bucket_for(self.attn.config, valid_len, self.granularity_blocks)
        g = self.graphs.get(bucket)
        if g is None:
            g = self.graphs[bucket] = BucketGraph(self.attn, bucket, self.q, self.packed_kv, self.out)
        return g.replay(valid_len)

    def close(self) -> None:
        for g in self.graphs.values():
            g.reset()
        self.graphs.clear()
