"""Spawn helper for multi-process tests: runs ``module.fn(rank, world)`` in
``world`` spawned processes with an initialised process group and returns
{rank: (status, payload)}."""

from __future__ import annotations

import datetime
import importlib
import os
import queue
import socket
import time
import traceback

import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, module, fn_name, backend, env, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), **env)
    try:
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        fn = getattr(importlib.import_module(module), fn_name)
        q.put((rank, "ok", fn(rank, world)))
    except Exception as exc:  # reported to the parent
        q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def run_ranks(module: str, fn_name: str, world: int, timeout: float = 120.0, backend: str = "gloo",
              env: dict | None = None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, module, fn_name, backend, env or {}, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.monotonic() + timeout
    try:
        # Collect until every rank reported or every process has exited (a
        # rank that leaves on purpose reports nothing).
        while len(results) < world and time.monotonic() < deadline:
            try:
                rank, status, payload = q.get(timeout=0.5)
                results[rank] = (status, payload)
            except queue.Empty:
                if not any(p.is_alive() for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    while True:
        try:
            rank, status, payload = q.get_nowait()
            results[rank] = (status, payload)
        except queue.Empty:
            break
    return results
