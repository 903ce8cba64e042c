"""Host-side placement for the host-buffer entry points.

``HistoryAttention.forward_host*`` copies each step's Q and KV shard in from
pinned host memory and the output back.  With one process per GPU on a
multi-socket host, a rank whose pinned buffers sit in the other socket's
memory pulls every copy across the socket link, and eight ranks doing so at
once share that link.  ``near_device`` runs a block of host code on the CPU
cores that the GPU's PCI device reports as local, so that pinned buffers
allocated inside it (first touch) live in the GPU's own NUMA node; the
process's previous CPU affinity comes back afterwards.  On a host without
that information (no sysfs entry, one NUMA node, a container that hides it)
it changes nothing.
"""

from __future__ import annotations

import contextlib
import os
from pathlib import Path


def _parse_cpulist(text: str) -> set[int]:
    """``"0-3,8,10-11"`` -> {0, 1, 2, 3, 8, 10, 11}."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-", 1)
            cpus.update(range(int(lo), int(hi) + 1))
        else:
            cpus.add(int(part))
    return cpus


def device_local_cpus(device: int, sysfs: Path = Path("/sys/bus/pci/devices")) -> set[int] | None:
    """CPU cores local to CUDA device ``device`` that this process may use, or
    None when the host does not say (or none of them is allowed)."""
    import torch

    props = torch.cuda.get_device_properties(device)
    bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    try:
        local = _parse_cpulist((sysfs / bus / "local_cpulist").read_text())
    except (OSError, ValueError):
        return None
    allowed = local & os.sched_getaffinity(0)
    return allowed or None


@contextlib.contextmanager
def near_device(device: int, enable: bool = True):
    """Run the block on ``device``'s local CPU cores; yields the core count
    used (None: placement unchanged)."""
    cpus = device_local_cpus(device) if enable else None
    if not cpus or cpus == os.sched_getaffinity(0):
        yield None
        return
    saved = os.sched_getaffinity(0)
    os.sched_setaffinity(0, cpus)
    try:
        yield len(cpus)
    finally:
        os.sched_setaffinity(0, saved)
