"""Host-side placement for multi-GPU runs: bind a rank to the CPU cores local to its GPU, so that the pinned host
buffers it allocates afterwards (first touch) sit on the GPU's NUMA node and host <-> device copies do not cross the
socket interconnect.  Linux sysfs only; a no-op where the information is unavailable."""
from __future__ import annotations

import os

import torch


def _parse_cpulist(text: str) -> set[int]:
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_local_cpus(device) -> set[int]:
    """CPU ids local to the GPU `device` (empty when unknown)."""
    try:
        p = torch.cuda.get_device_properties(torch.device(device))
        path = f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist"
        with open(path) as fh:
            return _parse_cpulist(fh.read())
    except (OSError, AttributeError, ValueError, RuntimeError):
        return set()


def bind_to_gpu_numa(device) -> bool:
    """Restrict this process to the CPUs local to `device` (intersected with the allowed set); True when bound."""
    local = gpu_local_cpus(device)
    try:
        allowed = os.sched_getaffinity(0)
    except AttributeError:
        return False
    cpus = local & allowed
    if not cpus or cpus == allowed:
        return False
    os.sched_setaffinity(0, cpus)
    return True
