"""NUMA placement of the host-resident value chunks.

The value gather reads page-locked host memory over the GPU's PCIe link.  If
those pages live on the other socket, every read also crosses the CPU
interconnect.  ``bind_to_gpu_numa`` pins the calling process to the CPUs of
the GPU's NUMA node before the pinned buffers are allocated, so the kernel's
first-touch placement puts them next to the GPU's root port.
"""
from __future__ import annotations

import os
import subprocess


def _bus_id(device_index: int) -> str | None:
    try:
        import torch
        p = torch.cuda.get_device_properties(device_index)
        return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:
        pass
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(device_index), "--query-gpu=pci.bus_id",
                              "--format=csv,noheader"], capture_output=True, text=True, timeout=20).stdout.strip()
        dom, rest = out.split(":", 1)
        return f"{int(dom, 16) & 0xffff:04x}:{rest.lower()}"
    except Exception:
        return None


def gpu_numa_node(device_index: int) -> int | None:
    """NUMA node of the GPU's PCIe device, or None when the platform does not report one."""
    bus = _bus_id(device_index)
    if bus is None:
        return None
    path = f"/sys/bus/pci/devices/{bus}/numa_node"
    try:
        node = int(open(path).read().strip())
    except (OSError, ValueError):
        return None
    return node if node >= 0 else None


def parse_cpulist(text: str) -> set[int]:
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


def node_cpus(node: int) -> set[int]:
    try:
        return parse_cpulist(open(f"/sys/devices/system/node/node{node}/cpulist").read())
    except OSError:
        return set()


def bind_to_gpu_numa(device_index: int) -> int | None:
    """Restrict this process to the CPUs of the GPU's NUMA node; returns the node (or None)."""
    node = gpu_numa_node(device_index)
    if node is None:
        return None
    cpus = node_cpus(node) & os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    return node
