"""Host-memory placement for the host-buffer forward (``MoELayer.forward_host``).

Pinned host buffers are placed on the NUMA node of the thread that first touches them.  On a
multi-socket host, buffers on the socket that is not attached to the GPU's PCIe root cross
the inter-socket link on every copy, which lowers host<->device bandwidth most when both
directions run at once (the host-buffer forward overlaps them).  ``bind_to_device_node``
pins the calling thread to the CPUs of the GPU's NUMA node (read from sysfs) so that the
pinned buffers it allocates afterwards land next to the GPU.
"""
from __future__ import annotations

import os


def device_numa_node(device: int) -> int | None:
    """NUMA node of CUDA device ``device`` (None when the host does not report one)."""
    import torch
    p = torch.cuda.get_device_properties(device)
    bus = getattr(p, "pci_bus_id", None)
    dev = getattr(p, "pci_device_id", None)
    dom = getattr(p, "pci_domain_id", 0) or 0
    if bus is None or dev is None:
        return None
    path = f"/sys/bus/pci/devices/{dom:04x}:{bus:02x}:{dev:02x}.0/numa_node"
    try:
        with open(path) as f:
            node = int(f.read().strip())
    except (OSError, ValueError):
        return None
    return node if node >= 0 else None


def node_cpus(node: int) -> set[int]:
    """CPUs of NUMA node ``node`` (from its sysfs cpulist, e.g. "0-23,48-71")."""
    cpus: set[int] = set()
    with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
        for part in f.read().strip().split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.update(range(int(a), int(b) + 1))
            elif part:
                cpus.add(int(part))
    return cpus


def bind_to_device_node(device: int) -> set[int] | None:
    """Pin the calling thread to the CPUs of ``device``'s NUMA node.

    Returns the previous CPU set (pass it to ``os.sched_setaffinity`` to undo), or None when
    the node is unknown or the host has one node (nothing changes then).
    """
    node = device_numa_node(device)
    if node is None:
        return None
    try:
        cpus = node_cpus(node) & os.sched_getaffinity(0)
    except OSError:
        return None
    prev = os.sched_getaffinity(0)
    if not cpus or cpus == prev:
        return None
    os.sched_setaffinity(0, cpus)
    return prev
