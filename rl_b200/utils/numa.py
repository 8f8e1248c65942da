"""Bind a rank's host threads to the CPU cores of its GPU's NUMA node.

Reference: ``bind_to_gpu_numa`` (``nemo_rl/distributed/numa_utils.py:40``, ctypes
libnuma).  Here the node's CPU list is read from sysfs (``/sys/bus/pci/devices/<bus
id>/local_cpulist``, ``numa_node``) and applied with ``os.sched_setaffinity``, so no
library is needed; ``sysfs_root`` lets tests point at a fake tree.
"""

from __future__ import annotations

import os
from typing import Optional

__all__ = ["parse_cpulist", "gpu_local_cpus", "bind_to_gpu_numa"]


def parse_cpulist(text: str) -> list[int]:
    """'0-3,8,10-11' -> [0, 1, 2, 3, 8, 10, 11]."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        else:
            cpus.append(int(part))
    return cpus


def gpu_local_cpus(pci_bus_id: str, sysfs_root: str = "/sys") -> Optional[list[int]]:
    bus = pci_bus_id.lower()
    if bus.count(":") == 1:  # "0000:xx:yy.z" form expected by sysfs
        bus = "0000:" + bus
    base = os.path.join(sysfs_root, "bus", "pci", "devices", bus)
    try:
        with open(os.path.join(base, "local_cpulist")) as f:
            cpus = parse_cpulist(f.read())
        return cpus or None
    except OSError:
        return None


def bind_to_gpu_numa(device_index: Optional[int] = None, sysfs_root: str = "/sys", pci_bus_id: Optional[str] = None
                     ) -> Optional[list[int]]:
    """Restrict this process to the cores local to its GPU; returns the CPU list
    applied (None when unknown, e.g. no GPU or no sysfs entry)."""
    if pci_bus_id is None:
        try:
            import torch

            if not torch.cuda.is_available():
                return None
            idx = torch.cuda.current_device() if device_index is None else device_index
            props = torch.cuda.get_device_properties(idx)
            pci_bus_id = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        except Exception:  # noqa: BLE001 - binding is an optimisation only
            return None
    cpus = gpu_local_cpus(pci_bus_id, sysfs_root)
    if not cpus:
        return None
    allowed = os.sched_getaffinity(0)
    use = [c for c in cpus if c in allowed] or cpus
    try:
        os.sched_setaffinity(0, use)
    except OSError:
        return None
    return use
