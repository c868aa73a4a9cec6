"""Keep a rank's host threads on the CPUs attached to its GPU (``QB_CPU_AFFINITY=1``).

A rank's host work (scheduling, input packing, pinned-memory staging) runs fastest on the
CPU socket whose PCIe root holds its GPU. The kernel publishes that set per PCI device as
``/sys/bus/pci/devices/<domain:bus:dev.fn>/local_cpulist``; this module reads it for the
rank's GPU (PCI address from the CUDA device properties) and restricts the process to it.
Off by default: the launcher or the container may already place the process.

Reference behaviour: the reference places MI300A ranks on NUMA nodes (``host_numa.py``); B200
boxes are discrete-GPU machines, so the GPU's own CPU list is the placement that matters.
"""

from __future__ import annotations

import os

from . import flags

SYSFS_PCI = "/sys/bus/pci/devices"


def parse_cpulist(text: str) -> set[int]:
    """``"0-3,8,10-11"`` -> ``{0, 1, 2, 3, 8, 10, 11}`` (the kernel's cpulist format)."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        lo, sep, hi = part.partition("-")
        a = int(lo)
        b = int(hi) if sep else a
        if b < a:
            raise ValueError(f"bad cpulist range {part!r}")
        cpus.update(range(a, b + 1))
    return cpus


def _norm_bus_id(bus_id: str) -> str:
    """CUDA reports ``00000000:1B:00.0``; sysfs names the device ``0000:1b:00.0``."""
    dom, _, rest = bus_id.strip().partition(":")
    return f"{int(dom, 16):04x}:{rest.lower()}"


def gpu_local_cpus(bus_id: str, root: str = SYSFS_PCI) -> set[int]:
    """CPUs local to the PCI device ``bus_id``; empty when sysfs does not say."""
    path = os.path.join(root, _norm_bus_id(bus_id), "local_cpulist")
    try:
        with open(path) as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError):
        return set()


def pin_to_gpu(bus_id: str, env: dict | None = None, root: str = SYSFS_PCI,
               setter=None, getter=None) -> str:
    """Restrict this process to the GPU's local CPUs when ``QB_CPU_AFFINITY`` is on. Only CPUs
    the process may already use are kept; returns a note for the log ("" when nothing changed)."""
    if not flags.get("QB_CPU_AFFINITY", env):
        return ""
    setter = setter or (lambda cpus: os.sched_setaffinity(0, cpus))
    getter = getter or (lambda: os.sched_getaffinity(0))
    local = gpu_local_cpus(bus_id, root)
    allowed = set(getter())
    cpus = local & allowed
    if not cpus:
        return ""
    setter(cpus)
    return f"{len(cpus)} CPUs local to GPU {bus_id}"


def pin_device(index: int) -> str:
    """``pin_to_gpu`` for CUDA device ``index`` (reads its PCI address from the driver)."""
    import torch

    props = torch.cuda.get_device_properties(index)
    bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    return pin_to_gpu(bus)
