"""Host placement of a rank process next to its GPU, and a boot probe of per-rank bandwidth.

On an HGX B200 node each GPU hangs off one CPU socket's PCIe root; the host side of a rank
(the pinned input/output buffers, the shared-memory command ring, the Python scheduler thread)
is fastest on that socket's NUMA node. ``apply()`` sets this process's CPU affinity and host
memory policy from flags before anything large is allocated; children inherit both. Device
allocations do not follow the host policy; only host pages move.

- ``QB_HOST_CPU_NODES=0,1`` or ``auto``: run this process's threads on those nodes' CPUs
  (``auto``: the node of this rank's GPU, read from sysfs by PCI bus id).
- ``QB_HOST_MEM_NODES=0`` or ``auto``: bind (one node) or interleave (several) host pages.

``probe()`` (``QB_RANK_BW_PROBE=1``) prints one ``[rank-bw]`` line per rank after boot: HBM read
bandwidth over the rank's largest device tensors, pinned host->device and device->host copy
bandwidth, the GPU's NUMA node and the per-node host memory. It changes no numbers.

Reference behaviour: ``host_numa.py:33-141`` (``parse_nodes``, ``node_cpus``, ``apply``,
``node_meminfo_gib``, ``probe``); the node list syntax and the ``[rank-bw]`` record are kept
alike so logs of both read the same way. The GPU-to-node lookup and the copy-bandwidth part are
this framework's (on MI300A the GPU index is the node; here the PCIe topology decides).
"""

from __future__ import annotations

import ctypes
import gc
import json
import os
import platform
from pathlib import Path

from . import flags

NODE_ROOT = Path("/sys/devices/system/node")
PCI_ROOT = Path("/sys/bus/pci/devices")
_MPOL_BIND, _MPOL_INTERLEAVE = 2, 3
_SYS_SET_MEMPOLICY = {"x86_64": 238, "aarch64": 237}


def parse_nodes(spec: str) -> list[int]:
    """``"1,2,3"`` or ``"1-3"`` -> sorted unique node ids; an empty spec -> []."""
    out: set[int] = set()
    for part in spec.replace(" ", "").split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        out.update(range(int(lo), int(hi or lo) + 1))
    return sorted(out)


def node_cpus(node: int, root: Path = NODE_ROOT) -> set[int]:
    return set(parse_nodes((Path(root) / f"node{node}" / "cpulist").read_text().strip()))


def pci_bus_id(device_index: int) -> str:
    """``dddd:bb:dd.0`` of a CUDA device (lower case, as sysfs names it)."""
    import torch

    p = torch.cuda.get_device_properties(device_index)
    return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"


def gpu_numa_node(bus_id: str, root: Path = PCI_ROOT) -> int:
    """The NUMA node of the PCI device ``bus_id`` (-1 when the platform does not say)."""
    f = Path(root) / bus_id.lower() / "numa_node"
    try:
        return int(f.read_text().strip())
    except (OSError, ValueError):
        return -1


def _resolve(spec: str, gpu_node: int) -> list[int]:
    if spec.strip().lower() == "auto":
        return [gpu_node] if gpu_node >= 0 else []
    return parse_nodes(spec)


def _set_mempolicy(nodes: list[int]) -> None:
    nr = _SYS_SET_MEMPOLICY.get(platform.machine())
    if nr is None:
        raise OSError(f"set_mempolicy: unknown syscall number on {platform.machine()}")
    mask = ctypes.c_ulong(sum(1 << n for n in nodes))
    mode = _MPOL_BIND if len(nodes) == 1 else _MPOL_INTERLEAVE
    libc = ctypes.CDLL(None, use_errno=True)
    if libc.syscall(nr, mode, ctypes.byref(mask), 64) != 0:
        raise OSError(ctypes.get_errno(), f"set_mempolicy({mode}, {nodes})")


def apply(env: dict | None = None, gpu_node: int = -1, root: Path = NODE_ROOT,
          setaffinity=os.sched_setaffinity, setmempolicy=_set_mempolicy) -> str:
    """Apply the placement flags to this process; returns a one-line summary ("" when none)."""
    notes = []
    cpu_nodes = _resolve(flags.get("QB_HOST_CPU_NODES", env), gpu_node)
    if cpu_nodes:
        setaffinity(0, set().union(*(node_cpus(n, root) for n in cpu_nodes)))
        notes.append(f"cpu_nodes={cpu_nodes}")
    mem_nodes = _resolve(flags.get("QB_HOST_MEM_NODES", env), gpu_node)
    if mem_nodes:
        setmempolicy(mem_nodes)
        notes.append(("mem_bind=" if len(mem_nodes) == 1 else "mem_interleave=") + str(mem_nodes))
    return " ".join(notes)


def apply_for_device(device_index: int) -> str:
    """``apply`` with ``auto`` resolved to the node of CUDA device ``device_index``."""
    if not (flags.get("QB_HOST_CPU_NODES") or flags.get("QB_HOST_MEM_NODES")):
        return ""
    return apply(gpu_node=gpu_numa_node(pci_bus_id(device_index)))


def node_meminfo_gib(root: Path = NODE_ROOT) -> dict[str, dict[str, float]]:
    """Per-node MemUsed / MemFree / FilePages in GiB (empty off Linux)."""
    out = {}
    for d in sorted(Path(root).glob("node[0-9]*"), key=lambda p: int(p.name[4:])):
        vals = {}
        try:
            lines = (d / "meminfo").read_text().splitlines()
        except OSError:
            continue
        for line in lines:
            p = line.split()
            if len(p) >= 4 and p[2].rstrip(":") in ("MemUsed", "MemFree", "FilePages"):
                vals[p[2].rstrip(":")] = round(int(p[3]) / 2**20, 1)
        out[d.name] = vals
    return out


def _device_tensors(device, top: int):
    import torch

    seen, tensors = set(), []
    for obj in gc.get_objects():
        try:
            if isinstance(obj, torch.Tensor) and obj.device == device and obj.numel():
                st = obj.untyped_storage()
                key = (st.data_ptr(), st.nbytes())
                if key not in seen:
                    seen.add(key)
                    tensors.append(obj)
        except Exception:  # noqa: BLE001 - some objects refuse inspection
            continue
    tensors.sort(key=lambda t: t.untyped_storage().nbytes(), reverse=True)
    return tensors[:top]


def _copy_gbs(device, nbytes: int, h2d: bool, iters: int = 5) -> float:
    import torch

    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
    src, dst = (host, dev) if h2d else (dev, host)
    dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        dst.copy_(src, non_blocking=True)
    e.record()
    e.synchronize()
    return nbytes * iters / (s.elapsed_time(e) * 1e-3) / 1e9


def probe(rank: int, device, top: int = 64, copy_bytes: int = 256 << 20) -> dict:
    """Print ``[rank-bw]``: HBM read TB/s over this rank's ``top`` largest device tensors, and
    pinned copy GB/s in both directions. Walks the garbage collector once: call it at boot."""
    import torch

    device = torch.device(device)
    views = []
    for t in _device_tensors(device, top):
        flat = torch.empty(0, dtype=torch.uint8, device=device).set_(t.untyped_storage())
        views.append(flat[: flat.numel() // 4 * 4].view(torch.float32))
    torch.cuda.synchronize(device)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()  # start together: peers polling this GPU would skew it
    rows = []
    for v in views:
        v.sum()
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(3):
            v.sum()
        e.record()
        e.synchronize()
        rows.append((v.numel() * 4, s.elapsed_time(e) / 3))
    rec = {"rank": rank, "device": str(device)}
    if rows:
        total_b, total_ms = sum(b for b, _ in rows), sum(ms for _, ms in rows)
        rates = sorted(b / (ms * 1e-3) / 1e12 for b, ms in rows)
        median = rates[len(rates) // 2]
        rec.update(tensors=len(rows), gib=round(total_b / 2**30, 2),
                   read_tbs=round(total_b / (total_ms * 1e-3) / 1e12, 3), slowest_tbs=round(rates[0], 3),
                   median_tbs=round(median, 3), n_below_60pct=sum(r < 0.6 * median for r in rates))
    rec["h2d_gbs"] = round(_copy_gbs(device, copy_bytes, True), 1)
    rec["d2h_gbs"] = round(_copy_gbs(device, copy_bytes, False), 1)
    try:
        rec["gpu_node"] = gpu_numa_node(pci_bus_id(device.index or 0))
    except Exception:  # noqa: BLE001 - no sysfs in some containers
        rec["gpu_node"] = -1
    rec["cpus"] = len(os.sched_getaffinity(0))
    rec["numa"] = node_meminfo_gib()
    rec["cpu_nodes"] = flags.get("QB_HOST_CPU_NODES")
    rec["mem_nodes"] = flags.get("QB_HOST_MEM_NODES")
    print(f"[rank-bw] {json.dumps(rec)}", flush=True)
    return rec
