"""Boot memory timeline, per-class read bandwidth and a free-memory preflight (diagnostics).

With ``QB_MEM_TIMELINE=1``, ``mark(label)`` prints one ``[mem]`` line at each named boot phase
(weights loaded, symmetric buffers mapped, pools allocated, graphs captured): the device's free
and total memory, the caching allocator's allocated and reserved bytes, the host NUMA node's free
memory, and which allocator segments appeared since the previous mark. ``report(model)`` then
sorts the live segments into buffer classes (weights, KV cache, DeltaNet state, snapshot pool,
graph pools, other), times a read of each class's largest tensors and prints ``[mem-cls]`` per
class. With the flag off every call returns at once.

On a 180 GB B200 the pools are sized from the free memory at boot (``serving.engine``), so a
previous job still holding HBM shrinks them; ``preflight`` (``QB_BOOT_MEM_PREFLIGHT_GIB``) waits
until the device has that much free memory and fails with a clear message after
``QB_BOOT_MEM_PREFLIGHT_WAIT_S``.

Reference behaviour: ``mem_timeline.py:62-266`` (``mark``, ``report``, ``preflight``); there the
concern is NUMA-node placement of MI300A's unified memory, here device residency and the pools.
"""

from __future__ import annotations

import bisect
import json
import time
from pathlib import Path

from . import flags

MIN_PROBE_BYTES = 32 << 20  # smaller tensors are counted but not timed (launch overhead)
_T0 = time.time()
_segs: dict[int, dict] = {}
_rank = 0


def enabled() -> bool:
    return flags.get("QB_MEM_TIMELINE")


def set_rank(rank: int) -> None:
    global _rank  # noqa: PLW0603
    _rank = rank


def _host_free_gib() -> float | None:
    from .hostinfo import node_meminfo_gib

    free = [v.get("MemFree") for v in node_meminfo_gib().values() if "MemFree" in v]
    return round(sum(free), 1) if free else None


def mark(label: str, device=None, sink=print) -> dict | None:
    """Log the device's memory state and tag the allocator segments made since the last mark."""
    import torch

    if not enabled() or not torch.cuda.is_available():
        return None
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        return None
    torch.cuda.synchronize(dev)
    free, total = torch.cuda.mem_get_info(dev)
    live, new_bytes = set(), 0
    for seg in torch.cuda.memory_snapshot():
        if seg.get("device") != dev.index:
            continue
        addr = seg["address"]
        live.add(addr)
        if addr in _segs and _segs[addr]["size"] == seg["total_size"]:
            continue
        pool = tuple(seg.get("segment_pool_id", (0, 0)))
        _segs[addr] = {"addr": addr, "size": seg["total_size"], "graph_pool": pool != (0, 0), "phase": label}
        new_bytes += seg["total_size"]
    for addr in [a for a in _segs if a not in live]:
        del _segs[addr]  # released; a later segment may reuse the address
    rec = {"rank": _rank, "t": round(time.time() - _T0, 1), "label": label,
           "free_gib": round(free / 2**30, 2), "total_gib": round(total / 2**30, 2),
           "allocated_gib": round(torch.cuda.memory_allocated(dev) / 2**30, 2),
           "reserved_gib": round(torch.cuda.memory_reserved(dev) / 2**30, 2),
           "new_gib": round(new_bytes / 2**30, 3), "host_free_gib": _host_free_gib()}
    sink(f"[mem] {json.dumps(rec)}")
    return rec


def _tensors(obj, out: list, depth: int = 0) -> None:
    import torch

    if depth > 6:
        return
    if isinstance(obj, torch.Tensor):
        out.append(obj)
    elif isinstance(obj, dict):
        for v in obj.values():
            _tensors(v, out, depth + 1)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            _tensors(v, out, depth + 1)


def classes(model) -> dict[str, list]:
    """Buffer class -> the model's tensors of that class."""
    m = getattr(model, "model", model)  # a GraphRunner wraps the model
    out: dict[str, list] = {}
    for name, obj in (("weights", m.w), ("kv_cache", (m.k_cache, m.v_cache)),
                      ("deltanet_state", (m.conv_state, m.rec_state)), ("snapshots", (m.snap_conv, m.snap_rec))):
        ts: list = []
        _tensors(obj, ts)
        out[name] = ts
    return out


def _read_tbs(ts: list) -> float | None:
    import torch

    ts = [t for t in ts if t.is_cuda and t.untyped_storage().nbytes() >= MIN_PROBE_BYTES]
    ts = sorted(ts, key=lambda t: t.untyped_storage().nbytes(), reverse=True)[:16]
    if not ts:
        return None
    views = []
    for t in ts:
        flat = torch.empty(0, dtype=torch.uint8, device=t.device).set_(t.untyped_storage())
        views.append(flat[: flat.numel() // 4 * 4].view(torch.float32))
    for v in views:
        v.sum()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for v in views:
        v.sum()
    e.record()
    e.synchronize()
    return sum(v.numel() * 4 for v in views) / (s.elapsed_time(e) * 1e-3) / 1e12


def report(model, device=None, sink=print) -> dict | None:
    """Print ``[mem-cls]`` per buffer class: GiB, the boot phase its segments came from, and the
    read TB/s of its largest tensors."""
    import torch

    if not enabled() or not torch.cuda.is_available():
        return None
    mark("report", device, sink)
    starts = sorted(_segs)
    cls_of: dict[int, str] = {}
    cls = classes(model)
    for name, ts in cls.items():
        for t in ts:
            if not t.is_cuda:
                continue
            ptr = t.untyped_storage().data_ptr()
            i = bisect.bisect_right(starts, ptr) - 1
            if i >= 0 and ptr < starts[i] + _segs[starts[i]]["size"]:
                cls_of.setdefault(starts[i], name)
    summary: dict[str, dict] = {}
    for addr in starts:
        s = _segs[addr]
        s["cls"] = cls_of.get(addr, "graph_pool" if s["graph_pool"] else "other")
        c = summary.setdefault(s["cls"], {"gib": 0.0, "phases": {}})
        c["gib"] += s["size"] / 2**30
        c["phases"][s["phase"]] = round(c["phases"].get(s["phase"], 0.0) + s["size"] / 2**30, 3)
    for name, ts in cls.items():
        if name in summary:
            tbs = _read_tbs(ts)
            summary[name]["read_tbs"] = round(tbs, 3) if tbs else None
    for name, c in sorted(summary.items()):
        c["gib"] = round(c["gib"], 2)
        sink(f"[mem-cls] {json.dumps({'rank': _rank, 'cls': name, **c})}")
    out_dir = flags.get("QB_MEM_TIMELINE_DIR")
    if out_dir:
        (Path(out_dir) / f"mem_segments_rank{_rank}.json").write_text(
            json.dumps(sorted(_segs.values(), key=lambda s: s["addr"])))
    return summary


def device_free_gib(device=None) -> float:
    import torch

    return torch.cuda.mem_get_info(device)[0] / 2**30


def preflight(min_free_gib: float | None = None, wait_s: float | None = None, read=None,
              sleep=time.sleep, clock=time.monotonic, sink=print) -> None:
    """Block until the device has ``min_free_gib`` free; ``RuntimeError`` after ``wait_s``."""
    min_free_gib = flags.get("QB_BOOT_MEM_PREFLIGHT_GIB") if min_free_gib is None else min_free_gib
    wait_s = flags.get("QB_BOOT_MEM_PREFLIGHT_WAIT_S") if wait_s is None else wait_s
    if min_free_gib <= 0:
        return
    read = read or device_free_gib
    deadline = clock() + wait_s
    while True:
        free = read()
        if free >= min_free_gib:
            sink(f"[mem-preflight] ok: {free:.1f} GiB free >= {min_free_gib}")
            return
        if clock() >= deadline:
            raise RuntimeError(f"[mem-preflight] device has {free:.1f} GiB free, below {min_free_gib} GiB after "
                               f"{wait_s:.0f} s: another process still holds device memory")
        sleep(2)
