"""Boot memory report and static pool plan (diagnostics; off unless ``QB_MEM_REPORT=1``).

``BootMemory.phase(name)`` prints one ``[mem]`` line per boot phase (weights loaded, pools
allocated, graphs captured): free and total device memory from the driver, the bytes the
caching allocator holds in tensors and in reserve, what each grew by since the previous phase,
and the process's resident host memory. ``pool_plan(model)`` prints one ``[pool-plan]`` line with
the bytes of every static pool the model owns, computed from the model's own attributes: weights
split into embedding / LM head, full-attention, DeltaNet, routed experts, shared expert and MTP
parts (storage shared between layers counted once), the paged KV cache, the DeltaNet lane state
and the snapshot pool. On a 180 GB B200 the KV pool is what is left after the weights, so this
is the line to read when a boot serves fewer tokens than expected.

Reference behaviour: the reference logs a boot memory timeline for MI300A's unified memory
(``mem_timeline.py``); this module reports device residency per pool instead.
"""

from __future__ import annotations

import os
import time

from . import flags

_GIB = float(1 << 30)


def enabled() -> bool:
    return bool(flags.get("QB_MEM_REPORT"))


def _rss_gib() -> float | None:
    try:
        with open("/proc/self/statm") as f:
            pages = int(f.read().split()[1])
        return pages * os.sysconf("SC_PAGE_SIZE") / _GIB
    except (OSError, ValueError, IndexError):
        return None


class BootMemory:
    """``[mem]`` lines at named boot phases of one rank (no-ops when disabled or off-GPU)."""

    def __init__(self, rank: int, device, sink=print, force: bool | None = None) -> None:
        self.rank = rank
        self.device = device
        self.sink = sink
        self.on = enabled() if force is None else force
        self.t0 = time.perf_counter()
        self.prev: tuple[int, int] | None = None
        self.phases: list[dict] = []

    def phase(self, name: str) -> dict | None:
        import torch

        dev = self.device
        if not self.on or getattr(dev, "type", "cpu") != "cuda":
            return None
        torch.cuda.synchronize(dev)
        free, total = torch.cuda.mem_get_info(dev)
        alloc, reserved = torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)
        d_alloc = alloc - self.prev[0] if self.prev else alloc
        d_res = reserved - self.prev[1] if self.prev else reserved
        self.prev = (alloc, reserved)
        rec = {"phase": name, "t_s": round(time.perf_counter() - self.t0, 2), "free_gib": round(free / _GIB, 2),
               "total_gib": round(total / _GIB, 2), "tensors_gib": round(alloc / _GIB, 2),
               "reserved_gib": round(reserved / _GIB, 2), "grew_tensors_gib": round(d_alloc / _GIB, 2),
               "grew_reserved_gib": round(d_res / _GIB, 2)}
        rss = _rss_gib()
        if rss is not None:
            rec["host_rss_gib"] = round(rss, 2)
        self.phases.append(rec)
        self.sink(f"[mem] rank={self.rank} " + " ".join(f"{k}={v}" for k, v in rec.items()))
        return rec


def _tensor_bytes(v, seen: set) -> int:
    """Bytes of the tensors held by ``v`` (a tensor, or a dict / list / tuple of them), counting
    each storage once across calls that share ``seen``."""
    import torch

    if isinstance(v, torch.Tensor):
        st = v.untyped_storage()
        key = (st.data_ptr(), v.device.type, v.device.index)
        if key in seen or st.nbytes() == 0:
            return 0
        seen.add(key)
        return st.nbytes()
    if isinstance(v, dict):
        return sum(_tensor_bytes(x, seen) for x in v.values())
    if isinstance(v, (list, tuple)):
        return sum(_tensor_bytes(x, seen) for x in v)
    return 0


def pool_bytes_of(model) -> dict[str, int]:
    """Bytes per static pool of a ``models.qwen35.Model`` (or a runner wrapping one)."""
    from ..models.config import FULL

    m = getattr(model, "model", model)
    w = m.w
    seen: set = set()
    out: dict[str, int] = {}

    def add(k: str, v) -> None:
        out[k] = out.get(k, 0) + _tensor_bytes(v, seen)

    add("embed_lmhead", [w.get("embed"), w.get("lm_head"), w.get("final_norm")])
    for L in w["layers"]:
        mixer = "attention" if L.get("kind") == FULL else "deltanet"
        for key, val in L.items():
            if key == "experts":
                add("experts", val)
            elif key.startswith("w_sh") or key.startswith("w_rsh") or key == "w_router":
                add("router_shared", val)
            else:
                add(mixer, val)
    if "mtp" in w:
        add("mtp_weights", w["mtp"])
    add("kv_cache", list(m.k_cache) + list(m.v_cache))
    add("deltanet_lanes", [m.conv_state, m.rec_state])
    add("snapshots", [m.snap_conv, m.snap_rec])
    return out


def pool_plan(model, rank: int = 0, sink=print, force: bool | None = None) -> dict | None:
    """Print ``[pool-plan]`` (GiB per pool, KV capacity in tokens and blocks, lanes, snapshot
    slots); returns the record, or ``None`` when disabled."""
    on = enabled() if force is None else force
    if not on:
        return None
    m = getattr(model, "model", model)
    b = pool_bytes_of(m)
    rec = {k: round(v / _GIB, 3) for k, v in sorted(b.items())}
    rec.update({"total_gib": round(sum(b.values()) / _GIB, 3), "kv_tokens": m.num_blocks * m.block_size,
                "kv_blocks": m.num_blocks, "lanes": m.max_batch, "snapshot_slots": m.num_snapshots})
    sink(f"[pool-plan] rank={rank} " + " ".join(f"{k}={v}" for k, v in rec.items()))
    return rec
