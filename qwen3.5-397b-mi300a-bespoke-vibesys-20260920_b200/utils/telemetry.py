"""Step timing, device idle-gap metering, per-step service traces and in-graph clock stamps.

All of it is off unless asked for (``QB_STEP_TIMING=<n>`` logs a ``[step-timing]`` line every
``n`` steps; ``QB_SERVICE_TRACE=<path>`` appends one JSON record per scheduler step).
Reference behaviour: ``step_timing.py`` (``GapMeter``, ``ServiceTrace``) and
``decode_stamps.py`` (in-graph stamps; here ``%globaltimer`` stamps written by a CUDA kernel,
``ops.stamp``).
"""

from __future__ import annotations

import json
import os
import threading
import time
from collections import defaultdict

from . import flags


class StepTimer:
    """Per-kind rolling windows of host wall time per scheduler step."""

    def __init__(self, every: int | None = None, sink=print) -> None:
        self.every = every if every is not None else flags.get("QB_STEP_TIMING")
        self.sink = sink
        self.win: dict[str, list[tuple[int, float]]] = defaultdict(list)
        self.total: dict[str, list[float]] = defaultdict(lambda: [0, 0.0, 0])
        self.n = 0
        self.last_kind = None  # kind of the most recent step
        trace = flags.get("QB_SERVICE_TRACE")
        self.trace = ServiceTrace(trace) if trace else None

    def record(self, kind: str, tokens: int, seconds: float) -> None:
        self.last_kind = kind
        t = self.total[kind]
        t[0] += 1
        t[1] += seconds
        t[2] += tokens
        self.n += 1
        if self.trace is not None:
            self.trace.write({"kind": kind, "tokens": tokens, "ms": seconds * 1e3, "t": time.time()})
        if self.every:
            self.win[kind].append((tokens, seconds))
            if self.n % self.every == 0:
                parts = []
                for k, v in sorted(self.win.items()):
                    ms = sum(s for _, s in v) / len(v) * 1e3
                    parts.append(f"{k}: n={len(v)} mean={ms:.2f}ms tok={sum(x for x, _ in v)}")
                self.sink("[step-timing] " + " | ".join(parts))
                self.win.clear()

    def summary(self) -> dict:
        return {k: {"steps": v[0], "seconds": v[1], "tokens": v[2]} for k, v in self.total.items()}


class ServiceTrace:
    """One JSON line per record; writing pauses while ``<path>.pause`` exists."""

    def __init__(self, path: str) -> None:
        self.path = path
        self._lock = threading.Lock()

    def write(self, rec: dict) -> None:
        if os.path.exists(self.path + ".pause"):
            return
        with self._lock, open(self.path, "a") as f:
            f.write(json.dumps(rec) + "\n")


class GapMeter:
    """Device idle time between consecutive steps, from CUDA events, without host syncs.

    ``begin()``/``end()`` bracket each step on the current stream; ``gaps_ms()`` resolves the
    events recorded so far (it syncs only on the newest one)."""

    def __init__(self) -> None:
        import torch

        self.torch = torch
        self.events: list[tuple] = []

    def begin(self) -> None:
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.append([e, None])

    def end(self) -> None:
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.events[-1][1] = e

    def gaps_ms(self) -> list[float]:
        if not self.events:
            return []
        self.events[-1][1].synchronize()
        out = []
        for (a0, a1), (b0, _) in zip(self.events, self.events[1:]):
            out.append(a1.elapsed_time(b0))
        return out


class Stamps:
    """In-graph clock stamps: ``mark(tag)`` ends the current segment of the stream as ``tag``.

    Each mark launches a one-thread kernel that writes ``%globaltimer`` (ns) into its slot of a
    device buffer. Timing events cannot be recorded inside a captured CUDA graph; a stamp can,
    and on one stream it runs after the previous kernel has finished, so the difference between
    consecutive stamps is the stream time of the segment that ended at the later one. Slots are
    assigned at record time, so a captured graph rewrites the same slots on every replay and
    ``segments_ms`` reads the latest replay. Reference behaviour: ``decode_stamps.py:43-76``
    (``Recorder``, ``mark``, ``segments_ms``), there with the 100 MHz ``s_memrealtime`` counter.
    """

    def __init__(self, device, capacity: int = 4096, detail: bool = False) -> None:
        import torch

        self.buf = torch.zeros(capacity, dtype=torch.int64, device=device)
        self.tags: list[str] = []
        self.detail = detail  # also stamp between the kernels inside a layer part

    def mark(self, tag: str) -> None:
        from ..ops import core as ops

        k = len(self.tags)
        if k >= self.buf.numel():
            raise RuntimeError("Stamps: capacity exceeded")
        self.tags.append(tag)
        ops.stamp(self.buf, k)

    def reset(self) -> None:
        self.tags = []

    def segments_ms(self) -> list[tuple[str, float]]:
        """``(tag, ms)`` per segment: the time from the previous stamp to this one."""
        t = self.buf[: len(self.tags)].tolist()
        return [(self.tags[k], (t[k] - t[k - 1]) * 1e-6) for k in range(1, len(self.tags))]

    def by_tag_ms(self) -> dict[str, float]:
        """Segment times summed per tag, plus ``total`` (first stamp to last)."""
        out: dict[str, float] = defaultdict(float)
        for tag, ms in self.segments_ms():
            out[tag] += ms
        out["total"] = sum(ms for _, ms in self.segments_ms())
        return dict(out)
