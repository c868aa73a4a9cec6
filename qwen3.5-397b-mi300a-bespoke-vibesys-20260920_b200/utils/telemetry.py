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


class StepTimer:
    """Per-kind rolling windows of host wall time per scheduler step."""

    def __init__(self, every: int | None = None, sink=print) -> None:
        env = os.environ.get("QB_STEP_TIMING", "0")
        self.every = every if every is not None else (int(env) if env.isdigit() else 0)
        self.sink = sink
        self.win: dict[str, list[tuple[int, float]]] = defaultdict(list)
        self.total: dict[str, list[float]] = defaultdict(lambda: [0, 0.0, 0])
        self.n = 0
        trace = os.environ.get("QB_SERVICE_TRACE")
        self.trace = ServiceTrace(trace) if trace else None

    def record(self, kind: str, tokens: int, seconds: float) -> None:
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
