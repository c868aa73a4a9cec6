"""Typed registry of every ``QB_*`` environment flag the framework reads.

Each flag is declared once with its type, default and meaning; code reads it through ``get``
(Python) or ``getenv`` (the CUDA launchers, marked ``native``). ``snapshot()`` returns the values
of the flags that must agree across ranks (they change a kernel's numerics, which collective runs
at a given size, or which steps are captured), and ``signature()`` hashes them: the multi-rank
driver folds that hash into its pool signature, so ranks started with different flags refuse to
run together instead of computing different numbers or waiting in different collectives.

Reference behaviour: the reference reads ``SEED_*`` variables ad hoc across its modules
(``mem_timeline.py:22``, ``host_numa.py:13``, ``step_timing.py``); here they are declared in one
place so a test can check that no module reads an undeclared name.
"""

from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Flag:
    name: str
    kind: type  # bool, int, float or str
    default: object
    doc: str
    lockstep: bool = False  # must agree across ranks: part of the pool signature
    native: bool = False  # read by the C++/CUDA side with getenv


_FLAGS: dict[str, Flag] = {}


def _def(name, kind, default, doc, lockstep=False, native=False) -> None:
    _FLAGS[name] = Flag(name, kind, default, doc, lockstep, native)


# ---- kernels and numerics
_def("QB_BOUNDS", bool, False, "load the debug build of the extension (_build_bounds: index checks and scratch "
     "canaries recorded in the device status word; build it with python -m qwen35_b200.ops.build --bounds)")
_def("QB_MOE_IMPL", str, "mx", "routed-expert kernel: mx (block-scaled fp8 tcgen05), f16 (fp4 decoded to "
     "f16 in TMEM), bf16 (dequantised weights)", lockstep=True)
_def("QB_MX_BN_MAX", int, 64, "largest token tile of the block-scaled MoE kernel", native=True)
_def("QB_MX_TILED", bool, True, "block-scaled MoE: expert codes re-laid tile-contiguous at load")
_def("QB_MX_WIDE", bool, True, "block-scaled MoE, tiled codes: one TMA box per operand and stage", native=True)
_def("QB_DN_VSPLIT", int, 0, "chunked DeltaNet state kernel: CTAs per value head (1: all 128 value columns, "
     "2: 64 each; 0: two when that packs the waves better)", native=True)
_def("QB_GEMM_BN_FIT", int, 1, "dense GEMM above 128 tokens: token-tile width fitted to the SM waves (0: the widest "
     "width, the tokens split evenly over ceil(T / 256) tiles)", native=True)
_def("QB_PDL", int, 1, "dense GEMMs launched as programmatic dependents (their prologue overlaps the previous "
     "kernel, which signals early; 0: plain launches); a multi-rank process group sets 0 unless given",
     lockstep=True, native=True)
_def("QB_MX_K2", int, -1, "block-scaled MoE, wide path: two 128-K atoms per pipeline stage (1), one (0), "
     "or two for token tiles of at most 32 rows (-1)", native=True)
_def("QB_MX_PROBE", bool, False, "block-scaled MoE: count the producer / MMA wait cycles (diagnostic)",
     native=True)
_def("QB_MOE_BN_MAX", int, 64, "largest token tile of the f16-decode MoE kernel", native=True)
_def("QB_MOE_SMEM_A", bool, False, "f16-decode MoE: stage decoded weights in shared memory", native=True)
_def("QB_FA", bool, True, "tcgen05 flash attention for full-attention layers (else the CUDA-core kernel)",
     lockstep=True)
_def("QB_FA_SPLITS", int, 0, "flash attention: key-range splits per tile (0: enough CTAs for one wave)",
     lockstep=True)
_def("QB_DN_DECODE", str, "", "DeltaNet decode mixer state path: reg (registers), sm (shared memory by bulk copies); "
     "empty: sm from 16 lanes up", native=True)
_def("QB_DN_PREFILL", str, "auto", "DeltaNet prefill segments: tc (chunked WY form, state in tensor memory, "
     "tcgen05 products), recurrence (fp32 token recurrence), chunked_fp32 (chunked WY form on CUDA cores), auto "
     "(tc up to 32 value heads per rank, and at more heads for batches whose longest segment has 128 tokens or more, "
     "else recurrence)",
     lockstep=True)
_def("QB_GRAPHS", bool, True, "capture decode steps in CUDA graphs", lockstep=True)
_def("QB_PREFILL_ORDER", str, "shortest", "scheduler: order prefill flights are packed in: shortest (fewest "
     "pending prompt tokens first, with aging) or fifo (admission order)")
_def("QB_PREFILL_PACK", str, "fill", "scheduler: fill (pack prefill chunks up to the token budget) or finish "
     "(once a step gives some request its first token, add only requests whose prompt also completes in it)")
_def("QB_OVERLAP", bool, True, "scheduler: launch decode step n+1 (tokens fed back on the device) before reading "
     "step n back", lockstep=True)
_def("QB_MTP_DEVICE_ACCEPT", bool, True, "speculative rounds: accepted lengths computed on the device and the whole "
     "round (draft, verify, accept, commit) replayed as one graph, read back once", lockstep=True)
_def("QB_PREFILL_GRAPHS", str, "", "widths (comma-separated token counts) of captured single-segment prefill steps, "
     "replayed for one segment of exactly that length (empty: prefill runs eagerly)", lockstep=True)
_def("QB_MIXED_GRAPHS", str, "", "captured mixed steps as decode-rows:prefill-width pairs (\"32:256,32:512\"): a mixed "
     "step with at most that many decode lanes and one prefill segment of exactly that width replays (empty: eager)",
     lockstep=True)
_def("QB_GREEDY_HEAD", bool, True, "greedy decode ids from each rank's (max, index) over its vocabulary slice, "
     "gathered as 8-byte pairs (off: the full logits rows are all-gathered, then the argmax)", lockstep=True)
_def("QB_MOE_FUSE_SHARED", bool, True, "MoE: the shared expert's gated rows are added in the routed combine kernel "
     "(off: a separate gate-and-add kernel)", lockstep=True)
_def("QB_FOLD_SUFFIX", bool, False, "scheduler: the chat template's generation suffix after the turn-open boundary "
     "is fed through the following decode steps (their sampled ids discarded) instead of a prefill step of its own")
_def("QB_PREFILL_ACCUM", bool, False, "scheduler: while at least QB_PREFILL_ACCUM_MIN_DECODE lanes decode, hold "
     "queued prefill until QB_PREFILL_ACCUM_TOKENS tokens are packable or the oldest has waited "
     "QB_PREFILL_ACCUM_WAIT_MS")
_def("QB_PREFILL_ACCUM_TOKENS", int, 1024, "scheduler: packable prefill tokens that fire a held prefill step")
_def("QB_PREFILL_ACCUM_WAIT_MS", float, 400.0, "scheduler: longest hold of a queued prefill (host clock)")
_def("QB_PREFILL_ACCUM_MIN_DECODE", int, 48, "scheduler: decoding lanes below which prefill fires at once")
_def("QB_MIXED", bool, False, "scheduler: decode steps also carry prefill chunks in the same forward")
# ---- collectives and multi-rank plumbing
_def("QB_COMM", str, "fused", "tensor-parallel all-reduce: fused (peer-memory kernels) or nccl", lockstep=True)
_def("QB_SYMM_MAX_ROWS", int, 512, "rows of the one-shot fused all-reduce buffers", lockstep=True)
_def("QB_SP_MAX_ROWS", int, 4096, "rows of the sequence-parallel fused all-reduce buffers (0: off)",
     lockstep=True)
_def("QB_NVLS_MIN_ROWS", int, -1, "all-reduce messages of at least this many rows use the NVLS (multimem) kernel "
     "(0: never; -1: by world size, from 1024 rows at 8 ranks and more, where the switch reduction measured "
     "ahead of the sequence-parallel kernel, never below)", lockstep=True)
_def("QB_SP_RES_LOCAL", bool, False, "prefill: the sequence-parallel all-reduce keeps the residual on each rank's own "
     "rows (only the normed rows are gathered) except in a forward's last all-reduce", lockstep=True)
_def("QB_AG_GEMM", bool, False, "prefill: the all-reduce after the MoE leaves the all-gather to the next layer's "
     "input projection, which pulls every rank's normed rows over NVLink inside its GEMM (sequence-parallel sizes)",
     lockstep=True)
_def("QB_SP_GEMM", bool, True, "prefill: fuse the mixers' output projection into the sequence-parallel all-reduce "
     "(GEMM epilogue stores rows into their owners' peer slots)", lockstep=True)
_def("QB_CMD_CHANNEL", str, "shm", "leader -> worker command channel: shm (shared-memory ring) or gloo (broadcast)",
     lockstep=True)
_def("QB_STATUS_EVERY", int, 64, "read the kernels' device status word every n model steps (0: never); a "
     "nonzero code aborts the requests in flight (rank 0) or ends the worker")
# ---- diagnostics (off by default; none of them changes a number)
_def("QB_STEP_TIMING", int, 0, "log a [step-timing] line every n scheduler steps (0: off)")
_def("QB_SERVICE_TRACE", str, "", "append one JSON record per scheduler step to this path")
_def("QB_STAMPS", bool, False, "in-graph %globaltimer stamps at layer boundaries")
_def("QB_MEM_REPORT", bool, False, "print a [mem] line at each boot phase and a [pool-plan] line (bytes per "
     "static pool)")
_def("QB_CPU_AFFINITY", bool, False, "restrict each rank's host threads to the CPUs local to its GPU (sysfs "
     "local_cpulist)")
_def("QB_GRAPH_LOG", bool, False, "print a [graph-capture] line per captured decode bucket (kernels, seconds)")
_def("QB_CACHE_STATS", int, 0, "log a [cache-stats] line (session-cache admissions, hit tokens) every n finished "
     "requests (0: off)")
_def("QB_FAULT_ENDPOINT", bool, False, "expose POST /debug/fault (accuracy-gate calibration faults)")


def registry() -> dict[str, Flag]:
    return dict(_FLAGS)


def _parse(f: Flag, raw: str):
    if f.kind is bool:
        return raw.strip().lower() in ("1", "true", "yes", "on")
    if f.kind is int:
        return int(raw)
    if f.kind is float:
        return float(raw)
    return raw


def get(name: str, env: dict | None = None):
    """The flag's value from ``env`` (default ``os.environ``), parsed to its type; its default
    when unset or empty. Reading an undeclared name is an error."""
    f = _FLAGS.get(name)
    if f is None:
        raise KeyError(f"undeclared flag {name}")
    raw = (os.environ if env is None else env).get(name)
    if raw is None or raw == "":
        return f.default
    try:
        return _parse(f, raw)
    except ValueError as e:
        raise ValueError(f"{name}={raw!r}: expected {f.kind.__name__}") from e


def put(name: str, value, only_if_unset: bool = False) -> None:
    """Set a declared flag in this process's environment (which child processes inherit and the
    native code reads), checking that the value parses; with ``only_if_unset`` an explicit
    setting of the user wins."""
    f = _FLAGS.get(name)
    if f is None:
        raise KeyError(f"undeclared flag {name}")
    raw = str(int(value) if isinstance(value, bool) else value)
    if raw:
        _parse(f, raw)
    if only_if_unset and os.environ.get(name) not in (None, ""):
        return
    os.environ[name] = raw


def snapshot(env: dict | None = None, numerics_only: bool = True) -> dict:
    return {n: get(n, env) for n, f in sorted(_FLAGS.items()) if f.lockstep or not numerics_only}


def signature(env: dict | None = None) -> str:
    return hashlib.sha256(json.dumps(snapshot(env), sort_keys=True).encode()).hexdigest()[:16]


def describe() -> str:
    """One line per flag: name, type, default, meaning (``python -m ... utils.flags``)."""
    rows = []
    for f in sorted(_FLAGS.values(), key=lambda f: f.name):
        tag = " [native]" if f.native else ""
        rows.append(f"{f.name:30s} {f.kind.__name__:5s} default={f.default!r:8s} {f.doc}{tag}")
    return "\n".join(rows)


if __name__ == "__main__":
    print(describe())
