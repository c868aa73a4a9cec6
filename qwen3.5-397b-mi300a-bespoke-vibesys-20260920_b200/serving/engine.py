"""Model construction for serving and benchmarking (one place for pool sizing).

``build_model`` creates this rank's ``Model`` either from a checkpoint directory (the published
safetensors layout) or with random-init weights of a named geometry (``full`` / ``tiny``), and
sizes the paged KV pool, lane count and snapshot pool from the arguments. On a single GPU the
full geometry does not fit (205 GB of MXFP4 experts); ``distinct_expert_layers`` then lets
later layers reuse earlier layers' expert storage, sized from free memory.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.config import Qwen35Config, full_config, load_config, tiny_config
from ..models.qwen35 import Model
from ..models.weights import expert_bytes_per_layer, load_weights, random_weights
from ..parallel.comm import Comm
from ..parallel.plan import plan
from ..utils import flags
from ..utils.memreport import BootMemory, pool_plan


@dataclass
class PoolSpec:
    lanes: int = 32
    max_seq: int = 16384
    block_size: int = 16
    kv_tokens: int | None = None  # paged KV capacity (tokens); default lanes * max_seq
    snapshots: int | None = None  # default 2 * lanes + 16


def pool_bytes(cfg: Qwen35Config, p, spec: PoolSpec) -> tuple[int, int, int]:
    kv_tokens = spec.kv_tokens or spec.lanes * spec.max_seq
    num_blocks = kv_tokens // spec.block_size + 1
    snaps = spec.snapshots or 2 * spec.lanes + 16
    kv = num_blocks * spec.block_size * len(cfg.full_layers) * 2 * p.kv.count * cfg.head_dim * 2
    nv, nk = p.dn_v.count, p.dn_k.count
    conv_ch = 2 * nk * cfg.dn_k_dim + nv * cfg.dn_v_dim
    per_state = len(cfg.linear_layers) * (nv * cfg.dn_k_dim * cfg.dn_v_dim * 4 + conv_ch * (cfg.conv_kernel - 1) * 2)
    return kv, (spec.lanes + snaps) * per_state, num_blocks


def prefill_graph_widths(flag: str) -> list[int]:
    """Widths of the captured single-segment prefill steps from ``QB_PREFILL_GRAPHS`` ("512,2048"; empty:
    none)."""
    return [int(w) for w in str(flag or "").replace(" ", "").split(",") if w.strip().isdigit() and int(w) > 0]


def mixed_graph_shapes(flag: str) -> list[tuple[int, int]]:
    """(decode rows, prefill width) of the captured mixed steps from ``QB_MIXED_GRAPHS``
    ("32:256,32:512"; empty: none)."""
    out = []
    for part in str(flag or "").replace(" ", "").split(","):
        b, _, w = part.partition(":")
        if b.isdigit() and w.isdigit() and int(b) > 0 and int(w) > 0:
            out.append((int(b), int(w)))
    return out


def nvls_min_rows(flag: int, world: int) -> int:
    """Smallest all-reduce (rows) that takes the NVLS kernel, 0 for never. ``flag`` -1 chooses by
    world size from the collective sweep (hidden 4096, device time, max over ranks): at 8 ranks the
    switch-reduced kernel beats the sequence-parallel one from 1024 rows (68 vs 71 us at 1024, 108
    vs 126 at 2048, 353 vs 409 at 8192) and loses below (55 vs 51 us at 512); at 2 and 4 ranks it
    never wins (each GPU's share of the reduction is already half or a quarter of the message)."""
    if flag >= 0:
        return flag
    return 1024 if world >= 8 else 0


def build_model(model: str, rank: int, world: int, device: torch.device, spec: PoolSpec,
                dtype=torch.bfloat16, seed: int = 0, with_mtp: bool = False, comm: Comm | None = None,
                reserve_bytes: float = 14e9, graphs: bool | None = None):
    """``model`` is a checkpoint directory, ``"full"`` or ``"tiny"`` (random init). On CUDA the
    result is wrapped in a ``GraphRunner`` (captured decode buckets) unless ``graphs=False``;
    every rank must call this in the same order, since capture runs the collectives."""
    if graphs is None:
        graphs = device.type == "cuda" and flags.get("QB_GRAPHS")
    mem = BootMemory(rank, device)
    mem.phase("start")
    if model in ("full", "tiny"):
        cfg = full_config() if model == "full" else tiny_config()
    else:
        cfg = load_config(model)
    p = plan(cfg, rank, world)
    kv, state, num_blocks = pool_bytes(cfg, p, spec)
    distinct = None
    if model == "full" and device.type == "cuda":
        total = torch.cuda.get_device_properties(device).total_memory
        dense = 20e9 / world + 4e9
        if with_mtp:  # the MTP layer: bf16 (or MXFP4) experts of this rank plus its dense part
            per = 3 * cfg.hidden * cfg.moe_inter
            dense += p.experts.count * (2 * per if cfg.mtp_experts_bf16 else per // 2 + per // 32) + 1e9
        budget = total - dense - kv - state - reserve_bytes
        n = max(1, min(cfg.layers, int(budget // expert_bytes_per_layer(cfg, p))))
        distinct = None if n >= cfg.layers else n
    if model in ("full", "tiny"):
        w = random_weights(cfg, p, device, dtype, seed=seed, with_mtp=with_mtp, distinct_expert_layers=distinct)
    else:
        w = load_weights(model, cfg, p, device, dtype, with_mtp=with_mtp)
    mem.phase("weights")
    if comm is None:
        comm = Comm(rank, world, None, device)
        if world > 1 and device.type == "cuda" and comm.mode == "fused":
            from ..parallel.symm import SymmComm, SymmUnavailable

            rows = flags.get("QB_SYMM_MAX_ROWS")
            sp_rows = flags.get("QB_SP_MAX_ROWS")  # prefill-sized messages: sequence-parallel kernel
            try:
                comm.symm = SymmComm(rank, world, device, max_rows=rows, hidden=cfg.hidden, sp_rows=sp_rows)
            except SymmUnavailable as e:  # raised on every rank together: all fall back to NCCL
                print(f"[rank {rank}] fused collectives unavailable, using NCCL: {e}", flush=True)
                comm.symm = None
            nvls_min = nvls_min_rows(flags.get("QB_NVLS_MIN_ROWS"), world)
            if comm.symm is not None and nvls_min > 0 and sp_rows > 0:
                # messages of nvls_min rows and more take the switch-reduced kernel; all ranks
                # keep the peer-memory kernels together when the fabric has no multicast
                if not comm.symm.enable_nvls(rows_cap=sp_rows, min_rows=nvls_min):
                    print(f"[rank {rank}] NVLS unavailable: large messages stay on the peer-memory kernel",
                          flush=True)
    m = Model(cfg, w, p, comm, device=device, dtype=dtype,
              max_batch=spec.lanes + (1 if graphs else 0), max_seq=spec.max_seq, block_size=spec.block_size,
              num_blocks=num_blocks, num_snapshots=spec.snapshots or 2 * spec.lanes + 16)
    mem.phase("pools")
    if device.type == "cuda":
        from ..utils.devstatus import StatusWatch

        m.status_watch = StatusWatch(device, flags.get("QB_STATUS_EVERY"))
    if graphs:
        from .graphs import GraphRunner

        g = GraphRunner(m)
        g.prepare()
        widths = prefill_graph_widths(flags.get("QB_PREFILL_GRAPHS"))
        if widths:
            g.prepare_prefill(widths)
        shapes = mixed_graph_shapes(flags.get("QB_MIXED_GRAPHS"))
        if shapes:
            g.prepare_mixed(shapes)
        mem.phase("graphs")
        pool_plan(m, rank)
        return g, distinct
    pool_plan(m, rank)
    return m, distinct
