"""Process group and the collectives the model runtime issues.

One OS process per GPU (or per gloo CPU rank in tests). ``init`` creates the
``torch.distributed`` group (NCCL on CUDA, gloo on CPU, rendezvous on 127.0.0.1 by default).
``Comm`` is what the model calls:

* ``all_reduce`` - sum of row-parallel partials, accumulated in fp32 and rounded once to the
  activation dtype (reference ``tp.py:50-64``);
* ``allreduce_add_rmsnorm`` - the per-layer hot collective: all-reduce of the mixer / MoE
  partials, residual add, and the next RMSNorm. On CUDA with ``world > 1`` this is one fused
  kernel over symmetric peer memory (``parallel.symm``); ``QB_COMM=nccl`` selects the NCCL
  baseline (all-reduce, then the fused add+norm kernel);
* ``all_gather_last`` - vocab-parallel logits (reference ``tp.py:304-321``);
* ``argmax_gather`` - vocab-parallel greedy token: local (max, index) pairs, all-gathered.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from ..ops import core as ops
from ..utils import flags


def env_rank_world() -> tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def init(backend: str | None = None, rank: int | None = None, world: int | None = None,
         timeout_s: float = 600.0) -> tuple[int, int]:
    """Initialise the default process group from the environment (idempotent)."""
    r, w, local = env_rank_world()
    rank = r if rank is None else rank
    world = w if world is None else world
    if world <= 1 or dist.is_initialized():
        return (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)
    # programmatic dependent launches of the GEMMs are measured and tested on one GPU; a
    # multi-rank run keeps plain launches unless QB_PDL is set explicitly (every rank alike)
    flags.put("QB_PDL", 0, only_if_unset=True)
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
        from ..utils.affinity import pin_device

        note = pin_device(local)  # host threads on the CPUs next to this rank's GPU
        if note:
            print(f"[cpu-affinity] rank {rank}: {note}", flush=True)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world


class Comm:
    """Collectives of one tensor-parallel group (``world == 1`` makes every call local)."""

    def __init__(self, rank: int = 0, world: int = 1, group=None, device=None, symm=None):
        self.rank, self.world, self.group = rank, world, group
        self.device = device
        self.symm = symm  # parallel.symm.SymmComm for the fused CUDA kernels, or None
        self.mode = flags.get("QB_COMM")
        self.sp_gemm = flags.get("QB_SP_GEMM")
        self.ag_gemm = flags.get("QB_AG_GEMM")
        self.sp_res_local = flags.get("QB_SP_RES_LOCAL")

    # ------------------------------------------------------------------ primitives
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        y = x.float()
        dist.all_reduce(y, group=self.group)
        return y.to(x.dtype)

    def all_gather_last(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.world)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.world)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, dim=0)

    def broadcast(self, x: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.world > 1:
            dist.broadcast(x, src, group=self.group)
        return x

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    # ------------------------------------------------------------------ fused
    def allreduce_add_rmsnorm(self, partial: torch.Tensor, residual: torch.Tensor, w1p: torch.Tensor,
                              eps: float, gather_out: bool = False, res_local: bool = False
                              ) -> tuple[torch.Tensor, torch.Tensor]:
        """``residual + sum_ranks(partial)`` and its RMSNorm; returns (residual, normed). With
        ``gather_out`` (the caller's only use of ``normed`` is one projection) and
        ``QB_AG_GEMM``, sequence-parallel sizes return the owner-only form: ``residual`` valid on
        this rank's rows only and ``normed`` a ``GatheredRows`` whose ``linear`` gathers inside
        the GEMM. With ``res_local`` (the residual is next read only by another sequence-parallel
        call) and ``QB_SP_RES_LOCAL``, the sequence-parallel kernel gathers only the normed rows and
        ``residual`` stays valid on this rank's rows."""
        if self.world > 1 and partial.is_cuda and self.symm is not None and self.mode == "fused":
            rows = residual.numel() // residual.shape[-1]
            own = gather_out and self.ag_gemm and self.symm.gathers(rows)
            got = self.symm.allreduce_add_rmsnorm(partial, residual, w1p, eps, gather_out=own,
                                                  res_local=res_local and self.sp_res_local)
            if got is not None:
                return got
        summed = self.all_reduce(partial)
        return ops.add_rmsnorm(summed, residual, w1p, eps)

    def fuses_linear(self, rows: int) -> bool:
        """True when ``linear_allreduce_add_rmsnorm`` runs the projection and the all-reduce as
        the fused GEMM -> reduce-scatter pair (multi-rank, fused comm, prefill-sized rows)."""
        return (self.world > 1 and self.symm is not None and self.mode == "fused" and self.sp_gemm
                and str(self.device).startswith("cuda") and self.symm.fuses_linear(rows))

    def linear_allreduce_add_rmsnorm(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                                     w1p: torch.Tensor, eps: float, res_local: bool = False
                                     ) -> tuple[torch.Tensor, torch.Tensor]:
        """``residual + sum_ranks(x @ w^T)`` and its RMSNorm, for a row-parallel projection
        (``res_local`` as in ``allreduce_add_rmsnorm``)."""
        if x.is_cuda and self.fuses_linear(residual.numel() // residual.shape[-1]):
            got = self.symm.linear_allreduce_add_rmsnorm(x, w, residual, w1p, eps,
                                                         res_local=res_local and self.sp_res_local)
            if got is not None:
                return got
        return self.allreduce_add_rmsnorm(ops.linear(x, w), residual, w1p, eps, res_local=res_local)

    def argmax_gather(self, local_logits: torch.Tensor, vocab_start: int) -> torch.Tensor:
        """Greedy token ids [B] over vocab-parallel logits (ties: lowest global index)."""
        val, idx = ops.argmax_rows(local_logits)
        idx = idx + vocab_start
        if self.world == 1:
            return idx
        pair = torch.stack([val.float(), idx.float()], dim=-1)  # exact for idx < 2**24
        allp = self.all_gather_rows(pair[None]).view(self.world, -1, 2)
        best = allp[..., 0].argmax(dim=0)  # first rank wins ties = lowest index
        return allp[best, torch.arange(allp.shape[1], device=allp.device), 1].long()
