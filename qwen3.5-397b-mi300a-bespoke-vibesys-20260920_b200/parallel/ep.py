"""Expert-parallel MoE over NVLink peer memory (dispatch -> grouped expert GEMMs -> combine).

Each rank holds a slice of the experts and its own tokens (for example the rows a
sequence-parallel collective left it, or a data-parallel batch). ``EPComm.moe`` sends every token
row to the ranks that own at least one of its experts, straight into their receive areas in a
symmetric IPC-mapped region; each rank runs the block-scaled grouped GEMMs of its experts over the
rows it received; the routing-weighted partial outputs are read back by the tokens' owners and
summed in rank order. Kernels and the protocol: ``csrc/ep.cu``. The expert GEMMs are those of
``ops.moe_routed`` (``csrc/moe_mx.cu``), fed directly from the receive area.

Reference counterpart: none as such; the reference replicates activations and folds the routed
sum into its tensor-parallel all-reduce (``model.py:2770-2790``); this module is the
dispatch/combine form its parallelism notes ask for (512 experts over 8 GPUs).
"""

from __future__ import annotations

import torch

from ..ops import core as ops
from ..ops._ext import ext
from .symm import alloc_region


class EPComm:
    """Symmetric receive areas for up to ``cap`` tokens per rank (``top_k`` experts each) of
    width ``hidden``; ``experts`` in total, split evenly over ``world`` ranks."""

    def __init__(self, rank: int, world: int, device, cap: int, hidden: int, top_k: int, experts: int,
                 group=None, timeout_s: float = 10.0, bases: list[int] | None = None):
        if world > 8 or experts % world:
            raise ValueError("expert parallelism over up to 8 ranks with an even expert split")
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.cap, self.hidden, self.top_k, self.experts = cap, hidden, top_k, experts
        self.per_rank = experts // world
        self.timeout_s = timeout_s
        nbytes = ext().ep_region_bytes(world, cap, hidden, top_k)
        if bases is not None:  # regions made by the caller (tests)
            self.bases, self.own, self.opened = list(bases), 0, []
        elif world == 1:
            ptr, _ = ext().symm_alloc(nbytes)
            self.bases, self.own, self.opened = [ptr], ptr, []
        else:
            self.bases, self.own, self.opened = alloc_region(rank, world, self.device, nbytes, group)
        self.state = torch.zeros(4, dtype=torch.int32, device=self.device)  # [epoch, dispatch blocks done]
        self.calls = 0

    def region_bytes(self) -> int:
        return ext().ep_region_bytes(self.world, self.cap, self.hidden, self.top_k)

    def moe(self, h: torch.Tensor, topw: torch.Tensor, topi: torch.Tensor, experts: dict) -> torch.Tensor:
        """Routed-expert output for this rank's tokens ``h`` [T, H] (T <= cap) with routing
        ``topw`` / ``topi`` [T, k] over all experts; ``experts`` holds this rank's slice
        (MXFP4 codes and scales). Every rank calls this together (eager; not graph-captured:
        the receive-area parity is chosen on the host)."""
        if "s13c" not in experts:
            ops.prepare_experts(experts)
        tiled = bool(experts.get("tiled", False))
        par = (self.calls + 1) & 1  # the device epoch after this call's increment, mod 2
        out = ext().ep_moe(self.bases, self.rank, h.contiguous(), topw.float().contiguous(),
                           topi.int().contiguous(), experts["w13"], experts["s13c"], experts["w2"], experts["s2c"],
                           self.rank * self.per_rank, self.per_rank, tiled, self.cap, self.per_rank, par, self.state,
                           self.timeout_s)
        self.calls += 1
        return out

    def close(self) -> None:
        for p in self.opened:
            ext().symm_close(p)
        self.opened = []
        if self.own:
            ext().symm_free(self.own)
            self.own = 0
