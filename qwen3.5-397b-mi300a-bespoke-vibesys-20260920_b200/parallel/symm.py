"""Symmetric peer memory and the fused collective kernels' host side.

Each rank allocates one device region (``cudaMalloc``), exports it with ``cudaIpcGetMemHandle``,
and maps every peer's region (``cudaIpcOpenMemHandle``), so a kernel on any rank can load and
store every rank's region directly over NVLink / NVSwitch. ``SymmComm.allreduce_add_rmsnorm``
launches the one-shot fused kernel in ``csrc/comm.cu``: all-reduce of the row-parallel partials
(rank-order fp32 sum, identical bits on every rank), residual add and RMSNorm in one kernel,
graph-capturable (the call epoch lives in device memory). Waits on peers are bounded
(``timeout_s``); an expired wait sets the device status word instead of hanging.
Reference counterpart: ``allreduce_custom.py`` (IPC buffers, one-shot residual-norm kernel,
device call counter).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext

MAX_BLOCKS = 296  # two CTAs per SM on a 148-SM B200


class SymmComm:
    def __init__(self, rank: int, world: int, device, max_rows: int, hidden: int, group=None,
                 timeout_s: float = 10.0, bases: list[int] | None = None):
        if world > 8:
            raise ValueError("one-shot symmetric all-reduce supports up to 8 ranks")
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.max_rows, self.hidden = max_rows, hidden
        self.slot_elems = max_rows * hidden
        self.max_blocks = MAX_BLOCKS
        self.timeout_s = timeout_s
        nbytes = 2 * self.slot_elems * 2 + 2 * self.max_blocks * 4
        self.own = None
        self.opened: list[int] = []
        if bases is None:
            with torch.cuda.device(self.device):
                ptr, handle = ext().symm_alloc(nbytes)
            self.own = ptr
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
            bases = []
            for r in range(world):
                if r == rank:
                    bases.append(ptr)
                else:
                    with torch.cuda.device(self.device):
                        p = ext().symm_open(handles[r])
                    self.opened.append(p)
                    bases.append(p)
        self.bases = list(bases)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=self.device)  # [epoch, finished blocks]

    @staticmethod
    def region_bytes(max_rows: int, hidden: int) -> int:
        return 2 * max_rows * hidden * 2 + 2 * MAX_BLOCKS * 4

    def fits(self, rows: int) -> bool:
        return rows <= self.max_rows

    def allreduce_add_rmsnorm(self, partial, residual, w1p, eps):
        """``residual += sum_ranks(partial)`` (in place) and returns (residual, rmsnorm(residual))."""
        rows = residual.numel() // residual.shape[-1]
        if not self.fits(rows):
            return None
        normed = torch.empty_like(residual)
        ext().symm_ar_add_rmsnorm(self.bases, self.rank, partial, residual, w1p, normed, float(eps), self.slot_elems,
                                  self.max_blocks, self.epoch, self.timeout_s)
        return residual, normed

    def close(self) -> None:
        for p in self.opened:
            ext().symm_close(p)
        self.opened.clear()
        if self.own is not None:
            ext().symm_free(self.own)
            self.own = None
