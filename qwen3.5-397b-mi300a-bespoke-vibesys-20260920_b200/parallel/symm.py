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

MAX_BLOCKS = 296  # one-shot kernel: two CTAs per SM on a 148-SM B200
SP_MAX_BLOCKS = 296  # sequence-parallel kernel: one row per CTA; more CTAs measured slower


class SymmUnavailable(RuntimeError):
    """Raised on every rank together when any rank could not set up its symmetric region."""


def vote_or_raise(ok: bool, err: Exception | None, device, what: str, group=None) -> None:
    """Every rank reports whether its local step worked (``dist.all_reduce`` MIN of a 0/1 flag);
    when any rank failed, every rank raises ``SymmUnavailable`` at this same point, so they all
    fall back to NCCL together instead of some waiting in a collective the others never reach.
    Reference behaviour: ``allreduce_custom.py:932-953`` (``_vote_or_raise``)."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) == 0:
        raise SymmUnavailable(f"{what} failed on at least one rank (this rank: {err!r})")


def alloc_region(rank: int, world: int, device, nbytes: int, group=None, alloc=None, open_=None, close=None,
                 free=None, vote_device=None) -> tuple[list[int], int, list[int]]:
    """Allocate this rank's region (``cudaMalloc``, zeroed), export it and map every peer's.
    Returns (every rank's base address as seen here, own pointer, opened peer pointers); every
    rank must call this together (it all-gathers the IPC handles). A failure on any rank, in the
    allocation or in mapping a peer, raises ``SymmUnavailable`` on every rank after a vote, with
    this rank's own mappings undone. ``alloc``/``open_``/``close``/``free`` default to the CUDA
    extension (tests pass host fakes)."""
    alloc = alloc or (lambda n: ext().symm_alloc(n))
    open_ = open_ or (lambda h: ext().symm_open(h))
    close = close or (lambda p: ext().symm_close(p))
    free = free or (lambda p: ext().symm_free(p))
    vdev = vote_device if vote_device is not None else device
    ptr = handle = err = None
    try:
        with torch.cuda.device(device) if torch.device(device).type == "cuda" else _nullctx():
            ptr, handle = alloc(nbytes)
    except Exception as e:  # noqa: BLE001 - reported through the vote
        err = e
    vote_or_raise(err is None, err, vdev, "symmetric region allocation", group)
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    bases, opened = [], []
    try:
        for r in range(world):
            if r == rank:
                bases.append(ptr)
            else:
                with torch.cuda.device(device) if torch.device(device).type == "cuda" else _nullctx():
                    p = open_(handles[r])
                opened.append(p)
                bases.append(p)
    except Exception as e:  # noqa: BLE001 - reported through the vote
        err = e
    try:
        vote_or_raise(err is None, err, vdev, "peer region mapping", group)
    except SymmUnavailable:
        for p in opened:
            close(p)
        free(ptr)
        raise
    return bases, ptr, opened


class _nullctx:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


class NvlsRegion:
    """A symmetric region bound to an NVSwitch multicast object (NVLS), for the switch-reduced
    all-reduce + residual add + RMSNorm of large messages (``csrc/comm.cu``,
    ``nvls_ar_add_rmsnorm_kernel``). The memory comes from PyTorch's symmetric-memory allocator
    (``torch.distributed._symmetric_memory``: one physical allocation per rank, every peer's
    mapped, plus the multicast address when the fabric supports it); the kernels are this
    package's. Every rank must construct it together; when any rank gets no multicast address
    all of them raise ``SymmUnavailable`` (``vote_or_raise``). Reference counterpart: none (the
    reference's MI300A fabric has no in-switch reduction); its large-message path is the
    row-sharded reduce-scatter + norm + all-gather family.

    The grid is fixed per region (the arrival counters count ``world x grid`` arrivals per
    call), and so is ``rows_cap``."""

    GRID = 148

    def __init__(self, rank: int, world: int, device, rows_cap: int, hidden: int, group=None,
                 timeout_s: float = 10.0):
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.rows_cap, self.hidden, self.timeout_s = rows_cap, hidden, timeout_s
        self.slot_elems = rows_cap * hidden
        self.buf = None
        err = None
        mc = 0
        try:
            import torch.distributed._symmetric_memory as symm_mem

            pg = group or dist.group.WORLD
            name = pg.group_name
            if hasattr(symm_mem, "enable_symm_mem_for_group"):
                try:
                    symm_mem.enable_symm_mem_for_group(name)
                except Exception:  # noqa: BLE001 - newer releases need no enabling
                    pass
            nbytes = int(ext().nvls_region_bytes(self.slot_elems))
            self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            self.hdl = symm_mem.rendezvous(self.buf, name)
            mc = int(getattr(self.hdl, "multicast_ptr", 0) or 0)
            if mc == 0:
                raise RuntimeError("no multicast address (NVLS unsupported on this fabric or driver)")
            self.buf.zero_()
            torch.cuda.synchronize(self.device)
        except Exception as e:  # noqa: BLE001 - reported through the vote
            err = e
        vote_or_raise(err is None, err, self.device, "NVLS multicast region", group)
        dist.barrier(group=group)  # every rank's counters are zero before any rank arrives
        self.uc = self.buf.data_ptr()
        self.mc = mc
        self.epoch = torch.zeros(2, dtype=torch.int32, device=self.device)

    def allreduce_add_rmsnorm(self, partial, residual, w1p, eps):
        rows = residual.numel() // residual.shape[-1]
        if rows > self.rows_cap:
            return None
        normed = torch.empty_like(residual)
        ext().nvls_ar_add_rmsnorm(self.uc, self.mc, self.world, self.rank, partial, residual, w1p, normed,
                                  float(eps), self.slot_elems, self.GRID, self.epoch, self.timeout_s)
        return residual, normed


class SymmComm:
    """One-shot region (``max_rows`` rows) for decode-sized messages and, when ``sp_rows`` > 0, a
    sequence-parallel region for prefill-sized ones (reduce-scatter + add + RMSNorm +
    all-gather, ``csrc/comm.cu``). Each family has its own slots, flags and device epoch."""

    # The one-shot kernel pulls (W - 1) x the message into every GPU in one phase; the sequence-
    # parallel kernel moves ~3 (W - 1) / W x in three. One-shot while (W - 1) x rows stays small.
    ONESHOT_ROW_BUDGET = 1024

    def __init__(self, rank: int, world: int, device, max_rows: int, hidden: int, group=None,
                 timeout_s: float = 10.0, bases: list[int] | None = None, sp_rows: int = 0,
                 sp_bases: list[int] | None = None):
        if world > 8:
            raise ValueError("one-shot symmetric all-reduce supports up to 8 ranks")
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.max_rows, self.hidden = max_rows, hidden
        self.slot_elems = max_rows * hidden
        self.max_blocks = MAX_BLOCKS
        self.timeout_s = timeout_s
        self.own: list[int] = []
        self.opened: list[int] = []
        self.bases = self._region(2 * self.slot_elems * 2 + 2 * self.max_blocks * 4, group, bases)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=self.device)  # [epoch, finished blocks]
        self.sp_rows = sp_rows
        # partial slots hold whole per-rank ranges: world x ceil(rows / world) rows
        self.sp_slot_elems = -(-sp_rows // world) * world * hidden
        self.sp_bases = None
        if sp_rows > 0:
            try:
                self.sp_bases = self._region(self.sp_region_bytes(-(-sp_rows // world) * world, hidden), group,
                                             sp_bases)
            except SymmUnavailable:
                self.close()  # the one-shot region is undone on every rank alike
                raise
            self.sp_epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.nvls = None
        self.nvls_min_rows = 1 << 30

    def enable_nvls(self, rows_cap: int, min_rows: int, group=None) -> bool:
        """Add the NVLS region (every rank together); messages of ``min_rows`` rows and more
        then take the switch-reduced kernel. False, on every rank, when the fabric has no
        multicast support."""
        try:
            self.nvls = NvlsRegion(self.rank, self.world, self.device, rows_cap, self.hidden, group,
                                   self.timeout_s)
        except SymmUnavailable:
            self.nvls = None
            return False
        self.nvls_min_rows = min_rows
        return True

    @staticmethod
    def sp_region_bytes(sp_rows: int, hidden: int) -> int:
        # two slots of [partial | result residual + normed] = 3 x rows x hidden bf16, then A and B flags
        # and the owner-only call's ready word
        return 2 * 3 * sp_rows * hidden * 2 + 4 * SP_MAX_BLOCKS * 4 + 64

    def _region(self, nbytes: int, group, bases):
        """Allocate and export this rank's region, map every peer's (or use given bases)."""
        if bases is not None:
            return list(bases)
        out, ptr, opened = alloc_region(self.rank, self.world, self.device, nbytes, group)
        self.own.append(ptr)
        self.opened.extend(opened)
        return out

    @staticmethod
    def region_bytes(max_rows: int, hidden: int) -> int:
        return 2 * max_rows * hidden * 2 + 2 * MAX_BLOCKS * 4

    def fits(self, rows: int) -> bool:
        return rows <= self.max_rows or rows <= self.sp_rows

    def allreduce_add_rmsnorm(self, partial, residual, w1p, eps, kind: str = "auto", gather_out: bool = False,
                              res_local: bool = False):
        """``residual += sum_ranks(partial)`` (in place) and returns (residual, rmsnorm(residual)).
        One-shot kernel while ``rows * (world - 1)`` is within ``ONESHOT_ROW_BUDGET`` (one peer
        round trip), the sequence-parallel kernel above that (``kind`` = "oneshot" / "sp" forces
        one); None when the message fits neither region."""
        rows = residual.numel() // residual.shape[-1]
        normed = torch.empty_like(residual)
        nvls = getattr(self, "nvls", None)
        if kind == "nvls" or (kind == "auto" and nvls is not None and rows >= self.nvls_min_rows):
            if nvls is not None:
                out = nvls.allreduce_add_rmsnorm(partial, residual, w1p, eps)
                if out is not None:
                    return out
            if kind == "nvls":
                return None
        fits_sp = self.sp_bases is not None and rows <= self.sp_rows
        if kind == "sp":
            use_sp = fits_sp
        elif kind == "oneshot":
            use_sp = False
        else:
            use_sp = fits_sp and (rows > self.max_rows or rows * (self.world - 1) > self.ONESHOT_ROW_BUDGET)
        if use_sp:
            ext().symm_sp_ar_add_rmsnorm(self.sp_bases, self.rank, partial, residual, w1p, normed, float(eps),
                                         self.sp_slot_elems, SP_MAX_BLOCKS, self.sp_epoch, self.timeout_s,
                                         gather_out, res_local)
            if gather_out:  # this rank's rows only: the next projection gathers (GatheredRows.linear)
                return residual, GatheredRows(self, rows, residual.shape[-1], residual.device, normed)
            return residual, normed
        if rows > self.max_rows:
            return None
        ext().symm_ar_add_rmsnorm(self.bases, self.rank, partial, residual, w1p, normed, float(eps), self.slot_elems,
                                  self.max_blocks, self.epoch, self.timeout_s)
        return residual, normed

    def gathers(self, rows: int) -> bool:
        """Whether ``allreduce_add_rmsnorm(..., gather_out=True)`` leaves the all-gather of ``rows``
        rows to the next projection (the sizes that take the sequence-parallel kernel)."""
        return self.fuses_linear(rows)

    def fuses_linear(self, rows: int) -> bool:
        """Whether ``linear_allreduce_add_rmsnorm`` takes the fused GEMM -> reduce-scatter path
        for ``rows`` (the sizes the automatic choice gives the sequence-parallel kernel)."""
        if self.sp_bases is None or rows < 1:
            return False
        if self.nvls is not None and rows >= self.nvls_min_rows and rows <= self.nvls.rows_cap:
            return False
        return rows <= self.sp_rows and (rows > self.max_rows or rows * (self.world - 1) > self.ONESHOT_ROW_BUDGET)

    def linear_allreduce_add_rmsnorm(self, x, w, residual, w1p, eps, res_local: bool = False):
        """``residual += sum_ranks(x @ w^T)`` (in place) and returns (residual, rmsnorm(residual)):
        the projection's epilogue stores every row into the symmetric region of the rank that owns
        it, then the sequence-parallel kernel reduces, normalises and gathers. None when
        ``fuses_linear`` is false (the caller runs the projection and the all-reduce apart)."""
        rows = residual.numel() // residual.shape[-1]
        if not self.fuses_linear(rows):
            return None
        normed = torch.empty_like(residual)
        ext().symm_linear_sp_ar_add_rmsnorm(x, w, self.sp_bases, self.rank, residual, w1p, normed, float(eps),
                                            self.sp_slot_elems, SP_MAX_BLOCKS, self.sp_epoch, self.timeout_s,
                                            res_local)
        return residual, normed

    def close(self) -> None:
        for p in self.opened:
            ext().symm_close(p)
        self.opened.clear()
        for p in self.own:
            ext().symm_free(p)
        self.own.clear()


class GatheredRows:
    """The normed rows of an owner-only sequence-parallel all-reduce: this rank holds its own
    range (``local``, other rows unset); every rank's range sits in that rank's symmetric result
    area. ``linear(w)`` is the all-gather -> GEMM: ``gathered @ w^T`` with each owner's token
    tiles loaded by TMA from its area once its ready word shows this call (csrc/gemm.cu
    ``gemm_ag``). It stands in for the normed tensor where its only consumer is the next layer's
    input projection."""

    gathered = True
    is_cuda = True
    dtype = torch.bfloat16

    def __init__(self, symm: "SymmComm", rows: int, hidden: int, device, local: torch.Tensor):
        self.symm, self.rows, self.hidden, self.device, self.local = symm, rows, hidden, device, local
        self.shape = (rows, hidden)

    def linear(self, w: torch.Tensor) -> torch.Tensor:
        s = self.symm
        return ext().symm_gemm_ag(s.sp_bases, s.rank, w, self.rows, self.hidden, s.sp_slot_elems, SP_MAX_BLOCKS,
                                  s.sp_epoch, s.timeout_s)
