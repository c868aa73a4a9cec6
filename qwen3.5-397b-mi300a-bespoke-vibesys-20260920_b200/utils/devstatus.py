"""Host-side watch over the kernels' device status word.

Every bounded wait in the CUDA kernels (TMA and MMA pipeline waits, peer flags of the fused
collectives, the expert-parallel receive) records an error code in a per-device status word when
its bound runs out, skips its work and returns, instead of trapping. ``StatusWatch`` reads that
word without stalling the launch stream: every ``every`` steps it queues a device->host copy of
the word into pinned memory behind a CUDA event, and on a later step, once the event has
completed, checks the value. A nonzero code raises ``DeviceStatusError`` (the scheduler aborts the
requests in flight; a worker rank exits, which turns ``/health`` to 503) after clearing the word.

Reference behaviour: ``allreduce_custom.py:956-975`` (``_check_error_flag``: raise once a
collective's spin bound ran out); here one word covers every kernel family.
"""

from __future__ import annotations

ERR_NAMES = {1: "tma_wait", 2: "mma_wait", 3: "accumulator_wait", 4: "epilogue_wait", 5: "peer_wait",
             6: "drain", 7: "bounds", 8: "canary"}
# debug build (QB_BOUNDS): words 1..3 of the status hold the failing check's site, value and capacity
BOUNDS_SITES = {1: "embed token id", 2: "paged KV row", 4: "DeltaNet lane", 11: "GEMM stream-K workspace",
                12: "attention split workspace", 13: "DeltaNet scratch", 14: "MoE dispatch metadata",
                15: "MoE activation planes"}


class DeviceStatusError(RuntimeError):
    def __init__(self, code: int):
        self.code = code
        super().__init__(f"device status {code} ({ERR_NAMES.get(code, 'unknown')}): a kernel's bounded wait ran "
                         f"out and its work was skipped")


class StatusWatch:
    """``step()`` after every model step. ``start`` queues a read and returns (ready, value)
    callables; ``clear`` zeroes the word (both default to the CUDA extension on ``device``)."""

    def __init__(self, device=None, every: int = 64, start=None, clear=None):
        self.every = every
        self.n = 0
        self.pending = None
        self._start = start
        self._clear = clear
        if device is not None and (start is None or clear is None):
            import torch

            self._like = torch.empty(1, device=device)
            self._host = None
            self._start = start or self._start_cuda
            self._clear = clear or self._clear_cuda

    def _start_cuda(self):
        import torch

        from ..ops._ext import ext

        st = ext().status(self._like)  # a copy of the word, on the current stream
        if self._host is None:
            self._host = torch.empty(st.shape, dtype=st.dtype, pin_memory=True)
        self._host.copy_(st, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        host = self._host
        return ev.query, lambda: int(host[0])

    def _clear_cuda(self):
        from ..ops._ext import ext

        ext().clear_status(self._like)

    def step(self) -> None:
        if self.every <= 0:
            return
        self.n += 1
        if self.pending is not None and self.pending[0]():
            code = self.pending[1]()
            self.pending = None
            if code:
                self._clear()
                raise DeviceStatusError(code)
        if self.pending is None and self.n % self.every == 0:
            self.pending = self._start()
