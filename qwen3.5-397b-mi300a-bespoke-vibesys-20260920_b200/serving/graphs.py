"""CUDA-graph decode buckets.

``GraphRunner`` wraps a ``Model`` (on every rank, so that the collectives inside the captured
graphs line up) and replays a captured whole-model decode step for batches of up to each
bucket size (default 1, 2, 4, 8, 16, 24, 32, ...). Inputs live in static device buffers that
are refilled from one pinned host buffer per step; the block tables are already a static device
tensor of the model. Batches smaller than the bucket are padded with rows of a dedicated pad
lane (``model.max_batch``, one lane beyond the scheduler's) whose KV rows land in the reserved
block 0, so a padded row can never touch a live lane's state. Everything else (prefill, mixed,
snapshots, blocks) is delegated to the wrapped model.

Reference behaviour: ``graph_decode.py:250-1725`` (``DEFAULT_BUCKET_SIZES``, ``GraphDecodeRunner``,
``fill``, ``prepare``, ``validate``), with its masked-row idea realised as a pad lane.
"""

from __future__ import annotations


import torch

from ..models.qwen35 import StepInputs
from ..utils import flags

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128)


class _Bucket:
    def __init__(self, model, B: int, pool):
        dev = model.device
        self.B = B
        self.tokens = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.rows = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lanes = torch.zeros(B, dtype=torch.int32, device=dev)
        self.cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self.logit_rows = torch.arange(B, dtype=torch.int64, device=dev)
        self.packed_host = torch.zeros(4 * B, dtype=torch.int32).pin_memory()
        self.packed_dev = torch.zeros(4 * B, dtype=torch.int32, device=dev)
        self.tok_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.graph = None
        self.out = None
        self.pool = pool

    def inputs(self, model) -> StepInputs:
        B = self.B
        return StepInputs(self.tokens, self.pos, self.rows, self.lanes, self.cu, self.pos, self.logit_rows,
                          list(range(B)), list(range(B + 1)), [0] * B, model.max_seq)


class GraphRunner:
    """Runner that replays captured decode graphs; see the module docstring."""

    def __init__(self, model, buckets=None):
        self.model = model
        self.max_batch = model.max_batch - 1  # the model is built with one spare lane: the pad lane
        self.max_seq = model.max_seq
        self.block_size = model.block_size
        self.pad_lane = model.max_batch - 1
        lim = self.max_batch
        self.buckets = sorted(b for b in (buckets or DEFAULT_BUCKETS) if b <= lim) or [lim]
        if self.buckets[-1] < lim:
            self.buckets.append(lim)
        self.pool = torch.cuda.graph_pool_handle()
        self._b = {}
        self.enabled = flags.get("QB_GRAPHS")
        self.replays = 0
        self.launch_per_replay: dict[int, int] = {}

    # ------------------------------------------------------------------ capture
    def _fill(self, bk: _Bucket, lanes, tokens, positions):
        m = self.model
        m._gpu_mark("in")
        B, n = bk.B, len(lanes)
        pos = list(positions) + [0] * (B - n)
        ln = list(lanes) + [self.pad_lane] * (B - n)
        rows = [m._row(l, p) for l, p in zip(lanes, positions)] + [0] * (B - n)
        ph = bk.packed_host
        ph[:B] = torch.tensor(pos, dtype=torch.int32)
        ph[B:2 * B] = torch.tensor(rows, dtype=torch.int32)
        ph[2 * B:3 * B] = torch.tensor(ln, dtype=torch.int32)
        bk.tok_host[:n] = torch.tensor([int(t) for t in tokens], dtype=torch.int64)
        bk.tok_host[n:] = 0
        bk.packed_dev.copy_(ph, non_blocking=True)
        bk.tokens.copy_(bk.tok_host, non_blocking=True)
        bk.pos.copy_(bk.packed_dev[:B])
        bk.rows.copy_(bk.packed_dev[B:2 * B])
        bk.lanes.copy_(bk.packed_dev[2 * B:3 * B])
        m._h2d += ph.numel() * 4 + bk.tok_host.numel() * 8
        m._sync_tables()

    def _run(self, bk: _Bucket):
        m = self.model
        return m.logits(m._forward(bk.inputs(m)))

    def prepare(self) -> None:
        """Capture every bucket (largest first, sharing one memory pool). Must run on every rank
        in the same order, before serving starts."""
        if not self.enabled or self.model.device.type != "cuda":
            return
        m = self.model
        m.begin(self.pad_lane)
        m.attach_blocks(self.pad_lane, [])
        from ..ops import _ext

        for B in sorted(self.buckets, reverse=True):
            bk = _Bucket(m, B, self.pool)
            self._fill(bk, [], [], [])
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._run(bk)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            l0 = _ext.ext().launches()
            with torch.cuda.graph(g, pool=self.pool):
                bk.out = self._run(bk)
            self.launch_per_replay[B] = _ext.ext().launches() - l0
            bk.graph = g
            self._b[B] = bk
        torch.cuda.synchronize()

    def attribution(self, B: int, replays: int = 10, detail: bool = False) -> dict[str, float]:
        """Device time per layer part (ms) of one captured ``B``-row decode step.

        Captures a separate diagnostic graph of the bucket with clock stamps between the layer
        parts (``utils.telemetry.Stamps``), replays it ``replays`` times and reads the stamps of
        the last replay (``detail``: also between the kernels of each part, tagged
        ``dn.*``/``attn.*``/``moe.*``); the serving graphs never contain a stamp. Every rank must call this
        (the capture runs the collectives). Reference behaviour: ``decode_stamps.py`` with its
        separate diagnostic capture."""
        from ..utils.telemetry import Stamps

        m = self.model
        bk = _Bucket(m, B, None)
        self._fill(bk, [], [], [])
        st = Stamps(m.device, detail=detail)
        m.stamps = st
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.inference_mode(), torch.cuda.stream(s):
                self._run(bk)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            st.reset()
            g = torch.cuda.CUDAGraph()
            with torch.inference_mode(), torch.cuda.graph(g):
                self._run(bk)
        finally:
            m.stamps = None
        for _ in range(replays):
            g.replay()
        torch.cuda.synchronize()
        out = st.by_tag_ms()
        del g
        return out

    def release(self) -> None:
        """Drop the graphs (before destroy_process_group: they hold NCCL work)."""
        for bk in self._b.values():
            bk.graph = None
            bk.out = None
        self._b.clear()

    # ------------------------------------------------------------------ runner
    def decode(self, lanes, tokens, positions):
        n = len(lanes)
        B = next((b for b in self.buckets if b >= n), None)
        if not self._b or B is None or B not in self._b or self.model.mtp is not None:
            return self.model.decode(lanes, tokens, positions)
        bk = self._b[B]
        with torch.inference_mode():
            self._fill(bk, lanes, tokens, positions)
            bk.graph.replay()
        self.replays += 1
        from ..ops import _ext

        _ext.ext().add_launches(self.launch_per_replay.get(B, 0))
        return bk.out[:n]

    def __getattr__(self, name):
        return getattr(self.model, name)
