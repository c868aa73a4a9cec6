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

Prefill steps (``prepare_prefill``, ``QB_PREFILL_GRAPHS``): one graph per width W replays a
single-segment prefill of exactly W tokens on any lane at any start position. The lane, the start
and every row's position and KV row are device inputs; the tables the host plans for a forward
(flash-attention tiles, DeltaNet chunks) depend only on the segment lengths, here always (W,), so
no padding is needed and nothing else changes between replays: the chunks of a long prompt cut at
the prefill chunk size, and follow-up turns of a captured length, replay instead of issuing their
~1250 launches. Batches of several segments and other lengths run eagerly. Reference behaviour:
``graph_prefill.py:812`` (``PrefillGraphRunner``, captured rows x width shapes).

Mixed steps (``prepare_mixed``, ``QB_MIXED_GRAPHS``): the same for a decode batch of up to B
lanes (padded with the pad lane) plus one prefill segment of exactly W tokens. Reference
behaviour: ``graph_mixed.py:308`` (``MixedGraphRunner``).
"""

from __future__ import annotations


import torch

from ..models.qwen35 import StepInputs
from ..utils import flags

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128)


def _host(t: torch.Tensor) -> torch.Tensor:
    """Page-locked when a CUDA device is present (async input copies), plain memory otherwise."""
    return t.pin_memory() if torch.cuda.is_available() else t


class CudaGraphs:
    """Capture backend: CUDA graphs in one shared memory pool (the serving backend)."""

    def __init__(self):
        self._pool = None

    def pool(self):
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        return self._pool

    def capture(self, fn, warmups: int = 2, pool=True):
        """Runs ``fn`` ``warmups`` times on a side stream, then captures it; returns (graph, the
        captured call's output)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmups):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool() if pool else None):
            out = fn()
        return g, out

    def sync(self):
        torch.cuda.synchronize()

    def count_launches(self) -> int:
        from ..ops import _ext

        return _ext.ext().launches()

    def add_launches(self, n: int) -> None:
        from ..ops import _ext

        _ext.ext().add_launches(n)


class _HostGraph:
    def __init__(self, fn, out):
        self.fn, self.out = fn, out

    def replay(self):
        res = self.fn()
        if isinstance(self.out, tuple):
            for o, r in zip(self.out, res):
                o.copy_(r)
        else:
            self.out.copy_(res)


class HostGraphs(CudaGraphs):
    """Capture backend without a GPU: "capture" keeps the step function and its output tensor,
    "replay" re-runs the function on the same static input buffers and writes the result into
    that output in place, as a CUDA-graph replay updates its captured output. Everything the
    runner does around a replay (bucket choice, padding with the pad lane, input packing, the
    overlap feedback, validation and the rank vote) then runs on CPU ranks in tests."""

    def pool(self):
        return None

    def capture(self, fn, warmups: int = 2, pool=True):
        for _ in range(warmups):
            fn()
        out = fn()
        return _HostGraph(fn, out), out

    def sync(self):
        pass

    def count_launches(self) -> int:
        return 0

    def add_launches(self, n: int) -> None:
        pass


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
        # two pinned input sets used alternately: with the one-step overlap the host fills step
        # n+1 while step n's input copies may still be queued
        self._hosts = [(_host(torch.zeros(4 * B, dtype=torch.int32)),
                        _host(torch.zeros(B, dtype=torch.int64))) for _ in range(2)]
        self._flip = 0
        self.packed_host, self.tok_host = self._hosts[0]
        self.packed_dev = torch.zeros(4 * B, dtype=torch.int32, device=dev)
        self.graph = None
        self.out = None
        self.pool = pool

    def inputs(self, model) -> StepInputs:
        """The bucket's static device inputs. The host lists are what the last fill put there (the
        CUDA kernels read only the device tensors and take nothing but the segment count from
        these; the host reference ops of a CPU rank read the lanes and starts)."""
        B = self.B
        lanes = getattr(self, "lanes_h", None) or [model.max_batch - 1] * B
        starts = getattr(self, "pos_h", None) or [0] * B
        return StepInputs(self.tokens, self.pos, self.rows, self.lanes, self.cu, self.pos, self.logit_rows,
                          list(lanes), list(range(B + 1)), list(starts), model.max_seq)


class _PrefillBucket:
    """Static buffers of one captured single-segment prefill of exactly ``W`` tokens."""

    def __init__(self, model, W: int):
        dev = model.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.W = W
        self.tokens = torch.zeros(W, dtype=torch.int64, device=dev)
        self.packed_dev = torch.zeros(2 * W + 2, **i32)  # positions | KV rows | lane | start
        self.pos = torch.zeros(W, **i32)
        self.rows = torch.zeros(W, **i32)
        self.lane = torch.zeros(1, **i32)
        self.start = torch.zeros(1, **i32)
        self.cu = torch.tensor([0, W], **i32)
        self.logit_rows = torch.tensor([W - 1], dtype=torch.int64, device=dev)
        # two pinned input sets used alternately (a fill never overwrites one whose copy may be queued)
        self._hosts = [(_host(torch.zeros(2 * W + 2, dtype=torch.int32)), _host(torch.zeros(W, dtype=torch.int64)))
                       for _ in range(2)]
        self._flip = 0
        self.lane_h, self.start_h = model.max_batch - 1, 0
        self.graph = None
        self.out = None

    def inputs(self, model) -> StepInputs:
        """The bucket's device inputs; the host lists are the last fill's lane and start (read only
        by the host reference ops of a CPU rank) and the fixed segment length."""
        return StepInputs(self.tokens, self.pos, self.rows, self.lane, self.cu, self.start, self.logit_rows,
                          [self.lane_h], [0, self.W], [self.start_h], model.max_seq)


class _MixedBucket:
    """Static buffers of one captured mixed step: ``B`` one-token decode rows (padded with the pad
    lane) followed by one prefill segment of exactly ``W`` tokens."""

    def __init__(self, model, B: int, W: int):
        dev = model.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.B, self.W = B, W
        T = B + W
        self.tokens = torch.zeros(T, dtype=torch.int64, device=dev)
        self.packed_dev = torch.zeros(2 * T + 2 * (B + 1), **i32)  # positions | rows | lanes | starts
        self.pos = torch.zeros(T, **i32)
        self.rows = torch.zeros(T, **i32)
        self.lanes = torch.zeros(B + 1, **i32)
        self.starts = torch.zeros(B + 1, **i32)
        self.cu_h = list(range(B + 1)) + [T]
        self.cu = torch.tensor(self.cu_h, **i32)
        self.logit_rows = torch.tensor(list(range(B)) + [T - 1], dtype=torch.int64, device=dev)
        self._hosts = [(_host(torch.zeros(2 * T + 2 * (B + 1), dtype=torch.int32)),
                        _host(torch.zeros(T, dtype=torch.int64))) for _ in range(2)]
        self._flip = 0
        self.lanes_h = [model.max_batch - 1] * (B + 1)
        self.starts_h = [0] * (B + 1)
        self.graph = None
        self.out = None

    def inputs(self, model) -> StepInputs:
        return StepInputs(self.tokens, self.pos, self.rows, self.lanes, self.cu, self.starts, self.logit_rows,
                          list(self.lanes_h), list(self.cu_h), list(self.starts_h), model.max_seq)


class _SpecBucket:
    """Static buffers of one captured speculative round for ``B`` lanes and draft depth ``k``:
    the draft steps' positions and KV rows, the verify forward's ``B x (k+1)`` rows, and the
    round's outputs (drafts, the verify argmax, the DeltaNet inputs it keeps for the commit)."""

    def __init__(self, model, B: int, k: int):
        dev = model.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.B, self.k = B, k
        R = B * (k + 1)
        # lanes | draft pos, rows | verify pos, rows | starts | real-row flags
        self.n_packed = B + 2 * k * B + 2 * R + B + B
        self.packed_host = torch.zeros(self.n_packed, dtype=torch.int32).pin_memory()
        self.packed_dev = torch.zeros(self.n_packed, **i32)
        self.tok_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.tok0 = torch.zeros(B, dtype=torch.int64, device=dev)
        self.lanes = torch.zeros(B, **i32)
        self.pos_d = [torch.zeros(B, **i32) for _ in range(k)]
        self.rows_d = [torch.zeros(B, **i32) for _ in range(k)]
        self.pos_v = torch.zeros(R, **i32)
        self.rows_v = torch.zeros(R, **i32)
        self.start_v = torch.zeros(B, **i32)
        self.real = torch.zeros(B, dtype=torch.int64, device=dev)  # 1 for a lane's row, 0 for padding
        self.cu_d = torch.arange(B + 1, **i32)
        self.cu_v = torch.arange(0, R + 1, k + 1, **i32)
        self.logit_rows_d = torch.arange(B, dtype=torch.int64, device=dev)
        self.logit_rows_v = torch.arange(R, dtype=torch.int64, device=dev)
        self.n_host = torch.zeros(B, dtype=torch.int64).pin_memory()  # accepted drafts per lane
        self.n_dev = torch.zeros(B, dtype=torch.int64, device=dev)
        self.graph = self.commit_graph = self.round_graph = None
        self.drafts = self.am = self.vb = self.vsave = self.h_all = None

    def unpack(self) -> None:
        B, k = self.B, self.k
        R = B * (k + 1)
        pd = self.packed_dev
        self.lanes.copy_(pd[:B])
        o = B
        for i in range(k):
            self.pos_d[i].copy_(pd[o:o + B])
            self.rows_d[i].copy_(pd[o + k * B:o + k * B + B])
            o += B
        o = B + 2 * k * B
        self.pos_v.copy_(pd[o:o + R])
        self.rows_v.copy_(pd[o + R:o + 2 * R])
        self.start_v.copy_(pd[o + 2 * R:o + 2 * R + B])
        self.real.copy_(pd[o + 2 * R + B:o + 2 * R + 2 * B])


class GraphRunner:
    """Runner that replays captured decode graphs; see the module docstring."""

    def __init__(self, model, buckets=None, backend=None):
        self.model = model
        self.backend = backend or (CudaGraphs() if model.device.type == "cuda" else HostGraphs())
        self.max_batch = model.max_batch - 1  # the model is built with one spare lane: the pad lane
        self.max_seq = model.max_seq
        self.block_size = model.block_size
        self.pad_lane = model.max_batch - 1
        lim = self.max_batch
        self.buckets = sorted(b for b in (buckets or DEFAULT_BUCKETS) if b <= lim) or [lim]
        if self.buckets[-1] < lim:
            self.buckets.append(lim)
        self.pool = self.backend.pool()
        self._b = {}
        self._spec: dict[int, _SpecBucket] = {}
        self.enabled = flags.get("QB_GRAPHS")
        self.replays = 0
        # kernels per replay: decode bucket B, prefill width -W, mixed shape (B, W)
        self.launch_per_replay: dict[int | tuple[int, int], int] = {}
        self._pb: dict[int, _PrefillBucket] = {}  # captured prefill widths
        self._mb: dict[tuple[int, int], _MixedBucket] = {}  # captured (decode rows, prefill width)
        self.mixed_replays = 0
        self.mixed_validated = False
        self.prefill_replays = 0
        self.prefill_validated = False

    # ------------------------------------------------------------------ capture
    def _fill(self, bk: _Bucket, lanes, tokens, positions):
        m = self.model
        m._gpu_mark("in")
        bk._flip ^= 1
        bk.packed_host, bk.tok_host = bk._hosts[bk._flip]
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
        bk.lanes_h, bk.pos_h = ln, pos
        bk.packed_dev.copy_(ph, non_blocking=True)
        bk.tokens.copy_(bk.tok_host, non_blocking=True)
        bk.pos.copy_(bk.packed_dev[:B])
        bk.rows.copy_(bk.packed_dev[B:2 * B])
        bk.lanes.copy_(bk.packed_dev[2 * B:3 * B])
        m._h2d += ph.numel() * 4 + bk.tok_host.numel() * 8
        m._sync_tables()

    def _run(self, bk: _Bucket):
        """The captured step: the forward and the vocabulary-parallel greedy head, whose output is
        (greedy ids [B], this rank's logits slice [B, V / world])."""
        m = self.model
        return m.greedy(m._forward(bk.inputs(m)))

    def prepare(self) -> None:
        """Capture every bucket (largest first, sharing one memory pool). Must run on every rank
        in the same order, before serving starts."""
        if not self.enabled or (self.model.device.type != "cuda" and not isinstance(self.backend, HostGraphs)):
            return
        m = self.model
        m.begin(self.pad_lane)
        m.attach_blocks(self.pad_lane, [])
        import time

        for B in sorted(self.buckets, reverse=True):
            t0 = time.perf_counter()
            bk = _Bucket(m, B, self.pool)
            self._fill(bk, [], [], [])
            l0 = self.backend.count_launches()
            g, bk.out = self.backend.capture(lambda bk=bk: self._run(bk))
            self.launch_per_replay[B] = (self.backend.count_launches() - l0) // 3  # warm-ups + capture
            bk.graph = g
            self._b[B] = bk
            if flags.get("QB_GRAPH_LOG"):
                print(f"[graph-capture] decode bucket {B}: {self.launch_per_replay[B]} kernels, "
                      f"{time.perf_counter() - t0:.2f}s", flush=True)
        self.backend.sync()
        self.validate()

    def validate(self, tol: float = 5e-2) -> bool:
        """Boot check of every captured bucket: a replay and an eager run of the same step, from
        the same lane states, must give the same logits (max abs difference within ``tol`` of
        the logits' scale: the two run the same kernels, and the margin only admits
        rounding-order differences of the reductions that finish in arrival order, while a replay
        reading a stale or freed table gives garbage far outside it). The step puts one token on
        each of B distinct lanes (lane i at position 0 of block 1 + i; nothing is being served
        yet), so rows do not share state as the pad rows of a padded batch do. Every rank reports
        its verdict and the ranks agree on the minimum (an all-reduce over the model's group), so
        either every rank serves from its graphs or none does. Returns whether the graphs stay
        on. Reference behaviour: ``graph_decode.py`` (``validate``, ``all_ranks``)."""
        m = self.model
        ok = True
        worst = 0.0
        with torch.inference_mode():
            for B, bk in sorted(self._b.items()):
                lanes = list(range(B))

                def reset():
                    for ln in lanes:
                        m.begin(ln)
                        m.attach_blocks(ln, [1 + ln])

                reset()
                self._fill(bk, lanes, [(7 * ln + 11) % 1000 for ln in lanes], [0] * B)
                bk.graph.replay()
                got = bk.out[1].float().clone()
                reset()
                m._sync_tables()
                exp = self._run(bk)[1].float()
                for ln in lanes:
                    m.begin(ln)
                    m.attach_blocks(ln, [])
                err = (got - exp).abs().max().item()
                scale = exp.abs().max().item() + 1e-6
                worst = max(worst, err / scale)
                if not (err <= tol * scale) or not bool(torch.isfinite(got).all()):
                    ok = False
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=m.device)
        world = getattr(m.comm, "world", 1)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        agreed = bool(int(flag.item()))
        if flags.get("QB_GRAPH_LOG") or not agreed:
            print(f"[graph-capture] validation: this rank {'ok' if ok else 'MISMATCH'} (worst relative "
                  f"{worst:.2e}), all ranks {'ok' if agreed else 'disagree: decode runs eagerly'}", flush=True)
        if not agreed:
            self.release()
        self.validated = agreed
        return agreed

    # ------------------------------------------------------------------ prefill steps
    def _prefill_fill(self, bk: _PrefillBucket, lane: int, ids, start: int, rows=None) -> None:
        m = self.model
        W = bk.W
        m._gpu_mark("in")
        bk._flip ^= 1
        ph, th = bk._hosts[bk._flip]
        if rows is None:
            rows = [m._row(lane, p) for p in range(start, start + W)]
        ph[:W] = torch.arange(start, start + W, dtype=torch.int32)
        ph[W:2 * W] = torch.tensor(rows, dtype=torch.int32)
        ph[2 * W] = lane
        ph[2 * W + 1] = start
        th.copy_(torch.tensor([int(t) for t in ids], dtype=torch.int64))
        bk.lane_h, bk.start_h = lane, start
        bk.packed_dev.copy_(ph, non_blocking=True)
        bk.tokens.copy_(th, non_blocking=True)
        bk.pos.copy_(bk.packed_dev[:W])
        bk.rows.copy_(bk.packed_dev[W:2 * W])
        bk.lane.copy_(bk.packed_dev[2 * W:2 * W + 1])
        bk.start.copy_(bk.packed_dev[2 * W + 1:])
        m._h2d += ph.numel() * 4 + th.numel() * 8
        m._sync_tables()

    def _prefill_run(self, bk: _PrefillBucket):
        """The captured step: the forward over the bucket's one segment and its last row's logits."""
        m = self.model
        return m.logits(m._forward(bk.inputs(m)))

    def prepare_prefill(self, widths) -> None:
        """Capture one single-segment prefill step per width (largest first, in the decode graphs'
        memory pool) on the pad lane, whose KV rows all go to the reserved block, then check each
        against an eager forward (``validate_prefill``). Every rank in the same order; skipped with
        an MTP head (its catch-up follows every forward) or when graphs are off."""
        m = self.model
        widths = sorted({int(w) for w in widths if 0 < int(w) <= m.max_seq}, reverse=True)
        if (not self.enabled or not widths or m.mtp is not None
                or (m.device.type != "cuda" and not isinstance(self.backend, HostGraphs))):
            return
        import time

        m.begin(self.pad_lane)
        m.attach_blocks(self.pad_lane, [])
        for W in widths:
            t0 = time.perf_counter()
            bk = _PrefillBucket(m, W)
            self._prefill_fill(bk, self.pad_lane, [0] * W, 0, rows=[0] * W)
            l0 = self.backend.count_launches()
            with torch.inference_mode():
                bk.graph, bk.out = self.backend.capture(lambda bk=bk: self._prefill_run(bk))
            self.launch_per_replay[-W] = (self.backend.count_launches() - l0) // 3  # warm-ups + capture
            self._pb[W] = bk
            if flags.get("QB_GRAPH_LOG"):
                print(f"[graph-capture] prefill width {W}: {self.launch_per_replay[-W]} kernels, "
                      f"{time.perf_counter() - t0:.2f}s", flush=True)
        self.backend.sync()
        self.validate_prefill()

    def validate_prefill(self, tol: float = 5e-2) -> bool:
        """Boot check of every captured prefill width: W tokens on lane 0 (nothing is served yet)
        through the replay and through an eager forward from the same reset state must give the
        same logits within ``tol`` of their scale; the ranks agree on the minimum (as the decode
        buckets do) and the prefill graphs are dropped on every rank if any disagrees."""
        m = self.model
        ok, worst, lane = True, 0.0, 0
        with torch.inference_mode():
            for W, bk in sorted(self._pb.items()):
                blocks = list(range(1, 1 + -(-W // m.block_size)))
                ids = [(13 * i + 7) % min(m.cfg.vocab, 1000) for i in range(W)]

                def reset():
                    m.begin(lane)
                    m.attach_blocks(lane, blocks)

                reset()
                self._prefill_fill(bk, lane, ids, 0)
                bk.graph.replay()
                got = bk.out.float().clone()
                reset()
                exp = m.forward([(lane, ids, 0)]).float()
                m.begin(lane)
                m.attach_blocks(lane, [])
                err = (got - exp).abs().max().item()
                scale = exp.abs().max().item() + 1e-6
                worst = max(worst, err / scale)
                if not (err <= tol * scale) or not bool(torch.isfinite(got).all()):
                    ok = False
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=m.device)
        if getattr(m.comm, "world", 1) > 1:
            import torch.distributed as dist

            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        agreed = bool(int(flag.item()))
        if flags.get("QB_GRAPH_LOG") or not agreed:
            print(f"[graph-capture] prefill validation: this rank {'ok' if ok else 'MISMATCH'} (worst relative "
                  f"{worst:.2e}), all ranks {'ok' if agreed else 'disagree: prefill runs eagerly'}", flush=True)
        if not agreed:
            for bk in self._pb.values():
                bk.graph = bk.out = None
            self._pb.clear()
        self.prefill_validated = agreed
        return agreed

    def prefill_batch(self, calls):
        """``Model.prefill_batch``; one segment of a captured length is replayed from its graph (the
        logits row is copied out: the session cache may keep it past the next replay)."""
        calls = list(calls)
        m = self.model
        if len(calls) == 1 and self._pb and not m.fault and m.mtp is None:
            lane, ids, start = calls[0]
            bk = self._pb.get(len(ids))
            if bk is not None and start + len(ids) <= m.max_seq:
                with torch.inference_mode():
                    self._prefill_fill(bk, lane, ids, start)
                    bk.graph.replay()
                    out = bk.out.clone()
                self.prefill_replays += 1
                self.backend.add_launches(self.launch_per_replay.get(-bk.W, 0))
                return [out]
        return m.prefill_batch(calls)

    def prefill(self, lane, ids, start):
        return self.prefill_batch([(lane, ids, start)])[0]

    # ------------------------------------------------------------------ mixed steps
    def _mixed_fill(self, bk: _MixedBucket, lanes, tokens, positions, call, capture: bool = False) -> None:
        m = self.model
        B, W, T = bk.B, bk.W, bk.B + bk.W
        m._gpu_mark("in")
        bk._flip ^= 1
        ph, th = bk._hosts[bk._flip]
        n = len(lanes)
        plane, pids, pstart = call
        ln = list(lanes) + [self.pad_lane] * (B - n)
        pos = list(positions) + [0] * (B - n)
        if capture:
            rows = [0] * T
        else:
            rows = [m._row(l, p) for l, p in zip(lanes, positions)] + [0] * (B - n)
            rows += [m._row(plane, p) for p in range(pstart, pstart + W)]
        allpos = pos + list(range(pstart, pstart + W))
        ph[:T] = torch.tensor(allpos, dtype=torch.int32)
        ph[T:2 * T] = torch.tensor(rows, dtype=torch.int32)
        ph[2 * T:2 * T + B + 1] = torch.tensor(ln + [plane], dtype=torch.int32)
        ph[2 * T + B + 1:] = torch.tensor(pos + [pstart], dtype=torch.int32)
        th[:n] = torch.tensor([int(t) for t in tokens], dtype=torch.int64)
        th[n:B] = 0
        th[B:] = torch.tensor([int(t) for t in pids], dtype=torch.int64)
        bk.lanes_h, bk.starts_h = ln + [plane], pos + [pstart]
        bk.packed_dev.copy_(ph, non_blocking=True)
        bk.tokens.copy_(th, non_blocking=True)
        bk.pos.copy_(bk.packed_dev[:T])
        bk.rows.copy_(bk.packed_dev[T:2 * T])
        bk.lanes.copy_(bk.packed_dev[2 * T:2 * T + B + 1])
        bk.starts.copy_(bk.packed_dev[2 * T + B + 1:])
        m._h2d += ph.numel() * 4 + th.numel() * 8
        m._sync_tables()

    def _mixed_run(self, bk: _MixedBucket):
        m = self.model
        return m.logits(m._forward(bk.inputs(m)))

    def prepare_mixed(self, shapes) -> None:
        """Capture one mixed step per (decode rows B, prefill width W) on the pad lane, then check
        each against an eager mixed step (``validate_mixed``). The decode rows are padded up to B
        with the pad lane, as the decode buckets do; the prefill segment must be exactly W tokens
        (the segment lengths fix every host-planned table). Every rank in the same order."""
        m = self.model
        shapes = sorted({(int(b), int(w)) for b, w in shapes if 0 < int(b) <= self.max_batch - 1
                         and 0 < int(w) <= m.max_seq}, reverse=True)
        if (not self.enabled or not shapes or m.mtp is not None
                or (m.device.type != "cuda" and not isinstance(self.backend, HostGraphs))):
            return
        m.begin(self.pad_lane)
        m.attach_blocks(self.pad_lane, [])
        for B, W in shapes:
            bk = _MixedBucket(m, B, W)
            self._mixed_fill(bk, [], [], [], (self.pad_lane, [0] * W, 0), capture=True)
            l0 = self.backend.count_launches()
            with torch.inference_mode():
                bk.graph, bk.out = self.backend.capture(lambda bk=bk: self._mixed_run(bk))
            self.launch_per_replay[(B, W)] = (self.backend.count_launches() - l0) // 3
            self._mb[(B, W)] = bk
        self.backend.sync()
        self.validate_mixed()

    def validate_mixed(self, tol: float = 5e-2) -> bool:
        """Boot check of every captured mixed shape: B decode lanes (one token each at position 0)
        and a W-token prefill on another lane, replayed and run eagerly from the same reset states,
        must give the same logits within ``tol`` of their scale; ranks agree on the minimum."""
        m = self.model
        ok, worst = True, 0.0
        with torch.inference_mode():
            for (B, W), bk in sorted(self._mb.items()):
                lanes, plane = list(range(B)), B
                pblocks = list(range(1 + B, 1 + B + -(-W // m.block_size)))
                ids = [(17 * i + 5) % min(m.cfg.vocab, 1000) for i in range(W)]
                toks = [(7 * ln + 11) % 1000 for ln in lanes]

                def reset():
                    for ln in lanes:
                        m.begin(ln)
                        m.attach_blocks(ln, [1 + ln])
                    m.begin(plane)
                    m.attach_blocks(plane, pblocks)

                reset()
                self._mixed_fill(bk, lanes, toks, [0] * B, (plane, ids, 0))
                bk.graph.replay()
                got = bk.out.float().clone()
                reset()
                dec, pre = m.decode_mixed(lanes, toks, [0] * B, [(plane, ids, 0)])
                exp = torch.cat([dec, pre[0]]).float()
                for ln in lanes + [plane]:
                    m.begin(ln)
                    m.attach_blocks(ln, [])
                err = (got - exp).abs().max().item()
                scale = exp.abs().max().item() + 1e-6
                worst = max(worst, err / scale)
                if not (err <= tol * scale) or not bool(torch.isfinite(got).all()):
                    ok = False
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=m.device)
        if getattr(m.comm, "world", 1) > 1:
            import torch.distributed as dist

            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        agreed = bool(int(flag.item()))
        if flags.get("QB_GRAPH_LOG") or not agreed:
            print(f"[graph-capture] mixed validation: this rank {'ok' if ok else 'MISMATCH'} (worst relative "
                  f"{worst:.2e}), all ranks {'ok' if agreed else 'disagree: mixed steps run eagerly'}", flush=True)
        if not agreed:
            for bk in self._mb.values():
                bk.graph = bk.out = None
            self._mb.clear()
        self.mixed_validated = agreed
        return agreed

    def decode_mixed(self, lanes, tokens, positions, prefill_calls):
        """``Model.decode_mixed``; one prefill segment of a captured width with at most a captured
        number of decode rows is replayed from the smallest such shape (rows copied out)."""
        m = self.model
        calls = list(prefill_calls)
        n = len(lanes)
        if len(calls) == 1 and self._mb and not m.fault and m.mtp is None:
            plane, pids, pstart = calls[0]
            W = len(pids)
            B = min((b for b, w in self._mb if w == W and b >= n), default=None)
            if B is not None and pstart + W <= m.max_seq:
                bk = self._mb[(B, W)]
                with torch.inference_mode():
                    self._mixed_fill(bk, lanes, tokens, positions, (plane, pids, pstart))
                    bk.graph.replay()
                    lg = bk.out.clone()
                self.mixed_replays += 1
                self.backend.add_launches(self.launch_per_replay.get((B, W), 0))
                return lg[:n], [lg[B:B + 1]]
        return m.decode_mixed(lanes, tokens, positions, calls)

    # ------------------------------------------------------------------ speculative rounds
    def _spec_fill(self, bk: _SpecBucket, lanes, tokens, positions) -> None:
        m = self.model
        m._gpu_mark("in")
        B, k, n = bk.B, bk.k, len(lanes)
        ln = list(lanes) + [self.pad_lane] * (B - n)
        pos = list(positions) + [0] * (B - n)
        real = [True] * n + [False] * (B - n)
        vals = list(ln)
        for i in range(k):  # draft step i writes the MTP KV row of position p + i
            vals.extend(p + i for p in pos)
        for i in range(k):
            vals.extend(m._row(l, p + i) if r else 0 for l, p, r in zip(ln, pos, real))
        vals.extend(p + j for p in pos for j in range(k + 1))
        vals.extend(m._row(l, p + j) if r else 0 for l, p, r in zip(ln, pos, real) for j in range(k + 1))
        vals.extend(pos)
        vals.extend(1 if r else 0 for r in real)
        bk.packed_host.copy_(torch.tensor(vals, dtype=torch.int32))
        bk.tok_host[:n] = torch.tensor([int(t) for t in tokens], dtype=torch.int64)
        bk.tok_host[n:] = 0
        bk.packed_dev.copy_(bk.packed_host, non_blocking=True)
        bk.tok0.copy_(bk.tok_host, non_blocking=True)
        bk.unpack()
        m._h2d += bk.n_packed * 4 + B * 8
        m._sync_tables()

    def _spec_run(self, bk: _SpecBucket) -> None:
        """Draft ``k`` tokens per lane with the MTP layer, then the wide verify forward and its
        argmax, all on the bucket's static buffers (the body of the captured graph)."""
        m, mtp = self.model, self.model.mtp
        B, k = bk.B, bk.k
        hidden = mtp.seed_h.index_select(0, bk.lanes.long())
        tok = bk.tok0
        outs = []
        for i in range(k):
            b = StepInputs(tok, bk.pos_d[i], bk.rows_d[i], bk.lanes, bk.cu_d, bk.pos_d[i], bk.logit_rows_d,
                           list(range(B)), list(range(B + 1)), [0] * B, m.max_seq)
            h = mtp.layer(mtp.combine(tok, hidden), b)
            tok = m.greedy(h)[0]
            outs.append(tok)
            hidden = h
        bk.drafts = torch.stack(outs, dim=1)
        vb = StepInputs(torch.cat([bk.tok0[:, None], bk.drafts], dim=1).reshape(-1), bk.pos_v, bk.rows_v, bk.lanes,
                        bk.cu_v, bk.start_v, bk.logit_rows_v, list(range(B)), list(range(0, B * (k + 1) + 1, k + 1)),
                        [0] * B, m.max_seq)
        vb.verify = True
        m._vsave = {}
        h = m._forward(vb)
        bk.am = m.greedy(h)[0].view(B, k + 1)
        bk.vb, bk.vsave, bk.h_all = vb, m._vsave, m.last_h_all
        m._vsave = {}

    def _spec_accept(self, bk: _SpecBucket) -> None:
        """Accepted drafts per lane on the device: the leading drafts that equal the verify argmax
        (``MTPHead.accept``), or with forced acceptance each further draft with probability p
        from the device generator; padding rows accept none."""
        mtp, k = self.model.mtp, bk.k
        if mtp.forced_accept is None:
            hit = bk.drafts.eq(bk.am[:, :k])
        else:
            hit = torch.rand(bk.B, k, device=bk.drafts.device) < mtp.forced_accept
        bk.n_dev.copy_(hit.to(torch.int64).cumprod(dim=1).sum(dim=1) * bk.real)

    def _spec_commit(self, bk: _SpecBucket) -> None:
        m = self.model
        m._vsave = bk.vsave
        m.last_h_all = bk.h_all
        m._commit_verify_device(bk.vb, bk.n_dev, bk.k)

    def prepare_speculative(self, buckets=None) -> None:
        """Capture per bucket the whole round as one graph (draft + wide verify + argmax, the
        accepted lengths on the device, the commit: DeltaNet state over the accepted rows, MTP
        catch-up), read back once after it; with ``QB_MTP_DEVICE_ACCEPT=0`` two graphs instead,
        between which the host reads the argmax and decides the accepted lengths. Every rank
        must call this in the same order."""
        m = self.model
        if not self.enabled or m.device.type != "cuda" or m.mtp is None:
            return
        m.begin(self.pad_lane)
        m.attach_blocks(self.pad_lane, [])
        k = m.mtp.k
        lim = self.max_batch
        for B in sorted((b for b in (buckets or self.buckets) if b <= lim), reverse=True):
            bk = _SpecBucket(m, B, k)
            self._spec_fill(bk, [], [], [])
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            # warm-up and capture run on the pad lane only: the commit advances its state, which
            # nothing reads
            with torch.inference_mode(), torch.cuda.stream(st):
                for _ in range(2):
                    self._spec_run(bk)
                    self._spec_commit(bk)
            torch.cuda.current_stream().wait_stream(st)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.inference_mode(), torch.cuda.graph(g, pool=self.pool):
                self._spec_run(bk)
            gc = torch.cuda.CUDAGraph()
            with torch.inference_mode(), torch.cuda.graph(gc, pool=self.pool):
                self._spec_commit(bk)
            bk.graph, bk.commit_graph = g, gc
            if flags.get("QB_MTP_DEVICE_ACCEPT"):
                gr = torch.cuda.CUDAGraph()
                with torch.inference_mode(), torch.cuda.graph(gr, pool=self.pool):
                    self._spec_run(bk)
                    self._spec_accept(bk)
                    self._spec_commit(bk)
                bk.round_graph = gr
            self._spec[B] = bk
        torch.cuda.synchronize()

    def speculative_decode(self, lanes, tokens, positions, budgets, stops):
        """One MTP round per lane replayed from the smallest captured bucket that holds the batch
        (eager when none does); same results as ``Model.speculative_decode``."""
        m = self.model
        n = len(lanes)
        B = next((b for b in sorted(self._spec) if b >= n), None)
        if B is None or m.fault:  # a calibration fault acts on the eager path only
            return m.speculative_decode(lanes, tokens, positions, budgets, stops)
        bk, mtp, k = self._spec[B], m.mtp, m.mtp.k
        if bk.round_graph is not None:
            with torch.inference_mode():
                self._spec_fill(bk, lanes, tokens, positions)
                bk.round_graph.replay()
                m._gpu_mark("out")
                res = torch.cat([bk.n_dev[:, None], bk.drafts, bk.am], dim=1)[:n].tolist()  # one host sync
            m._d2h += 8 * n * (2 * k + 2)
            ns = [int(r[0]) for r in res]
            dr_h = [r[1:1 + k] for r in res]
            am_h = [r[1 + k:] for r in res]
            mtp.rounds += n
            mtp.accepted += sum(ns)
            mtp.drafted += n * k
            self.replays += 1
            return self._spec_tokens(n, ns, dr_h, am_h, budgets, stops)
        with torch.inference_mode():
            self._spec_fill(bk, lanes, tokens, positions)
            bk.graph.replay()
            m._gpu_mark("out")
            am_h, dr_h = bk.am[:n].tolist(), bk.drafts[:n].tolist()  # the round's one host sync
            m._d2h += 8 * n * (2 * k + 1)
            ns = [mtp.accept(dr_h[i], am_h[i]) for i in range(n)]
            mtp.rounds += n
            mtp.accepted += sum(ns)
            mtp.drafted += n * k
            bk.n_host[:n] = torch.tensor(ns, dtype=torch.int64)
            bk.n_host[n:] = 0
            bk.n_dev.copy_(bk.n_host, non_blocking=True)
            m._h2d += 8 * B
            bk.commit_graph.replay()
        self.replays += 1
        return self._spec_tokens(n, ns, dr_h, am_h, budgets, stops)

    @staticmethod
    def _spec_tokens(n, ns, dr_h, am_h, budgets, stops):
        """Each lane's committed tokens: its accepted drafts and the verify argmax after them, cut
        at a stop id and at its budget."""
        out = []
        for i in range(n):
            toks = dr_h[i][:ns[i]] + [am_h[i][ns[i]]]
            st = set(stops[i])
            cut = next((j for j, t in enumerate(toks) if t in st), None)
            if cut is not None:
                toks = toks[:cut + 1]
            out.append(toks[:max(1, budgets[i])])
        return out

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
        for sb in self._spec.values():
            sb.graph = sb.commit_graph = None
        self._spec.clear()
        for pb in self._pb.values():
            pb.graph = pb.out = None
        self._pb.clear()
        for mb in self._mb.values():
            mb.graph = mb.out = None
        self._mb.clear()

    # ------------------------------------------------------------------ runner
    def decode(self, lanes, tokens, positions):
        n = len(lanes)
        B = next((b for b in self.buckets if b >= n), None)
        if not self._b or B is None or B not in self._b or self.model.mtp is not None or self.model.fault:
            return self.model.decode(lanes, tokens, positions)
        bk = self._b[B]
        with torch.inference_mode():
            self._fill(bk, lanes, tokens, positions)
            bk.graph.replay()
        self.replays += 1
        self.backend.add_launches(self.launch_per_replay.get(B, 0))
        return self.model.full_rows(bk.out[1][:n])  # gathered after the replay, on every rank

    def decode_launch(self, lanes, tokens, positions, src_rows, keep_rows=()):
        """``Model.decode_launch`` replayed from the smallest captured bucket that holds the
        batch: the host tokens go in with the bucket's inputs, the fed-back rows are then
        overwritten on the device from the previous launch's ids, and the argmax and its
        read-back run after the replay."""
        n = len(lanes)
        B = next((b for b in self.buckets if b >= n), None)
        m = self.model
        if not self._b or B is None or B not in self._b or m.mtp is not None or m.fault:
            return m.decode_launch(lanes, tokens, positions, src_rows, keep_rows)
        bk = self._b[B]
        with torch.inference_mode():
            self._fill(bk, lanes, [int(t) if t >= 0 else 0 for t in tokens], positions)
            m._feed_back(bk.tokens, tokens, src_rows)
            bk.graph.replay()
            self.replays += 1
            self.backend.add_launches(self.launch_per_replay.get(B, 0))
            return m._launch_tail(bk.out[0][:n], bk.out[1][:n], n, keep_rows)

    def __getattr__(self, name):
        return getattr(self.model, name)
