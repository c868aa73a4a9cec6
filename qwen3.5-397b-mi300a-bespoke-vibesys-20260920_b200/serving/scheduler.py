"""Continuous-batching scheduler with the cross-turn prefix/session cache (host only).

Iteration model: one ``step()`` is either one packed prefill call (several requests' prompt
chunks concatenated, up to ``token_budget`` tokens; packed shortest pending prompt first by
default, ``QB_PREFILL_ORDER``) or one batched decode step over every lane past prefill; prefill wins ties for at most ``max_prefill_burst`` consecutive steps while
lanes are decoding (reference ``scheduler.py:865-948``). With ``mixed=True`` a decode step
also carries prefill chunks in the same forward (Sarathi-style), and with an MTP-capable runner
decode steps are speculative rounds (draft, verify, accept).

Admission (``_admit``): any free lane; the session cache resolves the deepest reusable
boundary for the prompt, copy-on-write of its partial last block, adoption of its blocks and
load of its DeltaNet snapshot; only the remaining prompt tail is prefilled. An exact repeat of
a cached boundary is answered from the node's cached logits with no forward.

Publishing: a turn-open node at ``len(prompt) - suffix_len`` (the chat template's generation
suffix is excluded, so a follow-up turn whose history re-renders this turn without it still
matches), and a turn-close node when a request finishes, at the last forwarded position (the
final sampled token is never forwarded, so its logits are exactly the node's cached logits).

The scheduler is the only block allocator while serving: every forward's KV rows are reserved
here first (``_grow``), so under tensor parallelism every rank holds the same block ids.

Reference behaviour: ``scheduler.py:612-2186`` (``Scheduler``, ``_admit``, ``_acquire``,
``_grow_lanes``, ``_publish_boundary``, ``_publish_turn_close``, ``_select_prefill_batch``,
``_finish_prefill_chunk``, ``_decode_step``, ``_speculative_decode_step``, ``_mixed_step``,
``_emit``, ``_release``).
"""

from __future__ import annotations

import queue
import threading
import time
import traceback
from collections import deque
from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from typing import Any

from ..utils.telemetry import StepTimer
from .block_pool import blocks_for
from .session_cache import Node, SessionCache, SessionCacheError

Event = tuple[str, Any]

PREFILL_CHUNK = 512
PREFILL_TOKEN_BUDGET = 2048
MAX_PREFILL_BURST = 4
MAX_PREFILL_SKIPS = 8  # shortest-first: a flight passed over this many prefill steps goes first


@dataclass
class Request:
    """One completion. ``emit`` receives ``("tok", id)`` per generated token, then
    ``("end", (reason, generated, reused))`` or ``("error", message)``."""

    prompt: list[int]
    max_new: int
    emit: Callable[[Event], None]
    temperature: float = 0.0
    stop: frozenset[int] = frozenset()
    suffix_len: int = 0
    has_history: bool = False
    arrival: float = field(default_factory=time.perf_counter)
    first_token_at: float | None = None


@dataclass
class _Flight:
    req: Request
    lane: int
    pos: int
    pending: list[int]
    reused: int
    parent: Node
    resumed_from: Node
    blocks: list[int]
    boundary: int
    next_token: int | None = None
    skipped: int = 0  # prefill steps that ran without this flight (shortest-first aging)
    generated: int = 0
    out_ids: list[int] = field(default_factory=list)
    last_logits: Any = None
    done: bool = False
    forced: list[int] = field(default_factory=list)  # folded suffix ids still to feed after next_token
    queued_at: float = field(default_factory=time.perf_counter)  # entered the prefill queue


@dataclass
class _Inflight:
    """A decode step launched but not yet read back (one-step overlap)."""

    handle: Any
    flights: list  # the step's flights, in row order
    finishing: set  # ids of flights whose last token this step produces


@dataclass
class ScoreJob:
    ids: list[int]
    continuation_start: int
    finish: Callable[[Any], Any]
    done: threading.Event = field(default_factory=threading.Event)
    result: Any = None
    error: str | None = None


@dataclass
class _Control:
    fn: Callable[[], Any]
    done: threading.Event = field(default_factory=threading.Event)
    result: Any = None


class Scheduler:
    def __init__(self, runner, cache: SessionCache, prefill_chunk: int = PREFILL_CHUNK,
                 token_budget: int = PREFILL_TOKEN_BUDGET, max_prefill_burst: int = MAX_PREFILL_BURST,
                 mixed: bool = False, speculative: bool = False, timer: StepTimer | None = None,
                 prefill_order: str | None = None, max_skips: int = MAX_PREFILL_SKIPS,
                 overlap: bool | None = None, prefill_pack: str | None = None, fold_suffix: bool | None = None,
                 prefill_accum: bool | None = None) -> None:
        self.runner = runner
        self.cache = cache
        self.block_size = cache.block_size
        self.prefill_chunk = prefill_chunk
        self.token_budget = token_budget
        self.max_prefill_burst = max_prefill_burst
        self.mixed = mixed
        self.speculative = speculative
        if prefill_order is None:
            from ..utils import flags

            prefill_order = flags.get("QB_PREFILL_ORDER")
        if prefill_order not in ("fifo", "shortest"):
            raise ValueError(f"prefill_order must be fifo or shortest, got {prefill_order!r}")
        self.prefill_order = prefill_order
        self.max_skips = max_skips
        if prefill_pack is None:
            from ..utils import flags

            prefill_pack = flags.get("QB_PREFILL_PACK")
        if prefill_pack not in ("fill", "finish"):
            raise ValueError(f"prefill_pack must be fill or finish, got {prefill_pack!r}")
        self.prefill_pack = prefill_pack
        from ..utils import flags as _flags

        self.cache_stats_every = int(_flags.get("QB_CACHE_STATS"))
        self.fold_suffix = bool(_flags.get("QB_FOLD_SUFFIX")) if fold_suffix is None else fold_suffix
        self.prefill_accum = bool(_flags.get("QB_PREFILL_ACCUM")) if prefill_accum is None else prefill_accum
        self.accum_tokens = int(_flags.get("QB_PREFILL_ACCUM_TOKENS"))
        self.accum_wait_s = float(_flags.get("QB_PREFILL_ACCUM_WAIT_MS")) / 1e3
        self.accum_min_decode = int(_flags.get("QB_PREFILL_ACCUM_MIN_DECODE"))
        self.held_steps = 0  # steps on which queued prefill was held back (accumulation)
        self.finished = 0
        if overlap is None:
            overlap = bool(_flags.get("QB_OVERLAP"))
        self.overlap = overlap and hasattr(runner, "decode_launch")
        self.inflight: _Inflight | None = None
        self.free_lanes: list[int] = list(range(runner.max_batch - 1, -1, -1))
        self.incoming: queue.Queue = queue.Queue()
        self.waiting: deque[Request] = deque()
        self.prefilling: deque[_Flight] = deque()
        self.decoding: list[_Flight] = []
        self.burst = 0
        self.timer = timer or StepTimer()
        self.steps = 0
        self._stop = threading.Event()
        self.errors = 0

    # ================================================================== public
    def submit(self, req: Request) -> None:
        self.incoming.put(req)

    def reset_prefix_cache(self) -> int:
        """Evict every cache entry not held by a live request (runs on the scheduler thread)."""
        return self.control(lambda: self.cache.evict_all(self._live_parents()))

    def score(self, job: ScoreJob) -> None:
        self.incoming.put(job)

    def control(self, fn: Callable[[], Any], timeout: float | None = 600.0):
        c = _Control(fn)
        self.incoming.put(c)
        if not c.done.wait(timeout):
            raise TimeoutError("scheduler did not run the control message")
        return c.result

    def idle(self) -> bool:
        return (not (self.waiting or self.prefilling or self.decoding) and self.inflight is None
                and self.incoming.empty())

    def stop(self) -> None:
        self._stop.set()
        self.incoming.put(None)

    def run(self) -> None:
        while not self._stop.is_set():
            if self.idle():
                try:
                    item = self.incoming.get(timeout=0.05)
                except queue.Empty:
                    continue
                if item is not None:
                    self._accept(item)
            self.step()

    def run_until_idle(self, max_steps: int = 10**9) -> None:
        n = 0
        while not self.idle() and n < max_steps:
            self.step()
            n += 1

    # ================================================================== iteration
    def _accept(self, item) -> None:
        if isinstance(item, _Control):
            try:
                item.result = item.fn()
            finally:
                item.done.set()
        elif isinstance(item, ScoreJob):
            self._run_score(item)
        elif isinstance(item, Request):
            self.waiting.append(item)

    def _drain(self) -> None:
        while True:
            try:
                item = self.incoming.get_nowait()
            except queue.Empty:
                return
            if item is not None:
                self._accept(item)

    def step(self) -> bool:
        self._drain()
        try:
            while self.waiting and self.free_lanes:
                if not self._admit(self.waiting[0]):
                    break
                self.waiting.popleft()
            if self.prefilling and (not self.decoding or self.burst < self.max_prefill_burst) \
                    and not self._hold_prefill():
                self._complete_inflight()  # a prefill or mixed step starts from a quiet pipeline
                if self.mixed and self.decoding:
                    self._decode_step(with_prefill=True)
                else:
                    self._prefill_step()
                    self.burst += 1
                self.steps += 1
                self._watch_status()
                return True
            if self.decoding or self.inflight is not None:
                self._decode_step()
                self.burst = 0
                self.steps += 1
                self._watch_status()
                return True
            return False
        except Exception as e:  # abort everything in flight, keep serving
            self.errors += 1
            msg = f"{type(e).__name__}: {e}"
            traceback.print_exc()
            self._abort_all(msg)
            return True

    def _hold_prefill(self) -> bool:
        """Prefill accumulation: while many lanes decode, a prefill step costs nearly the same
        for few tokens as for a full budget (it streams every layer's experts either way), so
        queued prefill waits until ``accum_tokens`` tokens can be packed into one step or its
        oldest flight has waited ``accum_wait_s``; decode steps run meanwhile. Reference
        behaviour: ``scheduler.py:107-128`` (``SEED_PREFILL_ACCUM``)."""
        if not (self.prefill_accum and len(self.decoding) >= max(1, self.accum_min_decode)):
            return False
        packable = sum(min(len(f.pending), self.prefill_chunk) for f in self.prefilling)
        oldest = min(f.queued_at for f in self.prefilling)
        if packable >= min(self.accum_tokens, self.token_budget) or \
                time.perf_counter() - oldest >= self.accum_wait_s:
            return False
        self.held_steps += 1
        return True

    def _watch_status(self) -> None:
        """Poll the device status word (raises ``DeviceStatusError``: the step's caller aborts)."""
        watch = getattr(self.runner, "status_watch", None)
        if watch is not None:
            watch.step()

    # ================================================================== admission
    def _live_parents(self) -> list[Node]:
        return [f.parent for f in list(self.prefilling) + self.decoding]

    def _admit(self, req: Request) -> bool:
        if not req.prompt:
            req.emit(("error", "empty prompt"))
            return True
        if len(req.prompt) + max(req.max_new, 0) > self.runner.max_seq:
            req.emit(("error", f"prompt ({len(req.prompt)}) + max_tokens ({req.max_new}) exceeds the "
                               f"context limit {self.runner.max_seq}"))
            return True
        node = self.cache.lookup(req.prompt)
        self.cache.classify(req.prompt, node)  # counted in cache.admissions (diagnostics)
        lane = self.free_lanes[-1]
        protect = [node] + self._live_parents()
        try:
            if self.cache.needs_cow(node):
                new = self.cache.reserve_blocks(1, protect)
                self.runner.copy_block(new[0], node.blocks[-1], node.depth % self.block_size)
                blocks = self.cache.adopt(node, new[0])
            else:
                blocks = self.cache.adopt(node)
        except SessionCacheError:
            if not (self.prefilling or self.decoding):
                req.emit(("error", "KV block pool exhausted: no evictable cache entry left"))
                return True
            return False
        self.free_lanes.pop()
        self.runner.begin(lane)
        self.runner.attach_blocks(lane, blocks)
        if not node.is_root():
            self.runner.load_snapshot(lane, node.snapshot)
        boundary = len(req.prompt) - req.suffix_len
        f = _Flight(req, lane, node.depth, list(req.prompt[node.depth:]), node.depth, node, node, blocks,
                    boundary if boundary > node.depth else -1)
        if not f.pending:  # exact repeat of a cached boundary: answer from its cached logits
            logits = self.runner.cached_node_logits(node.snapshot)
            self._first_token(f, logits)
        else:
            self.prefilling.append(f)
        return True

    def _grow(self, flights: Sequence[_Flight], upto: Sequence[int]) -> None:
        grants = []
        protect = self._live_parents()
        for f, end in zip(flights, upto):
            need = blocks_for(end, self.block_size) - len(f.blocks)
            if need > 0:
                ids = self.cache.reserve_blocks(need, protect)
                f.blocks.extend(ids)
                grants.extend((f.lane, b) for b in ids)
        if grants:
            self.runner.extend_blocks(grants)

    # ================================================================== prefill
    def _prefill_queue(self) -> list[_Flight]:
        """Prefill flights in the order a step packs them. ``fifo``: admission order.
        ``shortest``: fewest pending prompt tokens first, so a follow-up turn's few hundred new
        tokens are not queued behind another session's long opening prompt; a flight passed
        over ``max_skips`` prefill steps in a row goes first (no starvation)."""
        q = list(self.prefilling)
        if self.prefill_order == "shortest":
            q.sort(key=lambda f: (f.skipped < self.max_skips, len(f.pending)))
        return q

    def _select_prefill(self) -> list[tuple[_Flight, list[int]]]:
        batch, budget = [], self.token_budget
        completing = False  # the batch already gives some request its first token
        for f in self._prefill_queue():
            n = min(len(f.pending), self.prefill_chunk, budget)
            if f.boundary > f.pos:
                n = min(n, f.boundary - f.pos)
            if n <= 0:
                break
            done = n == len(f.pending)
            if completing and self.prefill_pack == "finish" and not done:
                continue  # would only lengthen the step that delivers those first tokens
            batch.append((f, f.pending[:n]))
            completing |= done
            budget -= n
            if budget <= 0:
                break
        chosen = {id(f) for f, _ in batch}
        for f in self.prefilling:
            f.skipped = 0 if id(f) in chosen else f.skipped + 1
        return batch

    def _prefill_step(self) -> None:
        batch = self._select_prefill()
        self._grow([f for f, _ in batch], [f.pos + len(ids) for f, ids in batch])
        t0 = time.perf_counter()
        logits = self.runner.prefill_batch([(f.lane, ids, f.pos) for f, ids in batch])
        self._finish_prefill(batch, logits)
        self.timer.record("prefill", sum(len(i) for _, i in batch), time.perf_counter() - t0)

    def _finish_prefill(self, batch, logits) -> None:
        for (f, ids), lg in zip(batch, logits):
            f.pos += len(ids)
            f.pending = f.pending[len(ids):]
            if f.pos == f.boundary:
                self._publish(f, f.req.prompt, f.pos, lg)
                if self.fold_suffix and f.pending and f.req.max_new > 0:
                    # the suffix rides the next decode steps as forced input ids
                    self.prefilling.remove(f)
                    f.next_token, f.forced, f.pending = f.pending[0], list(f.pending[1:]), []
                    f.last_logits = lg
                    self.decoding.append(f)
                    continue
            if not f.pending:
                self.prefilling.remove(f)
                self._first_token(f, lg)

    def _first_token(self, f: _Flight, logits) -> None:
        if f.req.max_new <= 0:
            self._finish(f, "length")
            return
        tok = self.runner.sample_batch(logits, [f.req.temperature])[0]
        f.last_logits = logits
        self._emit(f, tok)
        if not f.done:
            self.decoding.append(f)

    # ================================================================== decode
    def _decode_step(self, with_prefill: bool = False) -> None:
        flights = list(self.decoding)
        if self.overlap and not with_prefill and not self.speculative and \
                all(not f.req.temperature and not f.forced for f in flights):
            return self._overlap_step()
        self._complete_inflight()
        flights = list(self.decoding)
        if not flights and not with_prefill:
            return
        if self.speculative and not with_prefill and self._spec_ok(flights):
            return self._speculative_step(flights)
        pre = self._select_prefill() if with_prefill else []
        self._grow(flights + [f for f, _ in pre], [f.pos + 1 for f in flights] + [f.pos + len(i) for f, i in pre])
        lanes = [f.lane for f in flights]
        toks = [f.next_token for f in flights]
        poss = [f.pos for f in flights]
        t0 = time.perf_counter()
        if pre:
            logits, plog = self.runner.decode_mixed(lanes, toks, poss, [(f.lane, i, f.pos) for f, i in pre])
        else:
            logits, plog = self.runner.decode(lanes, toks, poss), []
        sampled = self.runner.sample_batch(logits, [f.req.temperature for f in flights])
        for i, (f, t) in enumerate(zip(flights, sampled)):
            f.pos += 1
            f.last_logits = self.runner.decode_row(logits, i)
            if f.forced:  # a folded suffix id is still to be fed: the sample is not output
                f.next_token = f.forced.pop(0)
                continue
            self._emit(f, t)
        if pre:
            self._finish_prefill(pre, plog)
        self.timer.record("mixed" if pre else "decode", len(flights), time.perf_counter() - t0)

    # ------------------------------------------------------------------ one-step overlap
    def _overlap_step(self) -> None:
        """Launch the next decode step before reading the previous one back: rows of lanes that
        were in the in-flight step take their input token from its on-device argmax, so the host's
        read-back, emission and bookkeeping of step n run while the GPU computes step n+1. A lane
        whose last token (by length) the in-flight step produces is left out of the new launch, so
        its state at read-back is exactly its history and its turn-close node can be published;
        a lane that stops on a stop token rides one extra step whose token is dropped, and publishes
        no turn-close node (its state already holds that token). Greedy lanes only; anything else
        drains the pipeline first. Reference behaviour: ``scheduler.py:1850-1948`` (overlap)."""
        prev = self.inflight
        in_prev = {id(f): i for i, f in enumerate(prev.flights)} if prev is not None else {}
        fin_prev = prev.finishing if prev is not None else set()
        launch = [f for f in self.decoding if id(f) not in fin_prev and not f.done]
        t0 = time.perf_counter()
        new = None
        if launch:
            self._grow(launch, [f.pos + 1 for f in launch])
            toks = [-1 if id(f) in in_prev else f.next_token for f in launch]
            src = [in_prev.get(id(f), 0) for f in launch]
            finishing = {id(f) for f in launch
                         if f.generated + (1 if id(f) in in_prev else 0) + 1 >= f.req.max_new}
            keep = [i for i, f in enumerate(launch) if id(f) in finishing]
            handle = self.runner.decode_launch([f.lane for f in launch], toks, [f.pos for f in launch], src, keep)
            for f in launch:
                f.pos += 1
            new = _Inflight(handle, launch, finishing)
        self.inflight = new
        if prev is not None:
            self._collect(prev)
        self.timer.record("decode", len(launch), time.perf_counter() - t0)

    def _collect(self, inf: _Inflight) -> None:
        ids = self.runner.decode_collect(inf.handle)
        kept = self.runner.decode_kept(inf.handle)
        for i, (f, t) in enumerate(zip(inf.flights, ids)):
            if f.done:  # stopped at the previous step: this token is past its end
                continue
            f.last_logits = kept.get(i) if id(f) in inf.finishing else None
            self._emit(f, int(t))

    def _complete_inflight(self) -> None:
        inf, self.inflight = self.inflight, None
        if inf is not None:
            self._collect(inf)

    def _spec_ok(self, flights: Sequence[_Flight]) -> bool:
        k1 = self.runner.decode_tokens_per_step()
        return k1 > 1 and all(f.pos + k1 <= self.runner.max_seq and not f.forced for f in flights)

    def _speculative_step(self, flights: list[_Flight]) -> None:
        k1 = self.runner.decode_tokens_per_step()
        self._grow(flights, [f.pos + k1 for f in flights])
        t0 = time.perf_counter()
        budgets = [f.req.max_new - f.generated for f in flights]
        stops = [sorted(f.req.stop) for f in flights]
        committed = self.runner.speculative_decode([f.lane for f in flights], [f.next_token for f in flights],
                                                   [f.pos for f in flights], budgets, stops)
        n = 0
        for f, toks in zip(flights, committed):
            for t in toks:
                f.pos += 1
                n += 1
                f.last_logits = None
                self._emit(f, t)
                if f.done:
                    break
        self.timer.record("spec", n, time.perf_counter() - t0)

    # ================================================================== emit / finish
    def _emit(self, f: _Flight, tok: int) -> None:
        req = f.req
        if req.first_token_at is None:
            req.first_token_at = time.perf_counter()
        if tok in req.stop:
            self._finish(f, "stop")
            return
        f.generated += 1
        f.out_ids.append(tok)
        f.next_token = tok
        req.emit(("tok", tok))
        if f.generated >= req.max_new:
            self._finish(f, "length")

    def _publish(self, f: _Flight, tokens: Sequence[int], depth: int, logits) -> None:
        if depth <= f.parent.depth or logits is None:
            return
        try:
            snap = self.cache.reserve_snapshot([f.parent] + self._live_parents())
        except SessionCacheError:
            return
        self.runner.save_snapshot(f.lane, snap)
        self.runner.cache_node_logits(snap, logits)
        # the node this flight last extended (its admission node, or its own turn-open node when
        # the turn closes) is now behind the conversation: superseded, its snapshot reclaimable
        node = self.cache.publish(tokens, depth, f.blocks, snap, resumed_from=f.parent)
        f.parent = node

    def _finish(self, f: _Flight, reason: str) -> None:
        if f.done:
            return
        f.done = True
        full = list(f.req.prompt) + f.out_ids
        if f.pos > len(f.req.prompt) and f.last_logits is not None:
            self._publish(f, full, f.pos, f.last_logits)
        self._release(f)
        f.req.emit(("end", (reason, f.generated, f.reused)))
        self.finished += 1
        if self.cache_stats_every and self.finished % self.cache_stats_every == 0:
            self._log_cache_stats()

    def _log_cache_stats(self) -> None:
        """One ``[cache-stats]`` line: admissions by class, hit rate, snapshot and block use."""
        st = self.cache.stats()
        adm = " ".join(f"{k}={v}" for k, v in sorted(st.admissions.items()))
        print(f"[cache-stats] finished={self.finished} {adm} nodes={st.nodes} snapshots={st.snapshots_used}/"
              f"{st.snapshots_capacity} free_blocks={st.free_blocks} evictions={st.evictions} "
              f"reclaims={st.reclaims} hits={st.hits} misses={st.misses}", flush=True)

    def _release(self, f: _Flight) -> None:
        if f in self.decoding:
            self.decoding.remove(f)
        if f in self.prefilling:
            self.prefilling.remove(f)
        self.cache.release_lane_blocks(f.blocks)
        f.blocks = []
        self.free_lanes.append(f.lane)

    def _abort_all(self, msg: str) -> None:
        self.inflight = None
        for f in list(self.prefilling) + list(self.decoding):
            f.done = True
            try:
                self._release(f)
            except Exception:  # pragma: no cover - best effort
                pass
            f.req.emit(("error", msg))
        self.prefilling.clear()
        self.decoding.clear()

    # ================================================================== score
    def _run_score(self, job: ScoreJob) -> None:
        if not self.free_lanes:
            self.incoming.put(job)
            return
        lane = self.free_lanes.pop()
        blocks: list[int] = []
        try:
            blocks = self.cache.reserve_blocks(blocks_for(len(job.ids), self.block_size), self._live_parents())
            self.runner.begin(lane)
            self.runner.attach_blocks(lane, blocks)
            job.result = job.finish(self.runner.score(lane, job.ids, job.continuation_start))
        except Exception as e:
            job.error = f"{type(e).__name__}: {e}"
        finally:
            if blocks:
                self.cache.release_lane_blocks(blocks)
            self.free_lanes.append(lane)
            job.done.set()
