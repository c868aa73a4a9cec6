"""Synthetic multi-turn chat workload (token ids) and a closed-loop driver over the scheduler.

Shape (the headline benchmark configuration): ``sessions`` conversations of ``turns`` turns at a
closed-loop concurrency of ``concurrency``; the first user message is uniform
``first_len`` random token ids, every later user message is uniform ``user_len`` ids appended
to the full prior history (including the model's own reply), every turn generates uniform
``gen_len`` tokens greedily with EOS ignored, and there is no think time. All lengths and ids
come from ``seed``. The reference's own benchmark (``benchmark/run.py:71-126``) drives text chat
over HTTP with think times; this generator is the token-id form used for the B200 numbers.
"""

from __future__ import annotations

import random
import time
from dataclasses import dataclass, field



def _our_request(prompt, max_new, emit, has_history):
    from .scheduler import Request

    return Request(prompt, max_new, emit, temperature=0.0, has_history=has_history)


@dataclass(frozen=True)
class ChatSpec:
    sessions: int = 256
    concurrency: int = 32
    turns: int = 6
    first_len: tuple[int, int] = (2000, 8000)
    user_len: tuple[int, int] = (200, 1000)
    gen_len: tuple[int, int] = (200, 500)
    vocab: int = 151000
    seed: int = 0


@dataclass
class TurnRecord:
    session: int
    turn: int
    prompt_len: int
    max_new: int
    submit_step: int
    t_submit: float
    first_step: int = -1
    t_first: float = 0.0
    end_step: int = -1
    t_end: float = 0.0
    generated: int = 0
    reused: int = 0
    error: str | None = None


@dataclass
class _Session:
    sid: int
    history: list[int]
    turn: int
    rng: random.Random
    lengths: list[tuple[int, int]] = field(default_factory=list)  # (user_len, gen_len) per turn


class ClosedLoop:
    """Keeps ``spec.concurrency`` sessions in flight; a session's next turn is submitted as soon
    as its previous turn ends. ``step_index`` is read from the caller (the index of the next
    scheduler step) so device-side step events can be matched to each turn. ``make_request``
    builds the scheduler's request object from ``(prompt, max_new, emit, has_history)`` (this
    package's ``Request`` by default; another engine's scheduler can be driven the same way)."""

    def __init__(self, scheduler, spec: ChatSpec, step_index=lambda: 0, max_turn: int | None = None,
                 make_request=None):
        self.sched = scheduler
        self.make_request = make_request or _our_request
        self.spec = spec
        self.step_index = step_index
        self.max_turn = max_turn or spec.turns
        self.rng = random.Random(spec.seed)
        self.next_sid = 0
        self.active: dict[int, _Session] = {}
        self.records: list[TurnRecord] = []
        self.finished_sessions = 0
        self._done: list[tuple[_Session, TurnRecord, list[int]]] = []

    def _new_session(self) -> _Session:
        sid = self.next_sid
        self.next_sid += 1
        r = random.Random(self.spec.seed * 1_000_003 + sid)
        s = self.spec
        lens = [(r.randint(*s.first_len), r.randint(*s.gen_len))]
        lens += [(r.randint(*s.user_len), r.randint(*s.gen_len)) for _ in range(s.turns - 1)]
        return _Session(sid, [], 0, r, lens)

    def _submit(self, sess: _Session) -> None:
        ulen, glen = sess.lengths[sess.turn]
        sess.history = sess.history + [sess.rng.randrange(self.spec.vocab) for _ in range(ulen)]
        rec = TurnRecord(sess.sid, sess.turn, len(sess.history), glen, self.step_index(), time.perf_counter())
        toks: list[int] = []
        self.records.append(rec)

        def emit(ev, rec=rec, toks=toks, sess=sess):
            kind, val = ev
            if kind == "tok":
                if not toks:
                    rec.first_step = self.step_index()
                    rec.t_first = time.perf_counter()
                toks.append(val)
            elif kind == "end":
                rec.end_step = self.step_index()
                rec.t_end = time.perf_counter()
                rec.generated = val[1]
                rec.reused = val[2]
                self._done.append((sess, rec, toks))
            else:
                rec.error = str(val)
                rec.end_step = self.step_index()
                self._done.append((sess, rec, toks))

        self.sched.submit(self.make_request(list(sess.history), glen, emit, sess.turn > 0))

    def start(self) -> None:
        while len(self.active) < self.spec.concurrency and self.next_sid < self.spec.sessions:
            s = self._new_session()
            self.active[s.sid] = s
            self._submit(s)

    def pump(self) -> int:
        """Handle turns that ended since the last call; returns how many ended."""
        done, self._done = self._done, []
        for sess, rec, toks in done:
            sess.history = sess.history + toks
            sess.turn += 1
            if rec.error is None and sess.turn < min(self.max_turn, self.spec.turns):
                self._submit(sess)
            else:
                del self.active[sess.sid]
                self.finished_sessions += 1
                if self.next_sid < self.spec.sessions:
                    s = self._new_session()
                    self.active[s.sid] = s
                    self._submit(s)
        return len(done)


def percentile(xs: list[float], q: float) -> float:
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * q / 100.0
    lo, hi = int(k), min(int(k) + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)
