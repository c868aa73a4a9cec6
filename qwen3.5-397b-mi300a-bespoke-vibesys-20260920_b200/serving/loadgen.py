"""HTTP load generator: multi-turn sessions against a running server, concurrency ramp.

    python -m qwen35_b200.serving.loadgen --url http://127.0.0.1:8000 --levels 8 16 32 \\
        --warmup 10 --window 60 --c-ref 16 --out ramp.json [--mode chat|ids]

Every level holds exactly ``C`` requests in flight: ``C`` client tasks each run sessions back to
back (a session is 3-6 turns; each turn appends a user message to the full history and asks
for a fixed number of greedy tokens with EOS ignored; an optional think time separates turns).
``chat`` mode sends OpenAI chat messages (pseudo-word paragraphs) to ``/v1/chat/completions``
with SSE streaming and thinking off; ``ids`` mode sends token-id prompts to ``/v1/completions``
(streamed ``token_ids``), the id-level form of the same sessions, for checkpoints without a text
tokenizer. Time to first token is taken at the first chunk that carries generated content (at
the finish chunk for a reply whose tokens decode to no text).

Per level: a warm-up, then a measurement window; the level's turns are those STARTED inside
the window, and the level ends only when every one of them has finished (no right-censoring:
a slow turn is waited for, not dropped). Reported per level: goodput (their generated tokens /
time from window start to the last of them ending), p50/p95 TTFT over turns >= 2 and over all
turns, p95 time per output token, and failed / empty / short turns. The ramp stops at a level
with any failed turn, at a p95 TTFT (turns >= 2) above ``--ttft-guard-ms``, or when goodput
grows by less than ``--plateau`` over the best level so far. The result: the level table,
``peak_goodput_tok_s`` and ``p95_ttft_turn2plus_ms_at_ref`` (the level ``C == --c-ref``).

Reference behaviour: ``benchmark/run.py`` (in-flight load controller, per-level warm-up and
window, stop rules, drained reporting), ``benchmark/launcher.py``.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from dataclasses import asdict, dataclass, field

WORDS = ("the model routes every token through ten of five hundred twelve experts while the "
         "recurrent layers keep a fixed size state and the attention layers page their keys and "
         "values through a shared block pool so long conversations reuse what was computed before "
         "cache hit prefill decode latency throughput session history turn reply question answer").split()


@dataclass
class LoadSpec:
    levels: tuple[int, ...] = (8, 16, 32)
    warmup_s: float = 10.0
    window_s: float = 60.0
    turns: tuple[int, int] = (3, 6)
    words: tuple[int, int] = (30, 300)          # chat mode: words per user message
    ids: tuple[int, int] = (200, 1000)          # ids mode: ids per user message (turn 1: first_ids)
    first_ids: tuple[int, int] = (2000, 8000)
    max_tokens: tuple[int, int] = (80, 300)
    think_s: tuple[float, float] = (0.0, 0.0)
    vocab: int = 150000
    seed: int = 20261202
    ttft_guard_ms: float = 10_000.0
    plateau: float = 0.05
    c_ref: int = 16
    mode: str = "chat"
    timeout_s: float = 600.0


@dataclass
class Turn:
    session: int
    turn: int
    level: int
    t_start: float
    ttft_ms: float | None = None
    t_end: float | None = None
    tokens: int = 0
    expected: int = 0
    prompt_tokens: int = 0
    cached_tokens: int = 0
    error: str | None = None
    itl_ms: list[float] = field(default_factory=list)


class SessionStream:
    """An unbounded deterministic stream of sessions: session ``i`` is a function of (seed, i)."""

    def __init__(self, spec: LoadSpec):
        self.spec = spec
        self.next = 0

    def take(self) -> tuple[int, list[tuple[object, int]]]:
        i = self.next
        self.next += 1
        r = random.Random(self.spec.seed * 1_000_003 + i)
        n = r.randint(*self.spec.turns)
        turns = []
        for t in range(n):
            if self.spec.mode == "chat":
                msg = " ".join(r.choice(WORDS) for _ in range(r.randint(*self.spec.words)))
            else:
                lo, hi = self.spec.first_ids if t == 0 else self.spec.ids
                msg = [r.randrange(self.spec.vocab) for _ in range(r.randint(lo, hi))]
            turns.append((msg, r.randint(*self.spec.max_tokens)))
        return i, turns


def _percentile(xs: list[float], q: float) -> float | None:
    if not xs:
        return None
    s = sorted(xs)
    k = (len(s) - 1) * q / 100.0
    lo, hi = int(k), min(int(k) + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)


async def _sse(resp):
    """Yields the JSON payloads of an SSE response until ``data: [DONE]``."""
    buf = b""
    async for chunk in resp.content.iter_any():
        buf += chunk
        while b"\n\n" in buf:
            event, buf = buf.split(b"\n\n", 1)
            for line in event.split(b"\n"):
                if not line.startswith(b"data: "):
                    continue
                data = line[6:]
                if data == b"[DONE]":
                    return
                yield json.loads(data)


async def run_turn(http, url: str, spec: LoadSpec, rec: Turn, history, msg, max_tokens: int):
    """One streamed turn; returns the reply (text in chat mode, ids in ids mode) and fills ``rec``."""
    if spec.mode == "chat":
        body = {"messages": history + [{"role": "user", "content": msg}], "max_tokens": max_tokens,
                "temperature": 0.0, "ignore_eos": True, "stream": True,
                "stream_options": {"include_usage": True}, "chat_template_kwargs": {"enable_thinking": False}}
        path = "/v1/chat/completions"
    else:
        body = {"prompt": history + msg, "max_tokens": max_tokens, "temperature": 0.0, "ignore_eos": True,
                "stream": True, "stream_options": {"include_usage": True}}
        path = "/v1/completions"
    rec.expected = max_tokens
    text, ids = [], []
    last = t_fin = None
    try:
        async with http.post(url + path, json=body) as resp:
            if resp.status != 200:
                rec.error = f"HTTP {resp.status}: {(await resp.text())[:200]}"
                return None
            async for o in _sse(resp):
                if "error" in o:
                    rec.error = str(o["error"])[:200]
                    return None
                if o.get("usage"):
                    u = o["usage"]
                    rec.tokens = int(u.get("completion_tokens", 0))
                    rec.prompt_tokens = int(u.get("prompt_tokens", 0))
                    rec.cached_tokens = int((u.get("prompt_tokens_details") or {}).get("cached_tokens", 0))
                for ch in o.get("choices") or []:
                    piece = (ch.get("delta") or {}).get("content") if spec.mode == "chat" else ch.get("token_ids")
                    if ch.get("finish_reason") and t_fin is None:
                        t_fin = time.perf_counter()
                    if not piece:
                        continue
                    now = time.perf_counter()
                    if rec.ttft_ms is None:
                        rec.ttft_ms = (now - rec.t_start) * 1e3
                    elif last is not None:
                        rec.itl_ms.append((now - last) * 1e3)
                    last = now
                    (text.append(piece) if spec.mode == "chat" else ids.extend(piece))
    except Exception as e:  # connection reset, timeout: a failed turn
        rec.error = f"{type(e).__name__}: {e}"[:200]
        return None
    finally:
        rec.t_end = time.perf_counter()
    if rec.ttft_ms is None:
        if rec.tokens <= 0 or t_fin is None:
            rec.error = rec.error or "empty reply"
            return None
        # tokens that decode to no text (a byte tokenizer's partial characters): the first token
        # is known to have come by the finish chunk
        rec.ttft_ms = (t_fin - rec.t_start) * 1e3
    return "".join(text) if spec.mode == "chat" else ids


async def run_level(url: str, spec: LoadSpec, C: int, stream: SessionStream, http=None) -> dict:
    """Holds ``C`` requests in flight for warm-up + window, then drains the window's turns."""
    import aiohttp

    own = http is None
    if own:
        http = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=spec.timeout_s))
    t0 = time.perf_counter()
    w0, w1 = t0 + spec.warmup_s, t0 + spec.warmup_s + spec.window_s
    turns: list[Turn] = []

    async def client():
        while time.perf_counter() < w1:
            sid, plan = stream.take()
            history: list = []
            for t, (msg, n) in enumerate(plan):
                if time.perf_counter() >= w1:
                    return
                rec = Turn(sid, t, C, time.perf_counter())
                turns.append(rec)
                reply = await run_turn(http, url, spec, rec, history, msg, n)
                if reply is None:
                    break
                if spec.mode == "chat":
                    history = history + [{"role": "user", "content": msg}, {"role": "assistant", "content": reply}]
                else:
                    history = history + msg + reply
                if spec.think_s[1] > 0:
                    await asyncio.sleep(random.Random(sid * 31 + t).uniform(*spec.think_s))

    try:
        await asyncio.gather(*(client() for _ in range(C)))
    finally:
        if own:
            await http.close()
    win = [r for r in turns if w0 <= r.t_start < w1]
    ok = [r for r in win if r.error is None]
    failed = [r for r in win if r.error is not None]
    short = [r for r in ok if r.tokens and r.tokens < r.expected]
    t_last = max((r.t_end for r in win if r.t_end is not None), default=w1)
    gen = sum(r.tokens for r in ok)
    ttft2 = [r.ttft_ms for r in ok if r.turn >= 1]
    return {
        "concurrency": C, "turns": len(win), "turns_ge2": len(ttft2), "failed": len(failed), "short": len(short),
        "goodput_tok_s": round(gen / max(1e-9, t_last - w0), 2),
        "p50_ttft_turn2plus_ms": _percentile(ttft2, 50), "p95_ttft_turn2plus_ms": _percentile(ttft2, 95),
        "p95_ttft_all_ms": _percentile([r.ttft_ms for r in ok], 95),
        "p95_tpot_ms": _percentile([x for r in ok for x in r.itl_ms], 95),
        "cached_token_share": round(sum(r.cached_tokens for r in ok) / max(1, sum(r.prompt_tokens for r in ok)), 4),
        "errors": sorted({r.error for r in failed})[:5],
        "drain_s": round(max(0.0, t_last - w1), 2),
    }


async def ramp(url: str, spec: LoadSpec) -> dict:
    """The concurrency ramp with its stop rules; returns the whole result."""
    stream = SessionStream(spec)
    levels, best, stop = [], 0.0, None
    for C in spec.levels:
        lv = await run_level(url, spec, C, stream)
        levels.append(lv)
        if lv["failed"]:
            stop = f"level C={C}: {lv['failed']} failed turns"
            break
        p95 = lv["p95_ttft_turn2plus_ms"]
        if p95 is not None and p95 > spec.ttft_guard_ms:
            stop = f"level C={C}: p95 TTFT turns>=2 {p95:.0f} ms above the {spec.ttft_guard_ms:.0f} ms guard"
            break
        if best and lv["goodput_tok_s"] < best * (1 + spec.plateau):
            stop = f"level C={C}: goodput plateau ({lv['goodput_tok_s']:.0f} vs best {best:.0f} tok/s)"
            best = max(best, lv["goodput_tok_s"])
            break
        best = max(best, lv["goodput_tok_s"])
    ref = next((lv for lv in levels if lv["concurrency"] == spec.c_ref), None)
    return {"spec": asdict(spec), "levels": levels, "stop": stop,
            "peak_goodput_tok_s": max((lv["goodput_tok_s"] for lv in levels), default=0.0),
            "p95_ttft_turn2plus_ms_at_ref": ref["p95_ttft_turn2plus_ms"] if ref else None}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--url", required=True)
    ap.add_argument("--levels", type=int, nargs="+", default=list(LoadSpec.levels))
    ap.add_argument("--warmup", type=float, default=LoadSpec.warmup_s)
    ap.add_argument("--window", type=float, default=LoadSpec.window_s)
    ap.add_argument("--turns", type=int, nargs=2, default=LoadSpec.turns)
    ap.add_argument("--words", type=int, nargs=2, default=LoadSpec.words)
    ap.add_argument("--ids", type=int, nargs=2, default=LoadSpec.ids)
    ap.add_argument("--first-ids", type=int, nargs=2, default=LoadSpec.first_ids)
    ap.add_argument("--max-tokens", type=int, nargs=2, default=LoadSpec.max_tokens)
    ap.add_argument("--think", type=float, nargs=2, default=LoadSpec.think_s)
    ap.add_argument("--vocab", type=int, default=LoadSpec.vocab)
    ap.add_argument("--seed", type=int, default=LoadSpec.seed)
    ap.add_argument("--ttft-guard-ms", type=float, default=LoadSpec.ttft_guard_ms)
    ap.add_argument("--plateau", type=float, default=LoadSpec.plateau)
    ap.add_argument("--c-ref", type=int, default=LoadSpec.c_ref)
    ap.add_argument("--mode", choices=["chat", "ids"], default="chat")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    spec = LoadSpec(levels=tuple(a.levels), warmup_s=a.warmup, window_s=a.window, turns=tuple(a.turns),
                    words=tuple(a.words), ids=tuple(a.ids), first_ids=tuple(a.first_ids),
                    max_tokens=tuple(a.max_tokens), think_s=tuple(a.think), vocab=a.vocab, seed=a.seed,
                    ttft_guard_ms=a.ttft_guard_ms, plateau=a.plateau, c_ref=a.c_ref, mode=a.mode)
    res = asyncio.run(ramp(a.url.rstrip("/"), spec))
    line = json.dumps(res)
    print(line, flush=True)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    return res


if __name__ == "__main__":
    main()
