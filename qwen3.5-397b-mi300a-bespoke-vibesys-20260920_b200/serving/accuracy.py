"""Accuracy gates for a running server (exit 0 iff every gate passes).

    python -m qwen35_b200.serving.accuracy make-pins --model tiny --out pins.json
    python -m qwen35_b200.serving.accuracy check --url http://127.0.0.1:8000 --pins pins.json

Gates:

* **sessions** - multi-turn chat sessions through ``/v1/chat/completions`` (thinking off): every
  reply is non-empty with finish reason ``stop`` or ``length``, ``prompt_tokens`` grows from turn
  to turn, and every turn >= 2 reports cached prompt tokens (the session cache resumed it);
* **pins** - greedy-token pins: each pin's prompt ids go to ``/v1/completions`` (token ids in
  and out, so no re-tokenisation slack is needed) with ``max_tokens = n_tokens``, temperature 0
  and EOS ignored; at least ``MIN_EXACT_FRACTION`` of the pins must match all ``n_tokens`` ids
  and every other pin's first mismatch must come at index ``MIN_DIVERGENCE_POSITION`` or later;
* **semantic** (``--semantic``, trained checkpoints only) - a fact from turn 1 asked back in
  turn 3, and small arithmetic questions, checked by substring.

Pins come from ``make-pins``: the model built on the CPU in fp32 (random-init ``tiny``/``full``
geometry from a seed, or a checkpoint directory), each pin's continuation generated greedily by
re-running the whole sequence from scratch for every new token (no KV cache, no session cache,
no batching): an independent forward of the same weights that the served path (cached, batched,
bf16, graph-replayed) must reproduce.

Pins file: ``{"version": 1, "model": str, "seed": int, "n_tokens": int, "pins": [{"id": str,
"prompt_ids": [int], "expected_token_ids": [int]}]}``; fewer than ``MIN_PINS`` pins is an error.

Reference behaviour: ``accuracy_checker/checker.py`` (gates and budgets), ``make_pins.py``.
"""

from __future__ import annotations

import argparse
import json
import random
import sys

EXACT_PREFIX_TOKENS = 32
MIN_EXACT_FRACTION = 0.9
MIN_DIVERGENCE_POSITION = 8
MIN_PINS = 8


class PinsError(ValueError):
    pass


def load_pins(path: str) -> dict:
    try:
        with open(path) as f:
            d = json.load(f)
    except (OSError, json.JSONDecodeError) as e:
        raise PinsError(f"pins file {path}: {e}") from e
    pins = d.get("pins") if isinstance(d, dict) else None
    if d.get("version") != 1 or not isinstance(pins, list):
        raise PinsError(f"pins file {path}: expected version 1 with a list of pins")
    if len(pins) < MIN_PINS:
        raise PinsError(f"pins file {path}: {len(pins)} pins, at least {MIN_PINS} needed")
    for p in pins:
        if not (isinstance(p.get("prompt_ids"), list) and isinstance(p.get("expected_token_ids"), list)):
            raise PinsError(f"pins file {path}: pin {p.get('id')} lacks prompt_ids / expected_token_ids")
    return d


def make_pins(model: str = "tiny", n_pins: int = 10, n_tokens: int = EXACT_PREFIX_TOKENS, seed: int = 0,
              prompt_len: tuple[int, int] = (16, 200)) -> dict:
    """Greedy pins from uncached fp32 forwards on the CPU (see the module docstring)."""
    import torch

    from .engine import PoolSpec, build_model

    torch.manual_seed(seed)
    dev = torch.device("cpu")
    spec = PoolSpec(lanes=1, max_seq=prompt_len[1] + n_tokens + 16, kv_tokens=2 * (prompt_len[1] + n_tokens + 16),
                    snapshots=1)
    m, _ = build_model(model, 0, 1, dev, spec, dtype=torch.float32, seed=seed, graphs=False)
    vocab = min(m.cfg.vocab - 16, 150000)
    r = random.Random(seed + 1)
    pins = []
    for i in range(n_pins):
        seq = [r.randrange(vocab) for _ in range(r.randint(*prompt_len))]
        n0 = len(seq)
        with torch.inference_mode():
            for _ in range(n_tokens):
                m.begin(0)
                m.attach_blocks(0, list(range(1, 1 + (len(seq) + m.block_size) // m.block_size + 1)))
                lg = m.prefill(0, seq, 0)
                seq.append(m.sample_batch(lg, [0.0])[0])
        pins.append({"id": f"pin{i:02d}", "prompt_ids": seq[:n0], "expected_token_ids": seq[n0:]})
    return {"version": 1, "model": model, "seed": seed, "n_tokens": n_tokens, "pins": pins}


def _post(url: str, path: str, body: dict, timeout: float = 600.0) -> dict:
    import requests

    r = requests.post(url + path, json=body, timeout=timeout)
    r.raise_for_status()
    return r.json()


def check_pins(url: str, pins: dict) -> dict:
    n = int(pins.get("n_tokens", EXACT_PREFIX_TOKENS))
    rows = []
    for p in pins["pins"]:
        got = _post(url, "/v1/completions", {"prompt": p["prompt_ids"], "max_tokens": n, "temperature": 0.0,
                                             "ignore_eos": True})["choices"][0]["token_ids"]
        exp = p["expected_token_ids"][:n]
        first = next((i for i, (a, b) in enumerate(zip(got, exp)) if a != b), None)
        if first is None and len(got) != len(exp):
            first = min(len(got), len(exp))
        rows.append({"id": p["id"], "exact": first is None, "first_mismatch": first})
    exact = sum(r["exact"] for r in rows) / max(1, len(rows))
    early = [r for r in rows if not r["exact"] and r["first_mismatch"] < MIN_DIVERGENCE_POSITION]
    return {"gate": "pins", "pass": exact >= MIN_EXACT_FRACTION and not early, "exact_fraction": exact,
            "early_divergence": [r["id"] for r in early], "pins": rows}


def check_sessions(url: str, sessions: int = 6, turns: int = 3, seed: int = 7, max_tokens: int = 24) -> dict:
    r = random.Random(seed)
    words = "cache block expert router state token layer prefix reply turn history window".split()
    problems = []
    for s in range(sessions):
        msgs, last_prompt = [], 0
        for t in range(turns):
            msgs.append({"role": "user", "content": " ".join(r.choice(words) for _ in range(r.randint(8, 40)))})
            o = _post(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": max_tokens, "temperature": 0.0,
                                                    "chat_template_kwargs": {"enable_thinking": False}})
            ch, u = o["choices"][0], o["usage"]
            text = ch["message"]["content"]
            if ch.get("finish_reason") not in ("stop", "length"):
                problems.append(f"s{s}t{t}: finish_reason {ch.get('finish_reason')!r}")
            if u["completion_tokens"] < 1:
                problems.append(f"s{s}t{t}: no tokens")
            if u["prompt_tokens"] <= last_prompt:
                problems.append(f"s{s}t{t}: prompt_tokens {u['prompt_tokens']} did not grow from {last_prompt}")
            if t > 0 and u.get("prompt_tokens_details", {}).get("cached_tokens", 0) <= 0:
                problems.append(f"s{s}t{t}: no cached prompt tokens")
            last_prompt = u["prompt_tokens"]
            msgs.append({"role": "assistant", "content": text})
    return {"gate": "sessions", "pass": not problems, "problems": problems[:20]}


def check_semantic(url: str) -> dict:
    """Recall and arithmetic probes; only a trained checkpoint can pass them."""
    problems = []
    facts = [("My cat is called Tobermory.", "What is my cat called?", "Tobermory"),
             ("I was born in Reykjavik.", "In which city was I born?", "Reykjavik")]
    for fact, q, want in facts:
        msgs = [{"role": "user", "content": fact + " Please remember it."}]
        for content in (None, "Tell me a short joke.", q):
            if content is not None:
                msgs.append({"role": "user", "content": content})
            o = _post(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 48, "temperature": 0.0,
                                                    "chat_template_kwargs": {"enable_thinking": False}})
            msgs.append({"role": "assistant", "content": o["choices"][0]["message"]["content"]})
        if want.lower() not in msgs[-1]["content"].lower():
            problems.append(f"recall {want!r} missing from {msgs[-1]['content'][:80]!r}")
    for a, b in ((17, 25), (123, 456), (9, 8)):
        o = _post(url, "/v1/chat/completions", {
            "messages": [{"role": "user", "content": f"What is {a} + {b}? Answer with the number only."}],
            "max_tokens": 16, "temperature": 0.0, "chat_template_kwargs": {"enable_thinking": False}})
        if str(a + b) not in o["choices"][0]["message"]["content"]:
            problems.append(f"{a}+{b}: {o['choices'][0]['message']['content'][:40]!r}")
    return {"gate": "semantic", "pass": not problems, "problems": problems}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="accuracy gates for a running server")
    sub = ap.add_subparsers(dest="cmd", required=True)
    mk = sub.add_parser("make-pins")
    mk.add_argument("--model", default="tiny")
    mk.add_argument("--n", type=int, default=10)
    mk.add_argument("--tokens", type=int, default=EXACT_PREFIX_TOKENS)
    mk.add_argument("--seed", type=int, default=0)
    mk.add_argument("--out", required=True)
    ck = sub.add_parser("check")
    ck.add_argument("--url", required=True)
    ck.add_argument("--pins", default=None)
    ck.add_argument("--skip-pins", action="store_true")
    ck.add_argument("--semantic", action="store_true")
    ck.add_argument("--output-json", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "make-pins":
        d = make_pins(a.model, a.n, a.tokens, a.seed)
        with open(a.out, "w") as f:
            json.dump(d, f)
        print(f"{len(d['pins'])} pins of {d['n_tokens']} tokens -> {a.out}")
        return 0
    url = a.url.rstrip("/")
    gates = [check_sessions(url)]
    if not a.skip_pins:
        if not a.pins:
            gates.append({"gate": "pins", "pass": False, "problems": ["no --pins file given"]})
        else:
            try:
                gates.append(check_pins(url, load_pins(a.pins)))
            except PinsError as e:
                gates.append({"gate": "pins", "pass": False, "problems": [str(e)]})
    if a.semantic:
        gates.append(check_semantic(url))
    res = {"pass": all(g["pass"] for g in gates), "gates": gates}
    print(json.dumps(res), flush=True)
    if a.output_json:
        with open(a.output_json, "w") as f:
            json.dump(res, f)
    return 0 if res["pass"] else 1


if __name__ == "__main__":
    sys.exit(main())
