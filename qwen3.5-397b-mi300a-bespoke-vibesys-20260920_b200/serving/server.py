"""OpenAI-compatible HTTP server and process launcher.

    python -m qwen35_b200.serving.server --model-path DIR|full|tiny --tp N --port 8000

Rank 0 serves HTTP, runs the scheduler thread and drives the other ranks through the SPMD
command protocol (``parallel.driver``); it re-executes this module once per extra rank with
``--rank r`` (one process per GPU). Endpoints (reference ``server.py:1162-1183``):

* ``GET /health`` - 200 once the model is loaded and every worker process is alive, else 503;
* ``GET /v1/models``;
* ``POST /v1/chat/completions`` - streaming SSE (``data: [DONE]`` terminated) and non-streaming;
  honours ``max_tokens``, ``temperature``, ``ignore_eos``, ``chat_template_kwargs.enable_thinking``
  and ``stream_options.include_usage``; ``usage.prompt_tokens_details.cached_tokens`` reports
  prompt tokens served from the session cache;
* ``POST /v1/completions`` - ``prompt`` as text or as a list of token ids; the response carries
  the generated ``token_ids`` too (the id-level benchmark workloads use it);
* ``POST /reset_prefix_cache``; ``POST /v1/score`` (teacher-forced log-probabilities);
* ``POST /debug/fault`` (only with ``QB_FAULT_ENDPOINT=1``) - accuracy-gate calibration faults.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import subprocess
import sys
import threading
import time
import uuid

import torch

from ..utils import flags


def stop_ids(model_dir: str | None, cfg_eos: int, tok) -> frozenset[int]:
    """Ids that end a generation: the config's eos, every ``eos_token_id`` of the checkpoint's
    ``generation_config.json`` (chat checkpoints list the end-of-turn token there too) and the
    tokenizer's eos."""
    ids = {int(cfg_eos)}
    if model_dir:
        gen = os.path.join(model_dir, "generation_config.json")
        if os.path.exists(gen):
            with open(gen) as f:
                eos = json.load(f).get("eos_token_id", [])
            ids |= {int(eos)} if isinstance(eos, int) else {int(e) for e in eos}
    if getattr(tok, "eos_token_id", None) is not None:
        ids.add(int(tok.eos_token_id))
    return frozenset(ids)


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-path", default=os.environ.get("MODEL_PATH", "tiny"))
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--rank", type=int, default=0)
    ap.add_argument("--master-port", type=int, default=29555)
    ap.add_argument("--max-seq-len", type=int, default=16384)
    ap.add_argument("--max-batch", type=int, default=32)
    ap.add_argument("--kv-tokens", type=int, default=None)
    ap.add_argument("--snapshots", type=int, default=None)
    ap.add_argument("--prefill-chunk", type=int, default=2048)
    ap.add_argument("--token-budget", type=int, default=2048)
    ap.add_argument("--device", default="auto", choices=["auto", "cuda", "cpu"])
    ap.add_argument("--dtype", default="auto", choices=["auto", "bf16", "fp32"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--mtp-k", type=int, default=0,
                    help="MTP speculative decoding with this draft depth (0: off; the checkpoint needs mtp.*)")
    ap.add_argument("--mtp-forced-accept", type=float, default=None,
                    help="accept each draft position with this probability instead of greedy (benchmarking)")
    ap.add_argument("--mixed", action="store_true", help="decode steps also carry prefill chunks")
    ap.add_argument("--prefill-graphs", default=None,
                    help="widths (comma-separated token counts) of captured single-segment prefill steps, e.g. "
                         "the prefill chunk size: a prompt chunk of exactly that length replays its graph "
                         "(sets QB_PREFILL_GRAPHS on every rank)")
    ap.add_argument("--mixed-graphs", default=None,
                    help="decode-rows:prefill-width pairs of captured mixed steps (with --mixed), e.g. 32:256 "
                         "(sets QB_MIXED_GRAPHS on every rank)")
    args = ap.parse_args(argv)
    if args.mixed_graphs is not None:
        flags.put("QB_MIXED_GRAPHS", args.mixed_graphs)
    if args.prefill_graphs is not None:
        flags.put("QB_PREFILL_GRAPHS", args.prefill_graphs)  # read when the model and its graphs are built
    return args


def _device(args):
    use_cuda = args.device == "cuda" or (args.device == "auto" and torch.cuda.is_available())
    return torch.device("cuda", args.rank % max(1, torch.cuda.device_count())) if use_cuda else torch.device("cpu")


def _dtype(args, device):
    if args.dtype == "fp32" or (args.dtype == "auto" and device.type == "cpu"):
        return torch.float32
    return torch.bfloat16


def _init_dist(args):
    from ..parallel import comm as commmod

    os.environ.update(RANK=str(args.rank), WORLD_SIZE=str(args.tp), LOCAL_RANK=str(args.rank),
                      MASTER_ADDR=os.environ.get("MASTER_ADDR", "127.0.0.1"), MASTER_PORT=str(args.master_port))
    device = _device(args)
    if device.type == "cuda":
        torch.cuda.set_device(device)
    if args.tp > 1:
        commmod.init("nccl" if device.type == "cuda" else "gloo", timeout_s=3600)
    return device


def _build(args, device):
    from ..parallel.driver import command_group, pool_handshake
    from .engine import PoolSpec, build_model

    spec = PoolSpec(lanes=args.max_batch, max_seq=args.max_seq_len, kv_tokens=args.kv_tokens,
                    snapshots=args.snapshots)
    mtp_k = getattr(args, "mtp_k", 0)
    model, _ = build_model(args.model_path, args.rank, args.tp, device, spec, dtype=_dtype(args, device),
                           seed=args.seed, with_mtp=mtp_k > 0)
    if mtp_k > 0:
        from ..models import mtp as mtpmod

        inner = getattr(model, "model", model)  # the Model under a GraphRunner
        head = mtpmod.attach(inner, k=mtp_k, forced_accept=getattr(args, "mtp_forced_accept", None))
        if head is None:
            raise SystemExit("--mtp-k needs a checkpoint with an mtp block")
        head.rng.seed(args.seed)  # identical forced-acceptance draws on every rank
        if hasattr(model, "prepare_speculative"):
            model.prepare_speculative()
    group = command_group(args.tp)
    pool_handshake(model)
    return model, group


def run_worker(args) -> None:
    from ..parallel.driver import open_channel, serve_worker

    device = _init_dist(args)
    model, group = _build(args, device)
    serve_worker(model, open_channel(args.tp, args.rank, group, device.type))


# ============================================================================ engine
class Engine:
    """Rank 0: model + scheduler thread + tokenizer; owns the worker processes."""

    def __init__(self, args, workers: list[subprocess.Popen]):
        self.args = args
        self.workers = workers
        self.ready = False
        self.error: str | None = None
        self.sched = None
        self.runner = None
        self.tok = None
        self.stop_ids: frozenset[int] = frozenset()
        from .chat_history import ChatHistory

        self.history = ChatHistory()  # exact ids of the replies this server generated
        self.model_name = os.path.basename(str(args.model_path).rstrip("/")) or "qwen3.5"
        self.thread = threading.Thread(target=self._boot, daemon=True)
        self.thread.start()

    def _boot(self):
        try:
            from ..parallel.driver import Broadcaster, open_channel
            from .block_pool import BlockAllocator
            from .scheduler import Scheduler
            from .session_cache import SessionCache
            from .tokenizer import load_tokenizer

            device = _init_dist(self.args)
            model, group = _build(self.args, device)
            self.model = model
            self.runner = Broadcaster(model, open_channel(self.args.tp, 0, group, device.type))
            cache = SessionCache(BlockAllocator(model.num_blocks, model.block_size), model.block_size,
                                 model.num_snapshots)
            self.sched = Scheduler(self.runner, cache, prefill_chunk=self.args.prefill_chunk,
                                   token_budget=self.args.token_budget, mixed=getattr(self.args, "mixed", False),
                                   speculative=getattr(self.args, "mtp_k", 0) > 0)
            path = self.args.model_path if os.path.isdir(str(self.args.model_path)) else None
            self.tok = load_tokenizer(path, model.cfg.vocab, model.cfg.eos_token_id)
            self.stop_ids = stop_ids(path, model.cfg.eos_token_id, self.tok)
            self.ready = True
            self.sched.run()
        except Exception as e:  # surfaced through /health
            import traceback

            traceback.print_exc()
            self.error = f"{type(e).__name__}: {e}"

    def healthy(self) -> bool:
        return self.ready and self.error is None and all(w.poll() is None for w in self.workers)

    def shutdown(self):
        if self.sched is not None:
            self.sched.stop()
        if self.runner is not None and self.args.tp > 1:
            try:
                self.runner.shutdown()
            except Exception:
                pass
        for w in self.workers:
            if w.poll() is None:
                w.terminate()


# ============================================================================ HTTP
def make_app(engine: Engine):
    from aiohttp import web

    from .scheduler import Request, ScoreJob
    from .tokenizer import Detokenizer

    routes = web.RouteTableDef()

    def submit(prompt_ids, max_new, temperature, stop, suffix_len, has_history):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def emit(ev):
            loop.call_soon_threadsafe(q.put_nowait, ev)

        engine.sched.submit(Request(list(prompt_ids), int(max_new), emit, float(temperature), frozenset(stop),
                                    suffix_len, has_history))
        return q

    def stops(body):
        return set() if body.get("ignore_eos", False) else set(engine.stop_ids)

    async def stream_tokens(q, on_token):
        while True:
            kind, val = await q.get()
            if kind == "tok":
                await on_token(val)
            elif kind == "end":
                return val, None
            else:
                return None, str(val)

    @routes.get("/health")
    async def health(_):
        if engine.healthy():
            return web.json_response({"status": "ok"})
        return web.json_response({"status": "loading", "error": engine.error}, status=503)  # body as the reference gives it

    @routes.get("/v1/models")
    async def models(_):
        return web.json_response({"object": "list", "data": [{"id": engine.model_name, "object": "model"}]})

    async def generate(request, prompt_ids, suffix_len, has_history, body, chat: bool, on_done=None):
        max_new = int(body.get("max_tokens") or body.get("max_completion_tokens") or 256)
        max_new = max(1, min(max_new, engine.args.max_seq_len - len(prompt_ids)))  # clamped to the context
        temp = float(body.get("temperature", 0.0) or 0.0)
        stream = bool(body.get("stream", False))
        usage_opt = bool((body.get("stream_options") or {}).get("include_usage", False))
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        q = submit(prompt_ids, max_new, temp, stops(body), suffix_len, has_history)
        detok = Detokenizer(engine.tok)
        out_ids: list[int] = []
        obj = "chat.completion.chunk" if chat else "text_completion"

        def chunk(text=None, finish=None, role=False, ids=None):
            if chat:
                delta = {"role": "assistant"} if role else ({"content": text} if text is not None else {})
                ch = {"index": 0, "delta": delta, "finish_reason": finish}
            else:
                ch = {"index": 0, "text": text or "", "finish_reason": finish}
                if ids is not None:
                    ch["token_ids"] = ids
            return {"id": rid, "object": obj, "created": created, "model": engine.model_name, "choices": [ch]}

        if stream:
            resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
            await resp.prepare(request)

            async def send(o):
                await resp.write(b"data: " + json.dumps(o).encode() + b"\n\n")

            if chat:
                await send(chunk(role=True))

            async def on_tok(t):
                out_ids.append(t)
                text = detok.push(t)
                if text or not chat:
                    await send(chunk(text, ids=[t] if not chat else None))

            end, err = await stream_tokens(q, on_tok)
            if err is not None:
                await send({"error": {"message": err, "type": "server_error"}})
            else:
                tail = detok.flush()
                if tail:
                    await send(chunk(tail))
                if on_done is not None:
                    on_done(out_ids)
                reason = "stop" if end[0] == "stop" else "length"
                await send(chunk(None, reason))
                if usage_opt:
                    await send({"id": rid, "object": obj, "created": created, "model": engine.model_name,
                                "choices": [], "usage": usage(prompt_ids, end)})
            await resp.write(b"data: [DONE]\n\n")
            await resp.write_eof()
            return resp

        async def on_tok(t):
            out_ids.append(t)

        end, err = await stream_tokens(q, on_tok)
        if err is not None:
            return web.json_response({"error": {"message": err, "type": "server_error"}}, status=500)
        text = engine.tok.decode(out_ids)
        if on_done is not None:
            on_done(out_ids)
        reason = "stop" if end[0] == "stop" else "length"
        if chat:
            choice = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": reason}
            o = "chat.completion"
        else:
            choice = {"index": 0, "text": text, "token_ids": out_ids, "finish_reason": reason}
            o = "text_completion"
        return web.json_response({"id": rid, "object": o, "created": created, "model": engine.model_name,
                                  "choices": [choice], "usage": usage(prompt_ids, end)})

    def usage(prompt_ids, end):
        return {"prompt_tokens": len(prompt_ids), "completion_tokens": int(end[1]),
                "total_tokens": len(prompt_ids) + int(end[1]),
                "prompt_tokens_details": {"cached_tokens": int(end[2])}}

    @routes.post("/v1/chat/completions")
    async def chat(request):
        if not engine.healthy():
            return web.json_response({"error": {"message": "not ready"}}, status=503)
        body = await request.json()
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs or not all(isinstance(m, dict) and "role" in m for m in msgs):
            return web.json_response({"error": "messages must be a non-empty array of {role, content}"}, status=400)
        kw = body.get("chat_template_kwargs") or {}
        has_history = any(m.get("role") == "assistant" for m in msgs)
        stop_ids = set(engine.stop_ids)
        if getattr(engine.tok, "template", None) is not None:
            stop_ids.add(engine.tok.template.im_end)
        spliced = engine.history.splice(engine.tok, msgs, kw, stop_ids) if has_history else None
        if spliced is not None:
            ids, suffix = spliced
        else:
            ids, suffix = engine.tok.render_chat(msgs, enable_thinking=bool(kw.get("enable_thinking", False)))

        if len(ids) >= engine.args.max_seq_len:
            return web.json_response({"error": f"prompt has {len(ids)} tokens, max_seq_len is "
                                               f"{engine.args.max_seq_len}"}, status=400)

        def remember(out_ids):
            engine.history.record(msgs, kw, engine.tok.decode(out_ids), ids, out_ids)

        return await generate(request, ids, suffix, has_history, body, chat=True, on_done=remember)

    @routes.post("/v1/completions")
    async def completions(request):
        if not engine.healthy():
            return web.json_response({"error": {"message": "not ready"}}, status=503)
        body = await request.json()
        prompt = body.get("prompt")
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], list):
            if len(prompt) != 1:
                return web.json_response({"error": "one prompt per request (no batches)"}, status=400)
            prompt = prompt[0]
        if isinstance(prompt, list):
            if not all(isinstance(x, int) and not isinstance(x, bool) for x in prompt):
                return web.json_response({"error": "prompt must be an array of integer token ids (one prompt)"},
                                         status=400)
            ids = list(prompt)
        else:
            ids = engine.tok.encode(str(prompt or ""))
        if not ids:
            return web.json_response({"error": "prompt must not be empty"}, status=400)
        if len(ids) >= engine.args.max_seq_len:
            return web.json_response({"error": f"prompt has {len(ids)} tokens, max_seq_len is "
                                               f"{engine.args.max_seq_len}"}, status=400)
        return await generate(request, ids, 0, False, body, chat=False)

    @routes.post("/reset_prefix_cache")
    async def reset(_):
        """Drop every cached prefix no request is using, and the recorded chat replies, so a
        benchmark point cannot reuse what an earlier point sent."""
        if not engine.healthy():
            return web.json_response({"error": {"message": "not ready"}}, status=503)
        n = await asyncio.get_running_loop().run_in_executor(None, engine.sched.reset_prefix_cache)
        engine.history.clear()
        return web.json_response({"status": "ok", "cleared_slots": n, "evicted": n})

    @routes.post("/v1/score")
    async def score(request):
        """Teacher-forced log-probabilities of a continuation. Two request forms:
        ``{"prompt": [ids], "continuation_start": i, "top_k": k}`` scores ``prompt[i:]`` and
        answers ``{"object": "token_scores", "scores": [{token_id, logprob, top_logprobs}]}`` (the
        reference's form, ``server.py:723-880`` there); ``{"prompt": ..., "continuation": ...}``
        (ids or text) answers ``{"logprobs": [...], "tokens": [...]}``."""
        if not engine.healthy():
            return web.json_response({"error": {"message": "not ready"}}, status=503)
        body = await request.json()
        ref_form = "continuation_start" in body
        top_k = 0
        if ref_form:
            ids = body.get("prompt")
            cs = body.get("continuation_start")
            top_k = body.get("top_k", 5)
            if not isinstance(ids, list) or not all(isinstance(x, int) and not isinstance(x, bool) for x in ids):
                return web.json_response({"error": "prompt must be a list of token ids"}, status=400)
            if not isinstance(cs, int) or isinstance(cs, bool) or not 0 < cs < len(ids):
                return web.json_response({"error": f"continuation_start must satisfy 0 < continuation_start < "
                                                   f"len(prompt) ({len(ids)}), got {cs!r}"}, status=400)
            if not isinstance(top_k, int) or isinstance(top_k, bool) or top_k < 1:
                return web.json_response({"error": "top_k must be a positive integer"}, status=400)
            pids, cids = ids[:cs], ids[cs:]
        else:
            p = body.get("prompt", [])
            c = body.get("continuation", [])
            pids = [int(x) for x in p] if isinstance(p, list) else engine.tok.encode(p)
            cids = [int(x) for x in c] if isinstance(c, list) else engine.tok.encode(c)
        ids = pids + cids

        def finish(logits):
            lp = torch.log_softmax(logits.float(), dim=-1)
            tgt = torch.tensor(cids, device=lp.device)
            picked = lp[torch.arange(len(cids), device=lp.device), tgt].tolist()
            if not ref_form:
                return picked
            vals, tops = lp.topk(min(top_k, lp.shape[-1]), dim=-1)
            return [{"token_id": t, "logprob": v,
                     "top_logprobs": [{"token_id": i, "logprob": x} for x, i in zip(vr, ir)]}
                    for t, v, vr, ir in zip(cids, picked, vals.tolist(), tops.tolist())]

        job = ScoreJob(ids, len(pids), finish)
        engine.sched.score(job)
        await asyncio.get_running_loop().run_in_executor(None, job.done.wait, 600)
        if job.error:
            return web.json_response({"error": {"message": job.error}}, status=500)
        if ref_form:
            return web.json_response({"id": f"score-{uuid.uuid4().hex}", "object": "token_scores",
                                      "model": body.get("model") or engine.model_name, "prompt_tokens": len(ids),
                                      "continuation_start": len(pids), "scores": job.result})
        return web.json_response({"logprobs": job.result, "tokens": cids})

    @routes.post("/debug/fault")
    async def fault(request):
        if not flags.get("QB_FAULT_ENDPOINT"):
            return web.json_response({"error": {"message": "fault endpoint disabled"}}, status=404)
        body = await request.json()
        from .faults import FAULTS

        name = body.get("name")
        if name not in FAULTS:
            return web.json_response({"error": {"message": f"unknown fault {name}"}}, status=400)
        value = body.get("value")
        engine.sched.control(lambda: engine.runner.set_fault(name, value))
        m = engine.runner
        while not hasattr(m, "fault") and hasattr(m, "model"):
            m = m.model
        state = {n: getattr(m, "fault", {}).get(n) for n in sorted(FAULTS)}
        return web.json_response({"fault": name, "value": value, "faults": state})

    app = web.Application(client_max_size=64 * 1024 * 1024)
    app.add_routes(routes)
    return app


def start_workers(args) -> list[subprocess.Popen]:
    procs = []
    for r in range(1, args.tp):
        cmd = [sys.executable, "-m", "qwen35_b200.serving.server", "--rank", str(r)] + [
            a for a in sys.argv[1:] if not a.startswith("--rank")]
        procs.append(subprocess.Popen(cmd, env=dict(os.environ)))
    return procs


def main(argv=None):
    args = parse(argv)
    if args.rank > 0:
        run_worker(args)
        return
    from aiohttp import web

    workers = start_workers(args)
    engine = Engine(args, workers)
    try:
        web.run_app(make_app(engine), host=args.host, port=args.port, print=None)
    finally:
        engine.shutdown()


if __name__ == "__main__":
    main()
