"""Reference arm of ``bench.py``: the reference engine, unmodified, on the same workload.

``python bench.py --impl reference --gpus N`` (under torchrun for N > 1) runs the reference's
own stock serving path from the plain copy of its tree in ``baseline/_ref``: per rank
``server.build_model`` (process group, this rank's shards, its GEMM tuning) and
``server.build_runner`` (its captured decode graphs, as ``--enable-graph-capture`` gives), then on
rank 0 the same sequence ``server.Engine`` runs (``tp_driver.Broadcaster``, ``warmup``,
``pool_handshake``, ``session_cache.SessionCache``, ``scheduler.Scheduler``) and on the other
ranks ``tp_driver.serve_worker``. Every ``SEED_*`` flag keeps its default except
``SEED_BLAS_TUNE=0``: the reference's boot-time cuBLAS solution search calls
``torch.cuda.tunable.write_file``, which this PyTorch release does not have. The closed-loop client
is the same token-id generator as our arm (256 sessions x 6 turns, C32, seed 0), submitting the
reference's own ``scheduler.Request`` objects through ``Scheduler.submit`` and stepping its
``Scheduler.step``. Nothing of this repository's model, kernels or engine is imported on this path
(the workload generator is loaded by file path; no package import, no extension).

Weights: random init of the full geometry written once per box in the published checkpoint layout
(``models.weights.write_random_checkpoint``: one safetensors file per decoder layer, MXFP4
experts as packed e2m1 + e8m0 scales), every rank writing its share of the shards from its GPU;
later runs on the same box reuse the files. The reference then reads them through its own loader.

Timing is the same as our arm's: one CUDA event before and one after every scheduler step on rank
0; a turn's device TTFT is the sum of the step intervals from its admission to its first token;
the loop window is bracketed by a barrier + synchronize on every rank, max over ranks.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import shutil
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_DIR = os.path.join(HERE, "_ref")
PKG_DIR = os.path.join(ROOT, "qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200")


def _say(obj) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(obj), flush=True)


def unavailable(reason: str) -> None:
    _say({"impl": "reference", "unavailable": reason})


def _by_path(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _ckpt_dir(args, need_bytes: int, dense_bytes: int) -> tuple[str, bool]:
    """Where the random checkpoint lives on this box, and whether its expert codes must be file
    holes: ``QB_REF_CKPT_DIR`` if set, else the first of /tmp, the repository's parent and
    /dev/shm with room for all of it (random codes), else the first with room for everything but
    the codes (zero codes as holes)."""
    env = os.environ.get("QB_REF_CKPT_DIR")
    if env:
        return env, False
    bases = ("/tmp", os.path.dirname(ROOT), "/dev/shm")
    for zero in (False, True):
        name = f"qb_ref_ckpt_{args.model}_s{args.seed}" + ("_zc" if zero else "")
        need = dense_bytes if zero else need_bytes
        for base in bases:
            try:
                have = os.path.exists(os.path.join(base, name))
                free = shutil.disk_usage(base).free
            except OSError:
                continue
            if have or free > need * 1.1 + 8e9:
                return os.path.join(base, name), zero
    raise RuntimeError(f"no filesystem has {dense_bytes / 1e9:.0f} GB free for the random checkpoint")


def prepare_checkpoint(args, rank: int, world: int, device, timeout_s: float = 1200.0) -> str:
    """Write (or reuse) the random-init checkpoint; every rank writes shards ``i % world == rank``
    and then waits until all shard files exist."""
    import torch

    sys.path.insert(0, ROOT)
    from qwen35_b200.models import weights as wmod  # checkpoint writer only (torch + host code)
    from qwen35_b200.models.config import full_config, tiny_config

    cfg = full_config() if args.model == "full" else tiny_config()
    cfg = type(cfg)(**{**cfg.__dict__, "mtp_layers": 0})  # MTP is off in this configuration
    shards = wmod.checkpoint_shards(cfg)
    sizes, dense = [], 0
    for specs in shards:
        sizes.append(sum(int(torch.Size(s).numel()) * (2 if k == "bf16" else 1) for _, k, s in specs))
        dense += sum(int(torch.Size(s).numel()) * (2 if k == "bf16" else 1) for _, k, s in specs if k != "codes")
    path, zero = _ckpt_dir(args, sum(sizes), dense)
    n = len(shards)
    files = [os.path.join(path, f"model-{i + 1:05d}-of-{n:05d}.safetensors") for i in range(n)]
    mine = [i for i in range(n) if i % world == rank and not os.path.exists(files[i])]
    t0 = time.perf_counter()
    if mine:
        wmod.write_random_checkpoint(path, cfg, seed=args.seed, only=mine, device=device,
                                     write_config=(rank == 0), zero_codes=zero)
    elif rank == 0 and not os.path.exists(os.path.join(path, "config.json")):
        wmod.write_random_checkpoint(path, cfg, seed=args.seed, only=[], device=device, write_config=True)
    while not (all(os.path.exists(f) for f in files) and os.path.exists(os.path.join(path, "config.json"))):
        if time.perf_counter() - t0 > timeout_s:
            raise RuntimeError("timed out waiting for the other ranks' checkpoint shards")
        time.sleep(0.5)
    if rank == 0:
        print(f"[reference] checkpoint {path}: {sum(sizes) / 1e9:.1f} GB in {n} shards"
              f"{' (expert codes as zero-filled holes: no room for random codes)' if zero else ''}, "
              f"{time.perf_counter() - t0:.0f}s", file=sys.stderr, flush=True)
    args.ref_zero_codes = zero
    return path


def main(args, report) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if not os.path.exists(os.path.join(REF_DIR, "server.py")):
        unavailable("the reference tree is not present in baseline/_ref (copy it there; it has no "
                    "setup.py/pyproject.toml for pip)")
        return
    import torch

    on_gpu = torch.cuda.is_available()
    if not on_gpu and args.model == "full":
        unavailable("no CUDA device: the full geometry is timed on GPUs only")
        return
    if args.model == "full" and world == 1:
        unavailable("the full geometry keeps 205 GB of MXFP4 experts resident, more than one 180 GB "
                    "B200 holds; the reference has no way to share expert storage between layers")
        return
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if on_gpu:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local) if on_gpu else torch.device("cpu")
    t_boot = time.perf_counter()
    ckpt = prepare_checkpoint(args, rank, world, dev)
    wl = _by_path("qb_bench_workload", os.path.join(PKG_DIR, "serving", "workload.py"))

    # The reference's boot GEMM search (blas_tune, TunableOp) ends in torch.cuda.tunable.write_file,
    # which this PyTorch release no longer has; its own switch SEED_BLAS_TUNE=0 skips the search
    # (cuBLAS keeps its default heuristic), the one flag this arm sets.
    os.environ.setdefault("SEED_BLAS_TUNE", "0")
    sys.path.insert(0, REF_DIR)
    import server as ref_server  # the reference's own modules from here on
    import tp_driver
    from scheduler import OVERLAP_SCHED, Request, Scheduler
    from session_cache import SessionCache

    import torch.distributed as dist

    a = argparse.Namespace(model_path=ckpt, dtype="bfloat16", tp=world, rank=rank,
                           tp_port=int(os.environ.get("MASTER_PORT", "29500")), max_seq_len=args.max_seq,
                           max_batch=args.concurrency, enable_graph_capture=True,
                           devices=f"cuda:{local}" if on_gpu else "cpu")
    model = ref_server.build_model(a, rank)
    runner = ref_server.build_runner(a, model)
    chan = tp_driver.command_channel(model.tp.device, OVERLAP_SCHED) if world > 1 else None

    def stamp():
        """A point on the device timeline (CUDA event on the current stream; host clock on CPU)."""
        if not on_gpu:
            return time.perf_counter()
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def ms(a, b) -> float:
        return (b - a) * 1e3 if isinstance(a, float) else a.elapsed_time(b)

    def mark():
        if on_gpu:
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return stamp()

    if rank != 0:
        tp_driver.serve_worker(runner, chan.recv)  # warm-up, until rank 0's first STOP
        ev0 = mark()
        tp_driver.serve_worker(runner, chan.recv)  # the timed loop, until the second STOP
        ev1 = mark()
        gathered = [None] * world
        dist.all_gather_object(gathered, ms(ev0, ev1))
        dist.destroy_process_group()
        return

    r = tp_driver.Broadcaster(runner, chan.send) if world > 1 else runner
    r.warmup()
    if world > 1:
        r.pool_handshake()
    else:
        tp_driver.pool_handshake(model)
    cache = SessionCache(model.block_allocator, model.block_size, model.num_snapshots)
    sched = Scheduler(r, cache)
    boot_s = time.perf_counter() - t_boot

    def make_request(prompt, max_new, emit, has_history):
        return Request(prompt, max_new, 0.0, frozenset(), emit, has_history=has_history)

    vocab = min(151000, model.cfg.vocab - 16)
    step_no = [0]

    # ---- warm-up: the same side workload as our arm, drained, then the cache emptied
    t0 = time.perf_counter()
    wspec = wl.ChatSpec(sessions=min(4, args.concurrency), concurrency=min(4, args.concurrency), turns=2,
                        seed=args.seed + 7919, vocab=vocab, first_len=(256, 1024), user_len=(64, 256),
                        gen_len=(24, 48))
    wloop = wl.ClosedLoop(sched, wspec, step_index=lambda: step_no[0], make_request=make_request)
    wloop.start()
    n_warm = 0
    while n_warm < max(args.warmup, 3) or wloop.active:
        sched.step()
        step_no[0] += 1
        wloop.pump()
        n_warm += 1
    sched.reset_prefix_cache()
    warm_s = time.perf_counter() - t0
    print(f"[reference] warm-up: {n_warm} steps in {warm_s:.1f}s", file=sys.stderr, flush=True)

    # ---- the timed closed loop
    spec = wl.ChatSpec(sessions=args.sessions, concurrency=args.concurrency, turns=args.turns, seed=args.seed,
                       vocab=vocab, first_len=tuple(args.first_len), user_len=tuple(args.user_len),
                       gen_len=tuple(args.gen_len))
    if world > 1:
        r.stop()  # workers leave the warm-up serve loop and meet rank 0 at the barrier
    step_no[0] = 0
    loop = wl.ClosedLoop(sched, spec, step_index=lambda: step_no[0], make_request=make_request)
    sys.path.insert(0, ROOT)
    from bench import ClockSampler

    cvd = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = [int(x) for x in cvd.split(",") if x.strip().isdigit()] if cvd else list(range(8))
    clocks = ClockSampler(phys[:world] if phys else list(range(world)))
    clocks.start()
    ev_start = mark()
    t_host0 = time.perf_counter()
    brackets = []
    loop.start()
    last_log = t_host0
    from bench import loop_seconds

    limit_s = loop_seconds(args)
    while loop.active and time.perf_counter() - t_host0 < limit_s:
        s = stamp()
        sched.step()
        brackets.append((s, stamp()))
        step_no[0] += 1
        loop.pump()
        if time.perf_counter() - last_log > 30:
            last_log = time.perf_counter()
            done = sum(1 for x in loop.records if x.end_step >= 0)
            print(f"[reference] {time.perf_counter() - t_host0:.0f}s step {step_no[0]}: {done} turns done",
                  file=sys.stderr, flush=True)
    if world > 1:
        r.stop()
    ev_end = mark()
    t_host1 = time.perf_counter()
    clk = clocks.stop()
    window_ms = ms(ev_start, ev_end)
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, window_ms)
        window_ms = max(gathered)
    step_ms = [ms(s, e) for s, e in brackets]
    res = report(args, impl="reference", world=world, window_ms=window_ms, host_s=t_host1 - t_host0,
                 records=loop.records, step_ms=step_ms, kinds_summary=None, clocks=clk, h2d=0, d2h=0,
                 launches=0, sched_steps=step_no[0], boot_s=boot_s, warm_s=warm_s,
                 cfg_desc=(f"Qwen3.5-397B-A17B geometry ({len(model.layers)} layers, MXFP4 experts), reference "
                           f"engine (stock SEED_* defaults, graph capture on)" if args.model == "full"
                           else "tiny parity model, reference engine"),
                 expert_storage="all layers distinct", t_end=t_host1,
                 extra={"reference_tree": "baseline/_ref (plain copy of the reference)", "checkpoint": ckpt,
                        "checkpoint_expert_codes": "zeros (file holes; the box's disk cannot hold the random "
                        "codes; every byte is still read and multiplied)" if getattr(args, "ref_zero_codes", False)
                        else "random"})
    res["e2e"]["h2d_bytes_per_step"] = None  # the reference's copies are not counted here
    res["e2e"]["d2h_bytes_per_step"] = None
    print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()
