"""MTP speculative-decode benchmark (forced drafts).

    torchrun --nproc-per-node N -m qwen35_b200.serving.bench_mtp [--batches 1 8 32 64] [--ctx 2048]

Full geometry with random-init weights at TP=N, one MTP layer, draft depth ``k`` (3), every draft
position accepted with probability 0.7 (forced-draft mode), so the verify path is timed
independently of what random weights would predict. For each batch size: prefill ``ctx`` random
token ids per lane, then time ``rounds`` speculative rounds with CUDA events (max over ranks).
Reports per batch: mean round latency (draft + verify + commit), accepted tokens per lane per
round, accepted tok/s/user and aggregate tok/s.
"""

from __future__ import annotations

import argparse
import json
import os
import random

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--batches", type=int, nargs="*", default=[1, 8, 32, 64])
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--accept", type=float, default=0.7)
    ap.add_argument("--rounds", type=int, default=20)
    ap.add_argument("--graphs", type=int, default=1, help="replay captured rounds (CUDA; 0: eager)")
    args = ap.parse_args()
    from ..models import mtp as mtpmod
    from ..parallel import comm as commmod
    from ..parallel.driver import command_group, pool_handshake
    from .engine import PoolSpec, build_model

    rank, world = commmod.init(timeout_s=1800)
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank))) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    lanes = max(args.batches)
    spec = PoolSpec(lanes=lanes + 1, max_seq=args.ctx + 64 * (args.k + 1) + 64,  # + the graphs' pad lane
                    kv_tokens=(lanes + 1) * (args.ctx + 64 * (args.k + 1) + 64), snapshots=2)
    dtype = torch.bfloat16 if cuda else torch.float32
    model, _ = build_model(args.model, rank, world, dev, spec, dtype=dtype, with_mtp=True, graphs=False)
    command_group(world)
    pool_handshake(model)
    head = mtpmod.attach(model, k=args.k, forced_accept=args.accept)
    head.rng.seed(1234)  # identical acceptance draws on every rank
    runner = model
    if cuda and args.graphs:
        from .graphs import GraphRunner

        runner = GraphRunner(model, buckets=args.batches)
        runner.prepare_speculative()
    rng = random.Random(0)
    per = (spec.max_seq + model.block_size - 1) // model.block_size
    results = []
    for B in args.batches:
        ls = list(range(B))
        for l in ls:
            model.begin(l)
            model.attach_blocks(l, list(range(1 + l * per, 1 + (l + 1) * per)))
        ids = [[rng.randrange(150000 if args.model == "full" else 4000) for _ in range(args.ctx)] for _ in ls]
        for i in range(0, B, 8):  # prefill in groups to bound activation memory
            model.prefill_batch([(l, ids[l], 0) for l in ls[i:i + 8]])
        tok, pos = [5] * B, [args.ctx] * B
        acc0 = head.accepted
        for _ in range(2):  # warm-up rounds
            got = runner.speculative_decode(ls, tok, pos, [1 << 20] * B, [[] for _ in ls])
            pos = [p + len(g) for p, g in zip(pos, got)]
            tok = [g[-1] for g in got]
        if cuda:
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        acc0, t_ms = head.accepted, 0.0
        s = torch.cuda.Event(enable_timing=True) if cuda else None
        e = torch.cuda.Event(enable_timing=True) if cuda else None
        import time

        t0 = time.perf_counter()
        if cuda:
            s.record()
        committed = 0
        for _ in range(args.rounds):
            got = runner.speculative_decode(ls, tok, pos, [1 << 20] * B, [[] for _ in ls])
            committed += sum(len(g) for g in got)
            pos = [p + len(g) for p, g in zip(pos, got)]
            tok = [g[-1] for g in got]
        if cuda:
            e.record()
            torch.cuda.synchronize()
            t_ms = s.elapsed_time(e)
        else:
            t_ms = (time.perf_counter() - t0) * 1e3
        if world > 1:
            tt = torch.tensor([t_ms], device=dev if cuda else "cpu")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_ms = tt.item()
        round_ms = t_ms / args.rounds
        per_lane = committed / (B * args.rounds)
        results.append({"batch": B, "round_ms": round(round_ms, 3), "tokens_per_lane_per_round": round(per_lane, 3),
                        "accepted_tok_s_per_user": round(per_lane / round_ms * 1e3, 1),
                        "aggregate_tok_s": round(committed / t_ms * 1e3, 1),
                        "draft_accept_rate": round((head.accepted - acc0) / (B * args.rounds * args.k), 3)})
    if rank == 0:
        for r in results:
            print(json.dumps({"bench": "mtp_forced", "n_gpus": world, "k": args.k, "ctx": args.ctx,
                              "graphs": bool(cuda and args.graphs), **r}))
    if hasattr(runner, "release"):
        runner.release()  # graphs hold NCCL work: drop them before the process group
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
