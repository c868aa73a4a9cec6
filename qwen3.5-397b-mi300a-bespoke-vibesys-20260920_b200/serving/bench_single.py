"""Single-request benchmark: one prompt of ``--prompt`` random token ids, prefilled in chunks of
``--chunk`` tokens, then ``--decode`` greedy tokens (CUDA-graph decode steps).

    torchrun --nproc-per-node N -m qwen35_b200.serving.bench_single [--prompt 4096] [--decode 256]

Full geometry with random-init weights at TP=N (MTP off). Times with CUDA events (max over ranks):
the prefill (time to the first token, device) and the decode steps; reports TTFT, decode ms per
token and tokens/s. A 32k-token prompt (``--prompt 32768``) exercises long prefills: chunked
prefill over the paged KV cache, and at N > 1 the sequence-parallel fused collectives.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import time

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--decode", type=int, default=256)
    ap.add_argument("--chunk", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    from ..parallel import comm as commmod
    from ..parallel.driver import command_group, pool_handshake
    from .engine import PoolSpec, build_model

    rank, world = commmod.init(timeout_s=1800)
    cuda = torch.cuda.is_available()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank))) if cuda else torch.device("cpu")
    if cuda:
        torch.cuda.set_device(dev)
    max_seq = args.prompt + args.decode + 16
    spec = PoolSpec(lanes=1, max_seq=max_seq, kv_tokens=max_seq + 64, snapshots=2)
    dtype = torch.bfloat16 if cuda else torch.float32
    model, _ = build_model(args.model, rank, world, dev, spec, dtype=dtype, seed=args.seed)
    command_group(world)
    pool_handshake(model)
    vocab = model.cfg.vocab - 16
    rng = random.Random(args.seed)
    ids = [rng.randrange(vocab) for _ in range(args.prompt)]
    per = (max_seq + model.block_size - 1) // model.block_size
    model.begin(0)
    model.attach_blocks(0, list(range(1, 1 + per)))

    def event():
        if not cuda:
            return time.perf_counter()
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def ms(a, b):
        return a.elapsed_time(b) if cuda else (b - a) * 1e3

    if world > 1:
        dist.barrier()
    if cuda:
        torch.cuda.synchronize()
    e0 = event()
    logits = None
    for s in range(0, len(ids), args.chunk):  # chunked prefill continuing the lane's state
        logits = model.prefill(0, ids[s:s + args.chunk], s)
    tok = int(model.sample_batch(logits, [0.0])[0])
    e1 = event()
    out, pos = [tok], len(ids)
    for _ in range(args.decode - 1):
        lg = model.decode([0], [tok], [pos])
        tok = int(model.sample_batch(lg, [0.0])[0])
        out.append(tok)
        pos += 1
    e2 = event()
    if cuda:
        torch.cuda.synchronize()
    t = torch.tensor([ms(e0, e1), ms(e1, e2)], device=dev if cuda else "cpu")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ttft, dec = t.tolist()
    if rank == 0:
        n = max(1, args.decode - 1)
        print(json.dumps({"bench": "single_request", "n_gpus": world, "prompt": args.prompt, "chunk": args.chunk,
                          "decode_tokens": args.decode, "ttft_ms": round(ttft, 2),
                          "decode_ms_per_token": round(dec / n, 3),
                          "decode_tok_s": round(n / (dec / 1e3), 1) if dec else None,
                          "first_tokens": out[:8]}))
    if hasattr(model, "release"):
        model.release()  # graphs hold NCCL work: drop them before the process group
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
