"""One rank of the tensor-parallel CPU parity run (tiny model, TP=4 over gloo).

Every rank loads its shard of the tiny checkpoint in fp32 and joins a gloo group; rank 0 runs
the real scheduler + session cache through ``Broadcaster`` while the other ranks run
``serve_worker``. Rank 0 drives 2 chat sessions x 3 turns (random-id user messages wrapped in
the chat template, 32 greedy tokens per turn) and writes every turn's prompt and output."""

from __future__ import annotations

import json
import os
import random
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(rank: int, world: int, model_dir: str, out_path: str, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch
    import torch.distributed as dist

    torch.set_num_threads(2)
    from qwen35_b200.models.config import load_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import load_weights
    from qwen35_b200.parallel.comm import Comm
    from qwen35_b200.parallel.driver import Broadcaster, command_group, open_channel, pool_handshake, serve_worker
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.block_pool import BlockAllocator
    from qwen35_b200.serving.chat import TokenTemplate
    from qwen35_b200.serving.scheduler import Request, Scheduler
    from qwen35_b200.serving.session_cache import SessionCache

    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = load_config(model_dir)
    p = plan(cfg, rank, world)
    w = load_weights(model_dir, cfg, p, "cpu", torch.float32)
    m = Model(cfg, w, p, Comm(rank, world), device="cpu", dtype=torch.float32, max_batch=2, max_seq=1536,
              num_blocks=200, num_snapshots=8)
    group = command_group(world)
    pool_handshake(m)
    channel = open_channel(world, rank, group, "cpu")
    if rank != 0:
        serve_worker(m, channel)
        dist.destroy_process_group()
        return
    runner = Broadcaster(m, channel)
    cache = SessionCache(BlockAllocator(m.num_blocks, m.block_size), m.block_size, m.num_snapshots)
    sched = Scheduler(runner, cache, prefill_chunk=128, token_budget=256)
    tpl = TokenTemplate.for_vocab(cfg.vocab)
    rng = random.Random(0)
    lo = min(tpl.reserved)
    msgs = {0: [], 1: []}
    log = []
    for turn in range(3):
        outs = {}
        for s in (0, 1):
            msgs[s].append(("user", [rng.randrange(lo) for _ in range(rng.randint(64, 256))]))
            prompt, suffix = tpl.render(msgs[s])
            toks = []
            outs[s] = (prompt, toks)
            sched.submit(Request(prompt, 32, lambda e, toks=toks: toks.append(e[1]) if e[0] == "tok" else None,
                                 suffix_len=suffix))
        sched.run_until_idle()
        for s in (0, 1):
            prompt, toks = outs[s]
            log.append({"session": s, "turn": turn, "prompt": prompt, "out": toks})
            msgs[s].append(("assistant", toks))
    runner.shutdown()
    with open(out_path, "w") as f:
        json.dump({"turns": log, "hits": cache.hits}, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], int(sys.argv[5]))
