"""One rank of the two-rank graph-runner check on CPU (tiny model, TP=2 over gloo, host capture
backend): the decode buckets and a captured prefill width are prepared and validated on both
ranks (the validation vote is an all-reduce over the group), then both ranks take the same steps
through the runner and through the eager model on other lanes; rank 0 reports whether the greedy
ids (gathered as (max, index) pairs) and the kept full-vocabulary rows agree."""

from __future__ import annotations

import json
import os
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
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.graphs import GraphRunner, HostGraphs

    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = load_config(model_dir)
    p = plan(cfg, rank, world)
    m = Model(cfg, load_weights(model_dir, cfg, p, "cpu", torch.float32, with_mtp=False), p, Comm(rank, world),
              device="cpu", dtype=torch.float32, max_batch=6, max_seq=256)
    g = GraphRunner(m, buckets=(1, 2), backend=HostGraphs())
    g.prepare()
    g.prepare_prefill([32])
    res = {"validated": bool(g.validated), "prefill_validated": bool(g.prefill_validated)}
    ids = list(range(10, 42))
    for lane in range(4):
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + 8 * lane, 9 + 8 * lane)))
    lg_g = [g.prefill_batch([(lane, ids, 0)])[0] for lane in (0, 1)]  # captured width 32
    lg_e = [m.prefill_batch([(lane, ids, 0)])[0] for lane in (2, 3)]
    res["prefill_close"] = all(bool(torch.allclose(a, b, atol=1e-4, rtol=1e-4)) for a, b in zip(lg_g, lg_e))
    res["vocab"] = int(lg_g[0].shape[-1])
    toks = [int(lg_g[0].argmax())] * 2
    h = g.decode_launch([0, 1], toks, [32, 32], [0, 0], keep_rows=[1])
    got = g.decode_collect(h)
    kept = g.decode_kept(h)[1]
    ref = m.decode([2, 3], toks, [32, 32])
    res["ids_match"] = got == ref.argmax(-1).tolist()
    res["kept_close"] = bool(torch.allclose(kept[0], ref[1], atol=1e-4, rtol=1e-4))
    res["replays"] = [g.replays, g.prefill_replays]
    g.release()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4], int(sys.argv[5]))
