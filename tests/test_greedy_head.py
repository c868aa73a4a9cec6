"""Vocabulary-parallel greedy head: the ids from gathered (max, index) pairs equal the argmax of
the gathered logits rows, ties included (lowest global index), at one rank and over two gloo
ranks; the tiny model decodes the same tokens with the head on and off."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import torch


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _logits(rows: int, vocab: int) -> torch.Tensor:
    """bf16 rows with planted ties: a maximum repeated inside one slice, across the two slices'
    boundary, and in both slices at once (the lower index must win)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(rows, vocab, generator=g).bfloat16()
    half = vocab // 2
    x[0, 5] = x[0, 9] = 9.0  # both in slice 0
    x[1, half - 1] = x[1, half] = 9.0  # last of slice 0, first of slice 1
    x[2, half + 3] = x[2, 7] = 9.0  # slice 1 listed first, slice 0 has the lower index
    x[3, half + 11] = x[3, vocab - 1] = 9.0  # both in slice 1
    return x


def _rank(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    from qwen35_b200.parallel.comm import Comm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _logits(6, 64)
        per = full.shape[1] // world
        local = full[:, rank * per:(rank + 1) * per].contiguous()
        comm = Comm(rank, world, None, torch.device("cpu"))
        ids = comm.argmax_gather(local, rank * per)
        gathered = comm.all_gather_last(local)
        q.put((rank, ids.tolist(), gathered.float().argmax(dim=-1).tolist(), torch.equal(gathered, full)))
    finally:
        dist.destroy_process_group()


def test_argmax_gather_one_rank_matches_argmax():
    from qwen35_b200.parallel.comm import Comm

    x = _logits(6, 64)
    ids = Comm().argmax_gather(x, 0)
    assert ids.tolist() == x.float().argmax(dim=-1).tolist()
    assert ids.tolist()[:4] == [5, 31, 7, 43]


def test_argmax_gather_two_gloo_ranks_matches_full_argmax():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ids, ref, same in got:
        assert same, rank
        assert ids == ref, (rank, ids, ref)
        assert ids[:4] == [5, 31, 7, 43]


def test_tiny_model_greedy_head_on_and_off_decode_alike(monkeypatch):
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan

    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    w = random_weights(cfg, p, torch.device("cpu"), torch.float32, seed=0, with_mtp=False)
    outs = []
    for on in ("1", "0"):
        monkeypatch.setenv("QB_GREEDY_HEAD", on)
        m = Model(cfg, w, p, device="cpu", dtype=torch.float32, max_batch=3, max_seq=128)
        assert m.greedy_head == (on == "1")
        ids = list(range(3, 40))
        m.begin(0)
        m.attach_blocks(0, list(range(1, 9)))
        lg = m.prefill(0, ids, 0)
        toks = [int(lg.float().argmax())]
        pos = len(ids)
        for _ in range(6):  # the overlap path: ids from the head, the step's logits slice kept
            h = m.decode_launch([0], [toks[-1]], [pos], [0], keep_rows=[0])
            toks.append(m.decode_collect(h)[0])
            kept = m.decode_kept(h)[0]
            assert kept.shape[-1] == cfg.vocab and int(kept.float().argmax()) == toks[-1]
            pos += 1
        outs.append(toks)
    assert outs[0] == outs[1]
