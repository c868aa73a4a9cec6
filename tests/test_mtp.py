"""MTP speculative decoding on the tiny model (CPU): serving with speculative rounds emits
exactly the plain greedy tokens, with the real MTP drafter and with an oracle drafter whose drafts
come from the greedy trajectory with one corrupted position cycling per round (every accept
length 0..k occurs, so DeltaNet commit/rollback and the MTP catch-up are exercised). Forced-draft
mode accepts about the configured fraction."""

import random

import pytest
import torch

from qwen35_b200.models import mtp as mtpmod
from qwen35_b200.models.config import load_config
from qwen35_b200.models.qwen35 import Model
from qwen35_b200.models.weights import load_weights
from qwen35_b200.parallel.plan import plan
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Request, Scheduler
from qwen35_b200.serving.session_cache import SessionCache

K = 3


def _model(tiny_dir):
    cfg = load_config(tiny_dir)
    p = plan(cfg, 0, 1)
    return Model(cfg, load_weights(tiny_dir, cfg, p, "cpu", torch.float32), p, device="cpu", dtype=torch.float32,
                 max_batch=3, max_seq=1024, num_blocks=300, num_snapshots=8)


def _serve(m, spec, turns=2, new=18, hook=None):
    cache = SessionCache(BlockAllocator(m.num_blocks, m.block_size), m.block_size, 8)
    s = Scheduler(m, cache, prefill_chunk=64, token_budget=128, speculative=spec)
    if hook:
        hook(s)
    rng = random.Random(0)
    hist = [[rng.randrange(4000) for _ in range(rng.randint(40, 90))] for _ in range(3)]
    outs = []
    for _ in range(turns):
        res = []
        for h in hist:
            toks = []
            res.append(toks)
            s.submit(Request(list(h), new, lambda e, toks=toks: toks.append(e[1]) if e[0] == "tok" else None))
        s.run_until_idle()
        outs.append([list(r) for r in res])
        hist = [h + r + [rng.randrange(4000) for _ in range(15)] for h, r in zip(hist, res)]
    return outs


@pytest.fixture(scope="module")
def plain(tiny_dir):
    return _serve(_model(tiny_dir), False)


def test_mtp_greedy_equals_plain(tiny_dir, plain):
    m = _model(tiny_dir)
    mtpmod.attach(m, k=K)
    assert _serve(m, True) == plain


def test_oracle_drafts_exercise_every_accept_length(tiny_dir, plain):
    m = _model(tiny_dir)
    head = mtpmod.attach(m, k=K)
    trajectories = {}
    state = {"sched": None, "round": 0}
    real_draft = head.draft

    def oracle(lanes, tokens, positions):
        real_draft(lanes, tokens, positions)  # keep the MTP cache writes of a real round
        rows = []
        for lane, p in zip(lanes, positions):
            f = next(f for f in state["sched"].decoding if f.lane == lane)
            full = trajectories[tuple(f.req.prompt)]
            seq = f.req.prompt + full
            d = [seq[p + 1 + j] if p + 1 + j < len(seq) else 0 for j in range(K)]
            bad = (state["round"] + lane) % (K + 1)
            if bad < K:
                d[bad] = (d[bad] + 1) % 4000
            rows.append(d)
        state["round"] += 1
        return torch.tensor(rows, dtype=torch.int64)

    head.draft = oracle
    # greedy trajectory of each prompt (plain run, every turn)
    rng = random.Random(0)
    hist = [[rng.randrange(4000) for _ in range(rng.randint(40, 90))] for _ in range(3)]
    for turn in plain:
        for h, out in zip(hist, turn):
            trajectories[tuple(h)] = out + [0] * (K + 2)
        hist = [h + r + [rng.randrange(4000) for _ in range(15)] for h, r in zip(hist, turn)]
    got = _serve(m, True, hook=lambda s: state.__setitem__("sched", s))
    assert got == plain
    assert head.accepted > head.rounds  # more than one accepted draft per round on average


def test_forced_acceptance_rate(tiny_dir):
    m = _model(tiny_dir)
    head = mtpmod.attach(m, k=K, forced_accept=0.7)
    _serve(m, True, turns=1, new=40)
    rate = head.accepted / head.drafted
    # per-position acceptance 0.7 with early stop: E[accepted]/k = (0.7 + 0.49 + 0.343)/3 = 0.51
    assert 0.35 < rate < 0.7, rate
