"""The decode-graph runner without a GPU (CPU ranks, injected capture backend): every bucket's
"graph" is the step function kept with its static buffers and re-run on replay, so bucket
choice, pad-lane padding, input packing, the one-step overlap's on-device token feedback,
boot validation and its rank vote are checked on the host against eager decode of the same
lanes. The CUDA backend runs the same code in the GPU tests."""

import torch

from qwen35_b200.models.config import tiny_config
from qwen35_b200.models.qwen35 import Model
from qwen35_b200.models.weights import random_weights
from qwen35_b200.parallel.plan import plan
from qwen35_b200.serving.graphs import GraphRunner, HostGraphs


def _model(max_batch=7):
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    return Model(cfg, random_weights(cfg, p, "cpu", torch.float32, seed=3, with_mtp=False), p, device="cpu",
                 dtype=torch.float32, max_batch=max_batch, max_seq=256)


def _lanes(m, prompts, first=0):
    for i, ids in enumerate(prompts):
        lane = first + i
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + 8 * lane, 9 + 8 * lane)))
        m.prefill(lane, ids, 0)


def test_host_graph_decode_matches_eager_with_padding():
    m = _model()
    g = GraphRunner(m, buckets=(1, 2, 4), backend=HostGraphs())
    g.prepare()
    assert g.validated and set(g._b) == {1, 2, 4, 6}  # the lane count is always a bucket
    prompts = [list(range(3, 20)), list(range(40, 61)), list(range(70, 75))]
    _lanes(m, prompts, 0)  # lanes 0-2 through the runner (bucket 4, one pad row)
    _lanes(m, prompts, 3)  # lanes 3-5 eagerly, same histories
    toks, pos = [7, 9, 11], [len(p) for p in prompts]
    for _ in range(3):
        a = g.decode([0, 1, 2], toks, pos).clone()
        b = m.decode([3, 4, 5], toks, pos)
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-4)
        toks = a.argmax(-1).tolist()
        pos = [x + 1 for x in pos]
    assert g.replays == 3


def test_host_graph_overlap_feedback_matches_eager():
    """decode_launch with tokens fed back from the previous launch (-1) gives the same ids as
    eager greedy decoding with the tokens supplied by the host."""
    m = _model()
    g = GraphRunner(m, buckets=(2, 4), backend=HostGraphs())
    g.prepare()
    prompts = [list(range(5, 30)), list(range(60, 70))]
    _lanes(m, prompts, 0)
    _lanes(m, prompts, 2)
    pos = [len(p) for p in prompts]
    h = g.decode_launch([0, 1], [3, 4], pos, [0, 0], keep_rows=[1])
    ref_toks = [3, 4]
    for step in range(4):
        ref = m.decode([2, 3], ref_toks, [p + step for p in pos]).argmax(-1).tolist()
        nxt = None
        if step < 3:  # the next launch before reading this one back: both rows fed back
            nxt = g.decode_launch([0, 1], [-1, -1], [p + step + 1 for p in pos], [0, 1])
        ids = g.decode_collect(h)
        assert ids == ref, (step, ids, ref)
        if step == 0:
            assert set(g.decode_kept(h)) == {1}
        ref_toks = ids
        h = nxt


def test_host_graph_validation_failure_turns_graphs_off():
    """A replay that returns garbage fails the boot check; the runner then decodes eagerly."""
    class Broken(HostGraphs):
        def capture(self, fn, warmups=2, pool=True):
            g, out = super().capture(fn, warmups, pool)
            ids, local = out  # (greedy ids, logits slice): the slice comes back as garbage
            g.fn = lambda: (ids, torch.full_like(local, 1e4))
            return g, out

    m = _model()
    g = GraphRunner(m, buckets=(1, 2), backend=Broken())
    g.prepare()
    assert not g.validated and not g._b
    _lanes(m, [list(range(3, 12))], 0)
    out = g.decode([0], [5], [9])  # eager fallback
    assert torch.isfinite(out).all() and out.abs().max() < 1e3


def test_host_prefill_graphs_match_eager_and_keep_lane_state():
    """Captured single-segment prefill widths replay on any lane at any start: a 64-token prompt
    and a 32-token continuation through the graphs leave the lane exactly as the eager forwards
    do (logits, KV, DeltaNet and conv state: the decode steps that follow agree); other lengths
    and multi-segment batches run eagerly."""
    m = _model()
    g = GraphRunner(m, buckets=(1, 2), backend=HostGraphs())
    g.prepare()
    g.prepare_prefill([32, 64])
    assert g.prefill_validated and set(g._pb) == {32, 64}
    a, b = list(range(5, 69)), list(range(100, 132))
    for lane in (0, 1):
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + 8 * lane, 9 + 8 * lane)))
    ga = g.prefill_batch([(0, a, 0)])[0]
    gb = g.prefill_batch([(0, b, 64)])[0]
    assert g.prefill_replays == 2
    ea = m.prefill_batch([(1, a, 0)])[0]
    eb = m.prefill_batch([(1, b, 64)])[0]
    assert torch.allclose(ga, ea, atol=1e-4, rtol=1e-4) and torch.allclose(gb, eb, atol=1e-4, rtol=1e-4)
    toks, pos = [int(gb.argmax())] * 2, [96, 96]
    for _ in range(3):
        lg = m.decode([0, 1], toks, pos)
        assert torch.allclose(lg[0], lg[1], atol=1e-4, rtol=1e-4)
        toks = [int(lg[0].argmax())] * 2
        pos = [p + 1 for p in pos]
    m.begin(2)
    m.attach_blocks(2, list(range(17, 25)))
    g.prefill_batch([(2, list(range(40)), 0)])  # not a captured width: eager
    assert g.prefill_replays == 2


def test_host_prefill_graph_validation_failure_drops_them():
    class Broken(HostGraphs):
        def capture(self, fn, warmups=2, pool=True):
            g, out = super().capture(fn, warmups, pool)
            if isinstance(out, torch.Tensor):  # the prefill step: garbage logits on replay
                g.fn = lambda: torch.full_like(out, 1e4)
            return g, out

    m = _model()
    g = GraphRunner(m, buckets=(1,), backend=Broken())
    g.prepare_prefill([32])
    assert not g.prefill_validated and not g._pb
    m.begin(0)
    m.attach_blocks(0, list(range(1, 9)))
    out = g.prefill_batch([(0, list(range(32)), 0)])[0]  # eager
    assert torch.isfinite(out).all() and out.abs().max() < 1e3 and g.prefill_replays == 0


def test_host_mixed_graphs_match_eager():
    """Captured mixed steps (decode rows padded with the pad lane + one prefill segment of a
    captured width) give the eager mixed step's logits, and leave every lane's state alike: the
    decode steps that follow agree with lanes that took the eager path."""
    m = _model(max_batch=10)
    g = GraphRunner(m, buckets=(1, 2), backend=HostGraphs())
    g.prepare_mixed([(2, 32), (4, 32)])
    assert g.mixed_validated and set(g._mb) == {(2, 32), (4, 32)}
    prompts = [list(range(3, 20)), list(range(40, 61))]
    _lanes(m, prompts, 0)  # lanes 0, 1: through the runner
    _lanes(m, prompts, 3)  # lanes 3, 4: eager, same histories
    new = list(range(200, 232))
    for lane in (2, 5):  # the prefill segment's lanes
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + 8 * lane, 9 + 8 * lane)))
    toks, pos = [7, 9], [len(p) for p in prompts]
    dg, pg = g.decode_mixed([0, 1], toks, pos, [(2, new, 0)])
    de, pe = m.decode_mixed([3, 4], toks, pos, [(5, new, 0)])
    assert g.mixed_replays == 1  # 2 decode rows: the (2, 32) shape
    assert torch.allclose(dg, de, atol=1e-4, rtol=1e-4) and torch.allclose(pg[0], pe[0], atol=1e-4, rtol=1e-4)
    toks3 = dg.argmax(-1).tolist() + [int(pg[0].argmax())]
    pos3 = [p + 1 for p in pos] + [32]
    a = m.decode([0, 1, 2], toks3, pos3)
    b = m.decode([3, 4, 5], toks3, pos3)
    assert torch.allclose(a, b, atol=1e-4, rtol=1e-4)
    dg1, _ = g.decode_mixed([0], [5], [pos3[0] + 1], [(2, list(range(33)), 33)])  # width 33: eager
    assert g.mixed_replays == 1 and dg1.shape[0] == 1


def test_two_gloo_ranks_graph_runner_with_greedy_head(tiny_dir, tmp_path):
    """Two CPU ranks (TP=2 over gloo) prepare and validate decode buckets and a prefill width
    through the host capture backend (the validation vote runs over the group); the replayed
    steps give the eager steps' logits, greedy ids gathered as (max, index) pairs and the kept
    full-vocabulary row of a finishing lane."""
    import json
    import os
    import socket
    import subprocess
    import sys

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    here = os.path.dirname(os.path.abspath(__file__))
    out = str(tmp_path / "res.json")
    procs = [subprocess.Popen([sys.executable, os.path.join(here, "graphs_gloo_rank.py"), str(r), "2", tiny_dir,
                               out, str(port)]) for r in range(2)]
    assert [p.wait(timeout=600) for p in procs] == [0, 0]
    res = json.load(open(out))
    assert res["validated"] and res["prefill_validated"]
    assert res["prefill_close"] and res["vocab"] == 4096
    assert res["ids_match"] and res["kept_close"]
    assert res["replays"] == [1, 2]
