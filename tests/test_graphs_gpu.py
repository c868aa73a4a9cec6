"""CUDA-graph decode replay agrees with eager decode on identical lane states (tiny model)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graph_decode_matches_eager():
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.graphs import GraphRunner

    dev = torch.device("cuda")
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    m = Model(cfg, random_weights(cfg, p, dev, torch.bfloat16, seed=1, with_mtp=False), p, device=dev,
              max_batch=5, max_seq=512)
    g = GraphRunner(m, buckets=(1, 2, 4))
    g.prepare()
    assert g.validated and g._b  # boot replay-vs-eager check passed, graphs stay on
    assert set(g._b) == {1, 2, 4}
    prompts = [list(range(3, 40)), list(range(50, 130))]
    for i, ids in enumerate(prompts * 2):  # lanes 0,1 (graph) and 2,3 (eager) hold the same history
        m.begin(i)
        m.attach_blocks(i, list(range(1 + 12 * i, 13 + 12 * i)))
        m.prefill(i, ids, 0)
    toks, pos = [7, 9], [len(prompts[0]), len(prompts[1])]
    for step in range(3):
        a = g.decode([0, 1], toks, pos).float().clone()
        b = m.decode([2, 3], toks, pos).float()
        torch.cuda.synchronize()
        assert torch.equal(a.argmax(-1), b.argmax(-1))
        assert (a - b).abs().max().item() < 2e-2 * b.abs().max().item() + 1e-2
        toks = a.argmax(-1).tolist()
        pos = [x + 1 for x in pos]
    assert g.replays == 3


def test_prefill_graphs_match_eager():
    """Captured single-segment prefill widths (QB_PREFILL_GRAPHS): a prompt and a continuation of
    captured lengths replayed on one lane give the logits of the eager forwards on another lane
    with the same history, and the decode steps that follow agree (KV, DeltaNet and conv state
    written through the graphs)."""
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.graphs import GraphRunner

    dev = torch.device("cuda")
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    m = Model(cfg, random_weights(cfg, p, dev, torch.bfloat16, seed=2, with_mtp=False), p, device=dev,
              max_batch=4, max_seq=512)
    g = GraphRunner(m, buckets=(1, 2))
    g.prepare()
    g.prepare_prefill([64, 128])
    assert g.prefill_validated and set(g._pb) == {64, 128}
    a, b = list(range(7, 135)), list(range(300, 364))
    for lane in (0, 1):
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + 16 * lane, 17 + 16 * lane)))
    ga = g.prefill_batch([(0, a, 0)])[0].float()
    gb = g.prefill_batch([(0, b, 128)])[0].float()
    ea = m.prefill_batch([(1, a, 0)])[0].float()
    eb = m.prefill_batch([(1, b, 128)])[0].float()
    torch.cuda.synchronize()
    assert g.prefill_replays == 2
    for x, y in ((ga, ea), (gb, eb)):
        assert torch.equal(x.argmax(-1), y.argmax(-1))
        assert (x - y).abs().max().item() < 2e-2 * y.abs().max().item() + 1e-2
    toks, pos = [int(gb.argmax())] * 2, [192, 192]
    for _ in range(3):
        lg = m.decode([0, 1], toks, pos).float()
        torch.cuda.synchronize()
        assert torch.equal(lg[0].argmax(), lg[1].argmax())
        assert (lg[0] - lg[1]).abs().max().item() < 2e-2 * lg[1].abs().max().item() + 1e-2
        toks = [int(lg[0].argmax())] * 2
        pos = [x + 1 for x in pos]
    g.release()


def test_stamps_inside_captured_graph():
    """%globaltimer stamps recorded inside a CUDA graph: segments are positive and their sum is
    the replay's device time (CUDA events around the replay)."""
    from qwen35_b200.utils.telemetry import Stamps

    dev = torch.device("cuda")
    a = torch.randn(2048, 2048, device=dev, dtype=torch.bfloat16)
    st = Stamps(dev, capacity=16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        (a @ a).sum()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st.mark("start")
        b = a @ a
        st.mark("gemm")
        for _ in range(8):
            b = b * 1.0001
        st.mark("elementwise")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        g.replay()
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    seg = dict(st.segments_ms())
    assert seg["gemm"] > 0 and seg["elementwise"] > 0
    total = st.by_tag_ms()["total"]
    assert total <= e0.elapsed_time(e1) * 1.05 + 0.01


def test_graph_attribution_tiny():
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.graphs import GraphRunner

    dev = torch.device("cuda")
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    m = Model(cfg, random_weights(cfg, p, dev, torch.bfloat16, seed=1, with_mtp=False), p, device=dev,
              max_batch=5, max_seq=512)
    g = GraphRunner(m, buckets=(1, 4))
    g.prepare()
    att = g.attribution(4, replays=3)
    assert m.stamps is None
    for k in ("moe", "allreduce", "lm_head", "total"):
        assert k in att and att[k] >= 0
    assert att["total"] > 0
    parts = sum(v for k, v in att.items() if k != "total")
    assert abs(parts - att["total"]) < 1e-6 + 1e-6 * att["total"]


@pytest.mark.parametrize("device_accept", ["1", "0"])
def test_speculative_round_graph_matches_eager(device_accept, monkeypatch):
    """Captured speculative rounds emit the same tokens as the eager rounds on identical lane
    states: the whole round as one graph with the accepted lengths computed on the device, or
    (QB_MTP_DEVICE_ACCEPT=0) draft + verify in one graph, host accept, then the commit graph."""
    monkeypatch.setenv("QB_MTP_DEVICE_ACCEPT", device_accept)
    from qwen35_b200.models import mtp as mtpmod
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan
    from qwen35_b200.serving.graphs import GraphRunner

    dev = torch.device("cuda")
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    m = Model(cfg, random_weights(cfg, p, dev, torch.bfloat16, seed=5, with_mtp=True), p, device=dev,
              max_batch=5, max_seq=512)
    head = mtpmod.attach(m, k=2)
    g = GraphRunner(m, buckets=(1, 2, 4))
    g.prepare_speculative()
    assert set(g._spec) == {1, 2, 4}
    assert all((bk.round_graph is not None) == (device_accept == "1") for bk in g._spec.values())
    prompts = [list(range(7, 60)), list(range(100, 141))]
    for i, ids in enumerate(prompts * 2):  # lanes 0,1 (graph) and 2,3 (eager) hold the same history
        m.begin(i)
        m.attach_blocks(i, list(range(1 + 12 * i, 13 + 12 * i)))
        m.prefill(i, ids, 0)
    # each side runs its own rounds; the emitted streams must agree (acceptance lengths may differ
    # where a draft flips on a near-tie, the emitted tokens are the target's greedy tokens)
    streams = {}
    for name, runner, lanes in (("graph", g, [0, 1]), ("eager", m, [2, 3])):
        toks, pos = [9, 11], [len(prompts[0]), len(prompts[1])]
        out = [[], []]
        for _ in range(4):
            got = runner.speculative_decode(lanes, toks, pos, [64, 64], [[], []])
            for i in range(2):
                out[i].extend(got[i])
            pos = [x + len(t) for x, t in zip(pos, got)]
            toks = [t[-1] for t in got]
        streams[name] = out
    torch.cuda.synchronize()
    for i in range(2):
        n = min(len(streams["graph"][i]), len(streams["eager"][i]))
        assert n >= 4 and streams["graph"][i][:n] == streams["eager"][i][:n], (i, streams)
    assert g.replays == 4 and head.rounds == 16
    g.release()
