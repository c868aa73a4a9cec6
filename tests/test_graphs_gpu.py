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
