"""Batching equivalence on the tiny model (CPU, fp32): one varlen forward over several segments
must give every segment what it gets alone. Packed prefill (different lanes, lengths and start
positions, a continuation among them), batched decode, a mixed decode + prefill step, scoring,
and a DeltaNet snapshot taken and restored (the session cache's resume) against the same work
done one sequence at a time on other lanes."""

import pytest
import torch

from qwen35_b200.models.config import tiny_config
from qwen35_b200.models.qwen35 import Model
from qwen35_b200.models.weights import random_weights
from qwen35_b200.parallel.plan import plan

TOL = dict(atol=2e-4, rtol=2e-4)


@pytest.fixture(scope="module")
def model():
    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    return Model(cfg, random_weights(cfg, p, "cpu", torch.float32, seed=4, with_mtp=False), p, device="cpu",
                 dtype=torch.float32, max_batch=8, max_seq=256, num_snapshots=4)


def _lane(m, lane):
    m.begin(lane)
    m.attach_blocks(lane, list(range(1 + 16 * lane, 17 + 16 * lane)))


def _prompts():
    g = torch.Generator().manual_seed(9)
    return [torch.randint(0, 4000, (n,), generator=g).tolist() for n in (37, 5, 80)]


def test_packed_prefill_and_batched_decode_equal_single_sequences(model):
    m = model
    pr = _prompts()
    for lane in range(6):
        _lane(m, lane)
    # lane 2 already holds 16 tokens: its segment is a continuation
    m.prefill_batch([(2, pr[0][:16], 0)])
    m.prefill_batch([(5, pr[0][:16], 0)])
    packed = m.prefill_batch([(0, pr[1], 0), (1, pr[2], 0), (2, pr[0][16:], 16)])
    alone = [m.prefill_batch([(3, pr[1], 0)])[0], m.prefill_batch([(4, pr[2], 0)])[0],
             m.prefill_batch([(5, pr[0][16:], 16)])[0]]
    for a, b in zip(packed, alone):
        assert torch.allclose(a, b, **TOL)
    toks = [int(x.argmax()) for x in packed]
    pos = [len(pr[1]), len(pr[2]), len(pr[0])]
    for _ in range(3):
        batch = m.decode([0, 1, 2], toks, pos)
        single = torch.cat([m.decode([lane], [t], [p]) for lane, t, p in zip((3, 4, 5), toks, pos)])
        assert torch.allclose(batch, single, **TOL)
        toks = batch.argmax(-1).tolist()
        pos = [p + 1 for p in pos]


def test_mixed_step_equals_decode_plus_prefill(model):
    m = model
    pr = _prompts()
    for lane in range(4):
        _lane(m, lane)
    first = m.prefill_batch([(0, pr[0], 0)])[0]
    m.prefill_batch([(2, pr[0], 0)])
    tok = int(first.argmax())
    dec, pre = m.decode_mixed([0], [tok], [len(pr[0])], [(1, pr[2], 0)])
    dec2 = m.decode([2], [tok], [len(pr[0])])
    pre2 = m.prefill_batch([(3, pr[2], 0)])[0]
    assert torch.allclose(dec, dec2, **TOL) and torch.allclose(pre[0], pre2, **TOL)


def test_score_rows_equal_the_prefill_logits(model):
    m = model
    ids = _prompts()[2][:24]
    _lane(m, 0)
    scored = m.score(0, ids, 10)  # rows 9 .. 22 predict ids[10:]
    assert scored.shape[0] == len(ids) - 10
    _lane(m, 1)
    full = m.forward([(1, ids, 0)], logit_rows=list(range(len(ids))))
    assert torch.allclose(scored, full[9:len(ids) - 1], **TOL)


def test_snapshot_resume_equals_the_uninterrupted_sequence(model):
    m = model
    pr = _prompts()
    head, tail = pr[2][:48], pr[2][48:]
    _lane(m, 0)
    m.prefill_batch([(0, head, 0)])
    m.save_snapshot(0, 1)  # DeltaNet conv + recurrent state at position 48
    straight = m.prefill_batch([(0, tail, 48)])[0]
    # another lane resumes: the KV blocks are shared by copying them, the state from the snapshot
    _lane(m, 1)
    for b in range(3):  # positions 0..47 live in the first three 16-token blocks
        m.copy_block(m.tables[1][b], m.tables[0][b], 16)
    m.load_snapshot(1, 1)
    resumed = m.prefill_batch([(1, tail, 48)])[0]
    assert torch.allclose(straight, resumed, **TOL)
