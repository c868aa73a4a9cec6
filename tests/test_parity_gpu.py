"""Greedy-token parity of the compiled GPU path on the tiny model (bf16, TP=1) against the
reference repository's own modeling code (``reference/modeling_qwen3_5_moe.py``, fp32 on the
host): 32 greedy tokens after a 130-token prompt, through the real CUDA kernels. Every
generated token must be the oracle's top-1 on our own prefix up to a bf16-sized margin, except
at most two positions per sequence where the margin may reach 0.35: on this random-weight model
the router has near-ties (two experts' logits within bf16 rounding) that bf16 and fp32 resolve
differently, and one flipped expert moves the next logits by up to ~0.3 (measured: the same one
position with either MoE kernel path and either DeltaNet path, so it is not a kernel's error). The
first 8 tokens must equal the oracle's own greedy continuation."""

import pytest
import torch

from hf_oracle import build_hf, hf_greedy
from test_tp_gloo_parity import check_teacher_forced

pytestmark = pytest.mark.gpu


def test_tiny_gpu_greedy_matches_reference_modeling(tiny_dir):
    from qwen35_b200.models.config import load_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import load_weights
    from qwen35_b200.ops._ext import ext
    from qwen35_b200.parallel.plan import plan

    dev = torch.device("cuda", 0)
    cfg = load_config(tiny_dir)
    p = plan(cfg, 0, 1)
    m = Model(cfg, load_weights(tiny_dir, cfg, p, dev, torch.bfloat16), p, device=dev, dtype=torch.bfloat16,
              max_batch=2, max_seq=512)
    oracle, _ = build_hf(tiny_dir, reference="ref")
    for ids in (list(range(10, 140)), [(i * 37) % 4000 + 20 for i in range(70)]):
        ours = m.generate(ids, 32)
        torch.cuda.synchronize()
        check_teacher_forced(oracle, ids, ours, tol=6e-2, flips=2, flip_tol=0.35)
        ref = hf_greedy(oracle, ids, 32)
        same = next((i for i, (a, b) in enumerate(zip(ours, ref)) if a != b), len(ours))
        assert same >= 8, (same, ours[:12], ref[:12])
    st = ext().status(torch.empty(1, device=dev))
    assert int(st.abs().sum()) == 0
