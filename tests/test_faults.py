"""Accuracy-gate calibration faults on the tiny model (CPU)."""

import pytest
import torch


@pytest.mark.parametrize("fault", [{"flip_causal_mask": True, "flip_causal_mask_layer": 0},
                                   {"fp8_kv_no_scale": True}])
def test_attention_calibration_faults_change_logits(fault):
    """The KV-truncation and causal-flip faults change a tiny prefill's logits; cleared, the
    model gives the clean logits again."""
    from qwen35_b200.serving.engine import PoolSpec, build_model

    m, _ = build_model("tiny", 0, 1, torch.device("cpu"), PoolSpec(lanes=2, max_seq=64, kv_tokens=128),
                       dtype=torch.float32, graphs=False)
    ids = list(range(200, 240))

    def run():
        m.begin(0)
        m.attach_blocks(0, [1, 2, 3])
        return m.forward([(0, ids, 0)]).clone()

    clean = run()
    m.fault.update(fault)
    hurt = run()
    m.fault.clear()
    assert not torch.allclose(clean, hurt, atol=1e-4)
    assert torch.allclose(run(), clean, atol=1e-5)
