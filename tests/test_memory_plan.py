"""Memory plan of the full geometry on 180 GB B200s (no GPU): with the benchmark's pools (33
lanes with the pad lane, 16384-token sequences, the KV capacity bench.py asks for) every layer's
experts have their own storage from 2 GPUs on, and one GPU holds the first 34 layers' experts
(205 GB of MXFP4 experts exceed one GPU; the other layers reuse that storage)."""

import pytest

from qwen35_b200.models.config import full_config
from qwen35_b200.models.weights import expert_bytes_per_layer
from qwen35_b200.parallel.plan import plan
from qwen35_b200.serving.engine import PoolSpec, pool_bytes

B200_BYTES = 183_359 * 2**20  # nvidia-smi's memory total
RESERVE = 14e9  # build_model's default headroom for activations, graphs and scratch


def _distinct_layers(world: int) -> int:
    cfg = full_config()
    p = plan(cfg, 0, world)
    spec = PoolSpec(lanes=33, max_seq=16384, kv_tokens=min(32 * 16384, 480_000 * world))
    kv, state, _ = pool_bytes(cfg, p, spec)
    dense = 20e9 / world + 4e9
    budget = B200_BYTES - dense - kv - state - RESERVE
    return max(1, min(cfg.layers, int(budget // expert_bytes_per_layer(cfg, p))))


def test_expert_storage_at_each_gpu_count():
    cfg = full_config()
    total = cfg.layers * expert_bytes_per_layer(cfg, plan(cfg, 0, 1))
    assert 200e9 < total < 210e9  # ~205 GB of packed codes and scales
    assert _distinct_layers(1) == 34
    for world in (2, 4, 8):
        assert _distinct_layers(world) == cfg.layers, world


@pytest.mark.parametrize("world", [1, 8])
def test_pools_are_a_small_share(world):
    cfg = full_config()
    kv, state, blocks = pool_bytes(cfg, plan(cfg, 0, world), PoolSpec(lanes=33, max_seq=16384,
                                                                       kv_tokens=min(32 * 16384, 480_000 * world)))
    assert kv + state < 0.2 * B200_BYTES
    assert blocks * 16 >= min(32 * 16384, 480_000 * world)
