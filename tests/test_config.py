"""The two geometries (no GPU): the full config is the published 397B-A17B text model, the tiny
one is the parity model both benchmark configurations name; a config.json in either layout
(top level or under text_config) parses to the same dataclass, and the HuggingFace form the
oracle is built from round-trips."""

import json
from dataclasses import replace

from qwen35_b200.models.config import FULL, LINEAR, from_hf_dict, full_config, load_config, tiny_config, to_hf_text_config


def test_full_geometry_is_the_published_model():
    c = full_config()
    assert (c.hidden, c.layers, c.vocab) == (4096, 60, 248320)
    assert list(c.layer_types) == ([LINEAR] * 3 + [FULL]) * 15  # 15 x (3 DeltaNet + 1 gated attention)
    assert (c.q_heads, c.kv_heads, c.head_dim, c.partial_rotary) == (32, 2, 256, 0.25)
    assert (c.dn_k_heads, c.dn_v_heads, c.dn_k_dim, c.dn_v_dim, c.conv_kernel) == (16, 64, 128, 128, 4)
    assert (c.experts, c.top_k, c.moe_inter, c.shared_inter) == (512, 10, 1024, 1024)
    assert c.mtp_layers == 1
    assert len(c.full_layers) == 15 and len(c.linear_layers) == 45


def test_tiny_geometry_is_the_parity_model():
    c = tiny_config()
    assert (c.hidden, c.layers, c.vocab) == (256, 8, 4096)
    assert list(c.layer_types) == ([LINEAR] * 3 + [FULL]) * 2
    assert (c.q_heads, c.kv_heads, c.head_dim, c.partial_rotary) == (8, 2, 64, 0.25)
    assert (c.dn_k_heads, c.dn_v_heads, c.dn_k_dim, c.dn_v_dim, c.conv_kernel) == (4, 8, 32, 32, 4)
    assert (c.experts, c.top_k, c.moe_inter) == (32, 4, 128)
    assert c.mtp_layers == 1


def test_config_json_layouts_and_hf_round_trip(tmp_path):
    # how the checkpoint stores its MTP experts is a storage fact, not a config.json field: a loaded
    # config keeps the published layout's default, and the loader reads the stored dtype anyway
    c = replace(tiny_config(), mtp_experts_bf16=full_config().mtp_experts_bf16)
    hf = to_hf_text_config(c)
    assert from_hf_dict(hf) == c
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    (tmp_path / "a" / "config.json").write_text(json.dumps(hf))
    (tmp_path / "b" / "config.json").write_text(json.dumps({"model_type": "qwen3_5_moe", "text_config": hf}))
    assert load_config(str(tmp_path / "a")) == c == load_config(str(tmp_path / "b"))
