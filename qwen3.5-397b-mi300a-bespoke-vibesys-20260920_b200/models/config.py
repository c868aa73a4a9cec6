"""Model configuration for the Qwen3.5-MoE text path.

Parses a HuggingFace ``config.json`` (top level or its ``text_config``) into a frozen
dataclass, and provides the two geometries this framework is tested and benchmarked on:
``full_config()`` (the 397B-A17B geometry of the published checkpoint) and ``tiny_config()``
(the hidden-256 parity model).

Field meaning follows the reference's ``reference/config.json:7-113`` and its ``Cfg``
(``model.py:529-581``).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field, replace

LINEAR = "linear_attention"
FULL = "full_attention"


@dataclass(frozen=True)
class Qwen35Config:
    hidden: int = 4096
    layers: int = 60
    layer_types: tuple[str, ...] = field(default_factory=tuple)
    vocab: int = 248320
    # gated full attention
    q_heads: int = 32
    kv_heads: int = 2
    head_dim: int = 256
    rope_theta: float = 1e7
    partial_rotary: float = 0.25
    # gated DeltaNet
    dn_k_heads: int = 16
    dn_v_heads: int = 64
    dn_k_dim: int = 128
    dn_v_dim: int = 128
    conv_kernel: int = 4
    # MoE
    experts: int = 512
    top_k: int = 10
    moe_inter: int = 1024
    shared_inter: int = 1024
    # misc
    eps: float = 1e-6
    eos_token_id: int = 248044
    mtp_layers: int = 1
    max_position: int = 262144
    mtp_experts_bf16: bool = True  # the published checkpoint stores MTP experts unquantized

    def __post_init__(self) -> None:
        if not self.layer_types:
            object.__setattr__(
                self, "layer_types", tuple(FULL if (i + 1) % 4 == 0 else LINEAR for i in range(self.layers))
            )
        if len(self.layer_types) != self.layers:
            raise ValueError(f"layer_types has {len(self.layer_types)} entries for {self.layers} layers")

    # ------------------------------------------------------------------ derived sizes
    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

    @property
    def dn_key_dim(self) -> int:
        return self.dn_k_heads * self.dn_k_dim

    @property
    def dn_value_dim(self) -> int:
        return self.dn_v_heads * self.dn_v_dim

    @property
    def dn_conv_dim(self) -> int:
        return 2 * self.dn_key_dim + self.dn_value_dim

    @property
    def linear_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == LINEAR]

    @property
    def full_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == FULL]

    def to_json(self) -> str:
        d = asdict(self)
        d["layer_types"] = list(self.layer_types)
        return json.dumps(d, sort_keys=True)


def from_hf_dict(d: dict) -> Qwen35Config:
    """Build a config from a HuggingFace config dict (``text_config`` is used when present)."""
    t = d.get("text_config", d)
    rope = t.get("rope_parameters") or t.get("rope_scaling") or {}
    return Qwen35Config(
        hidden=t["hidden_size"],
        layers=t["num_hidden_layers"],
        layer_types=tuple(t.get("layer_types") or ()),
        vocab=t["vocab_size"],
        q_heads=t["num_attention_heads"],
        kv_heads=t["num_key_value_heads"],
        head_dim=t.get("head_dim", t["hidden_size"] // t["num_attention_heads"]),
        rope_theta=float(rope.get("rope_theta", t.get("rope_theta", 1e7))),
        partial_rotary=float(rope.get("partial_rotary_factor", t.get("partial_rotary_factor", 0.25))),
        dn_k_heads=t["linear_num_key_heads"],
        dn_v_heads=t["linear_num_value_heads"],
        dn_k_dim=t["linear_key_head_dim"],
        dn_v_dim=t["linear_value_head_dim"],
        conv_kernel=t["linear_conv_kernel_dim"],
        experts=t["num_experts"],
        top_k=t["num_experts_per_tok"],
        moe_inter=t["moe_intermediate_size"],
        shared_inter=t["shared_expert_intermediate_size"],
        eps=t.get("rms_norm_eps", 1e-6),
        eos_token_id=int(t.get("eos_token_id", 248044) if not isinstance(t.get("eos_token_id"), list) else t["eos_token_id"][0]),
        mtp_layers=t.get("mtp_num_hidden_layers", 0),
        max_position=t.get("max_position_embeddings", 262144),
    )


def load_config(model_dir: str) -> Qwen35Config:
    with open(os.path.join(model_dir, "config.json")) as f:
        d = json.load(f)
    if "qwen35_b200" in d:  # our own tiny-checkpoint writer stores the dataclass verbatim
        raw = dict(d["qwen35_b200"])
        raw["layer_types"] = tuple(raw["layer_types"])
        return Qwen35Config(**raw)
    return from_hf_dict(d)


def full_config(**over) -> Qwen35Config:
    """The Qwen3.5-397B-A17B geometry (``reference/config.json``)."""
    return replace(Qwen35Config(), **over)


def tiny_config(**over) -> Qwen35Config:
    """The parity model: hidden 256, vocab 4096, 8 layers ``[DN, DN, DN, attn] x 2``, 8 Q / 2 KV
    heads of dim 64, DeltaNet 4 QK / 8 V heads of dim 32, 32 experts top-4, expert width 128."""
    base = Qwen35Config(
        hidden=256,
        layers=8,
        vocab=4096,
        q_heads=8,
        kv_heads=2,
        head_dim=64,
        dn_k_heads=4,
        dn_v_heads=8,
        dn_k_dim=32,
        dn_v_dim=32,
        experts=32,
        top_k=4,
        moe_inter=128,
        shared_inter=128,
        eos_token_id=4095,
        mtp_layers=1,
        max_position=65536,
        mtp_experts_bf16=False,
    )
    return replace(base, **over)


def to_hf_text_config(cfg: Qwen35Config) -> dict:
    """The HuggingFace ``text_config`` dict describing ``cfg`` (used to build the parity oracle)."""
    return {
        "model_type": "qwen3_5_moe_text",
        "hidden_size": cfg.hidden,
        "num_hidden_layers": cfg.layers,
        "layer_types": list(cfg.layer_types),
        "vocab_size": cfg.vocab,
        "num_attention_heads": cfg.q_heads,
        "num_key_value_heads": cfg.kv_heads,
        "head_dim": cfg.head_dim,
        "rope_parameters": {
            "rope_type": "default",
            "rope_theta": cfg.rope_theta,
            "partial_rotary_factor": cfg.partial_rotary,
            "mrope_section": [11, 11, 10],
            "mrope_interleaved": True,
        },
        "linear_num_key_heads": cfg.dn_k_heads,
        "linear_num_value_heads": cfg.dn_v_heads,
        "linear_key_head_dim": cfg.dn_k_dim,
        "linear_value_head_dim": cfg.dn_v_dim,
        "linear_conv_kernel_dim": cfg.conv_kernel,
        "num_experts": cfg.experts,
        "num_experts_per_tok": cfg.top_k,
        "moe_intermediate_size": cfg.moe_inter,
        "shared_expert_intermediate_size": cfg.shared_inter,
        "rms_norm_eps": cfg.eps,
        "hidden_act": "silu",
        "attn_output_gate": True,
        "attention_bias": False,
        "tie_word_embeddings": False,
        "eos_token_id": cfg.eos_token_id,
        "mtp_num_hidden_layers": cfg.mtp_layers,
        "max_position_embeddings": cfg.max_position,
        "full_attention_interval": 4,
    }
