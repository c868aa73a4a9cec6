"""Builds the HuggingFace ``Qwen3_5MoeForCausalLM`` oracle from one of our checkpoints.

The oracle is transformers' own ``qwen3_5_moe`` modeling code (the same code as the
reference's ``reference/modeling_qwen3_5_moe.py``). Routed experts are dequantized from
MXFP4 into HF's fused ``gate_up_proj`` [E, 2I, H] / ``down_proj`` [E, H, I] parameters."""

from __future__ import annotations

import torch

from qwen35_b200.models.config import load_config, to_hf_text_config
from qwen35_b200.models.weights import PREFIX
from qwen35_b200.utils import mxfp4
from qwen35_b200.utils.safetensors_io import Checkpoint


def build_hf(model_dir: str, dtype=torch.float32):
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeForCausalLM

    cfg = load_config(model_dir)
    hcfg = Qwen3_5MoeTextConfig(**{k: v for k, v in to_hf_text_config(cfg).items()
                                   if k not in ("model_type", "attn_output_gate", "full_attention_interval",
                                                "mtp_num_hidden_layers")})
    hcfg._attn_implementation = "eager"
    model = Qwen3_5MoeForCausalLM(hcfg).to(dtype).eval()
    ck = Checkpoint(model_dir)
    sd = {}
    for name in ck.names(PREFIX):
        if ".mlp.experts." in name:
            continue
        sd["model." + name[len(PREFIX):]] = ck.load(name).to(dtype)
    sd["lm_head.weight"] = ck.load("lm_head.weight").to(dtype)
    for i in range(cfg.layers):
        b = f"{PREFIX}layers.{i}.mlp.experts."
        gu, dn = [], []
        for e in range(cfg.experts):
            deq = lambda n: mxfp4.dequantize(ck.load(f"{b}{e}.{n}.weight"), ck.load(f"{b}{e}.{n}.weight_scale"),
                                             torch.float32)
            gu.append(torch.cat([deq("gate_proj"), deq("up_proj")]))
            dn.append(deq("down_proj"))
        sd[f"model.layers.{i}.mlp.experts.gate_up_proj"] = torch.stack(gu).to(dtype)
        sd[f"model.layers.{i}.mlp.experts.down_proj"] = torch.stack(dn).to(dtype)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [m for m in missing if "rotary" not in m]
    assert not missing and not unexpected, (missing, unexpected)
    return model, cfg


@torch.inference_mode()
def hf_greedy(model, ids, n: int) -> list[int]:
    x = torch.tensor([ids])
    out = model.generate(x, max_new_tokens=n, do_sample=False, min_new_tokens=n, eos_token_id=None,
                         pad_token_id=0)
    return out[0, len(ids):].tolist()
