"""Builds the ``Qwen3_5MoeForCausalLM`` oracle from one of our checkpoints.

Two sources of the modeling code: ``reference="ref"`` loads the reference repository's own
``reference/modeling_qwen3_5_moe.py`` (from the plain copy of the reference tree in
``baseline/_ref``; the test skips when that copy is absent), the oracle its parity tests and its
pins were made with; ``reference="hf"`` uses the installed transformers' ``qwen3_5_moe`` code.
The reference file was written against a slightly different transformers release: it is
loaded as a module of transformers' ``qwen3_5_moe`` package, and the one helper it imports
that this release lacks are supplied for its vision parts only (``accepts_precomputed_kwargs``,
a decorator on its vision methods, as a pass-through; the ``vision_utils`` helpers of its vision
tower as functions that raise), so its text model runs as written. Routed experts are dequantized from MXFP4 into the
fused ``gate_up_proj`` [E, 2I, H] / ``down_proj`` [E, H, I] parameters."""

from __future__ import annotations

import importlib.util
import os
import sys

import pytest
import torch

from qwen35_b200.models.config import load_config, to_hf_text_config
from qwen35_b200.models.weights import PREFIX
from qwen35_b200.utils import mxfp4
from qwen35_b200.utils.safetensors_io import Checkpoint


REF_MODELING = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref",
                            "reference", "modeling_qwen3_5_moe.py")


def reference_modeling():
    """The reference repository's modeling module (skips the calling test when absent)."""
    name = "transformers.models.qwen3_5_moe.modeling_qwen3_5_moe_reference"
    if name in sys.modules:
        return sys.modules[name]
    if not os.path.exists(REF_MODELING):
        pytest.skip("the reference tree is not present in baseline/_ref")
    import transformers.models.qwen3_5_moe  # noqa: F401  (the package its relative imports resolve in)
    import transformers.utils.generic as generic

    if not hasattr(generic, "accepts_precomputed_kwargs"):
        generic.accepts_precomputed_kwargs = lambda **kw: (lambda f: f)
    if importlib.util.find_spec("transformers.vision_utils") is None:  # vision-tower helpers only
        import types

        vu = types.ModuleType("transformers.vision_utils")

        def _vision_only(*a, **k):
            raise NotImplementedError("vision tower helper (not used by the text model)")

        for n in ("get_vision_bilinear_indices_and_weights", "get_vision_cu_seqlens", "get_vision_position_ids"):
            setattr(vu, n, _vision_only)
        sys.modules["transformers.vision_utils"] = vu
    spec = importlib.util.spec_from_file_location(name, REF_MODELING)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _torch_paths_only(mod) -> None:
    """The oracle runs on host tensors: drop the modeling module's optional GPU kernels (the
    flash-linear-attention and causal-conv1d packages, which it picks whenever they import, as
    they do on a GPU box), so its own PyTorch implementations run."""
    for n in ("causal_conv1d_fn", "causal_conv1d_update", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule",
              "FusedRMSNormGated"):
        if hasattr(mod, n):
            setattr(mod, n, None)
    if hasattr(mod, "is_fast_path_available"):
        mod.is_fast_path_available = False


def build_hf(model_dir: str, dtype=torch.float32, reference: str = "hf"):
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig

    if reference == "ref":
        mod = reference_modeling()
    else:
        import transformers.models.qwen3_5_moe.modeling_qwen3_5_moe as mod
    _torch_paths_only(mod)
    Qwen3_5MoeForCausalLM = mod.Qwen3_5MoeForCausalLM

    cfg = load_config(model_dir)
    hcfg = Qwen3_5MoeTextConfig(**{k: v for k, v in to_hf_text_config(cfg).items()
                                   if k not in ("model_type", "attn_output_gate", "full_attention_interval",
                                                "mtp_num_hidden_layers")})
    hcfg._attn_implementation = "eager"
    hcfg._experts_implementation = "eager"  # the plain loop over experts (no GPU kernels on host tensors)
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
