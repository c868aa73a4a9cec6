"""Per-rank model weights: checkpoint loading, load-time fusion, random init, and the tiny
parity checkpoint writer.

Checkpoint naming is the published one (``reference/README.md:27-83``): the prefix
``model.language_model.``, per-expert MXFP4 tensors (``experts.E.{gate,up,down}_proj.weight``
U8 codes and ``.weight_scale`` U8 e8m0), untied ``lm_head.weight`` and one ``mtp.*`` block.
Sharded reads and load-time fusions follow the reference's ``model.py:758-988``
(``load_experts``, ``load_attention``, ``load_deltanet``, ``load_moe_dense``, ``fuse_rows``):

* DeltaNet ``in_proj_qkv | in_proj_z | in_proj_b | in_proj_a`` -> one ``w_in`` (one GEMM);
* attention ``q_proj | k_proj | v_proj`` -> one ``w_qkv``;
* router ``gate`` plus ``shared_expert_gate`` -> one ``w_router`` (``E + 1`` rows);
* shared expert ``gate_proj | up_proj`` -> one ``w_sh13``;
* routed experts stacked per rank as ``w13`` (``[gate; up]``) and ``w2`` codes + scales.

RMSNorm weights are stored as fp32 ``1 + w`` (the ``(1 + w)`` form of the model), except the
DeltaNet gated norm which uses plain ``w``.
"""

from __future__ import annotations

import json
import os
from concurrent.futures import ThreadPoolExecutor

import torch

from ..parallel.plan import Plan
from ..utils import mxfp4
from ..utils.safetensors_io import Checkpoint, save_file
from .config import FULL, Qwen35Config, to_hf_text_config

PREFIX = "model.language_model."


# ============================================================================ loading
class _Rd:
    def __init__(self, ck: Checkpoint, prefix: str, device, dtype):
        self.ck, self.prefix, self.device, self.dtype = ck, prefix, device, dtype

    def has(self, name: str) -> bool:
        return self.ck.has(self.prefix + name)

    def raw(self, name: str, rows=None) -> torch.Tensor:
        return self.ck.load(self.prefix + name, rows)

    def w(self, name: str, rows=None) -> torch.Tensor:
        return self.raw(name, rows).to(self.device, self.dtype)

    def cols(self, name: str, c0: int, c1: int) -> torch.Tensor:
        return self.raw(name)[:, c0:c1].contiguous().to(self.device, self.dtype)

    def norm1p(self, name: str) -> torch.Tensor:
        return (1.0 + self.raw(name).float()).to(self.device)

    def f32(self, name: str) -> torch.Tensor:
        return self.raw(name).float().to(self.device)


def _dn_rows(cfg: Qwen35Config, p: Plan):
    """Row ranges of ``in_proj_qkv`` owned by ``p``: q heads, k heads, v heads."""
    kd, vd = cfg.dn_k_dim, cfg.dn_v_dim
    q = (p.dn_k.start * kd, p.dn_k.stop * kd)
    k = (cfg.dn_key_dim + p.dn_k.start * kd, cfg.dn_key_dim + p.dn_k.stop * kd)
    v = (2 * cfg.dn_key_dim + p.dn_v.start * vd, 2 * cfg.dn_key_dim + p.dn_v.stop * vd)
    return q, k, v


def load_deltanet(r: _Rd, cfg: Qwen35Config, p: Plan) -> dict:
    q, k, v = _dn_rows(cfg, p)
    vd = cfg.dn_v_dim
    z = (p.dn_v.start * vd, p.dn_v.stop * vd)
    vh = (p.dn_v.start, p.dn_v.stop)
    w_in = torch.cat(
        [
            r.w("linear_attn.in_proj_qkv.weight", q),
            r.w("linear_attn.in_proj_qkv.weight", k),
            r.w("linear_attn.in_proj_qkv.weight", v),
            r.w("linear_attn.in_proj_z.weight", z),
            r.w("linear_attn.in_proj_b.weight", vh),
            r.w("linear_attn.in_proj_a.weight", vh),
        ]
    )
    conv = r.raw("linear_attn.conv1d.weight")[:, 0, :]
    conv_w = torch.cat([conv[q[0]:q[1]], conv[k[0]:k[1]], conv[v[0]:v[1]]]).to(r.device, r.dtype)
    return {
        "w_in": w_in.contiguous(),
        "conv_w": conv_w.contiguous(),
        "A_log": r.f32("linear_attn.A_log")[vh[0]:vh[1]].contiguous(),
        "dt_bias": r.f32("linear_attn.dt_bias")[vh[0]:vh[1]].contiguous(),
        "norm_w": r.w("linear_attn.norm.weight"),
        "w_out": r.cols("linear_attn.out_proj.weight", z[0], z[1]),
    }


def load_attention(r: _Rd, cfg: Qwen35Config, p: Plan) -> dict:
    hd = cfg.head_dim
    qrows = (p.q.start * 2 * hd, p.q.stop * 2 * hd)
    kvrows = (p.kv.start * hd, p.kv.stop * hd)
    w_qkv = torch.cat(
        [
            r.w("self_attn.q_proj.weight", qrows),
            r.w("self_attn.k_proj.weight", kvrows),
            r.w("self_attn.v_proj.weight", kvrows),
        ]
    )
    return {
        "w_qkv": w_qkv.contiguous(),
        "q_norm": r.norm1p("self_attn.q_norm.weight"),
        "k_norm": r.norm1p("self_attn.k_norm.weight"),
        "w_o": r.cols("self_attn.o_proj.weight", p.q.start * hd, p.q.stop * hd),
    }


def fuse_router_shared(d: dict) -> dict:
    """One weight for the two projections of the MoE input: router rows (plus the shared-expert
    gate row), zero rows up to a multiple of 8, then the shared expert's gate|up rows. One GEMM
    then reads ``h`` once and launches once; ``w_router`` and ``w_sh13`` become row views of it
    (no second copy), and the shared-expert columns of its output start 16-byte aligned."""
    wr, ws = d["w_router"], d["w_sh13"]
    off = (wr.shape[0] + 7) // 8 * 8
    w = torch.zeros(off + ws.shape[0], wr.shape[1], dtype=wr.dtype, device=wr.device)
    w[: wr.shape[0]] = wr
    w[off:] = ws
    d.update(w_rsh=w, rsh_off=off, w_router=w[: wr.shape[0]], w_sh13=w[off:])
    return d


def load_moe_dense(r: _Rd, cfg: Qwen35Config, p: Plan) -> dict:
    sh = (p.shared.start, p.shared.stop)
    return fuse_router_shared({
        "w_router": torch.cat([r.w("mlp.gate.weight"), r.w("mlp.shared_expert_gate.weight")]).contiguous(),
        "w_sh13": torch.cat(
            [r.w("mlp.shared_expert.gate_proj.weight", sh), r.w("mlp.shared_expert.up_proj.weight", sh)]
        ).contiguous(),
        "w_sh2": r.cols("mlp.shared_expert.down_proj.weight", sh[0], sh[1]),
    })


def _device_experts(ex: dict) -> dict:
    """On a CUDA device with the block-scaled MoE path, re-lay the e8m0 scales once into the
    chunk layout its MMA reads (same bytes, permuted); the row-major copy is dropped."""
    from ..ops import core as ops

    if ex["w13"].is_cuda and ops.moe_impl() == "mx" and ex["w13"].shape[2] * 2 % 128 == 0 \
            and ex["w2"].shape[2] * 2 % 128 == 0:
        ops.prepare_experts(ex)
    return ex


def load_experts(r: _Rd, p: Plan, threads: int = 16) -> dict:
    """Stack this rank's experts. MXFP4 experts stay packed (codes + scales, uint8); bf16
    experts (the MTP layer of the published checkpoint) are stacked as bf16."""
    first = p.experts.start
    n = p.experts.count
    name = f"mlp.experts.{first}.gate_proj.weight"
    quant = r.ck.entries[r.prefix + name].dtype == "U8"

    def one(e):
        b = f"mlp.experts.{e}."
        if quant:
            w13 = torch.cat([r.raw(b + "gate_proj.weight"), r.raw(b + "up_proj.weight")])
            s13 = torch.cat([r.raw(b + "gate_proj.weight_scale"), r.raw(b + "up_proj.weight_scale")])
            return w13, s13, r.raw(b + "down_proj.weight"), r.raw(b + "down_proj.weight_scale")
        w13 = torch.cat([r.raw(b + "gate_proj.weight"), r.raw(b + "up_proj.weight")])
        return w13, r.raw(b + "down_proj.weight")

    with ThreadPoolExecutor(threads) as ex:
        parts = list(ex.map(one, range(first, first + n)))
    if quant:
        return _device_experts({
            "w13": torch.stack([x[0] for x in parts]).to(r.device),
            "s13": torch.stack([x[1] for x in parts]).to(r.device),
            "w2": torch.stack([x[2] for x in parts]).to(r.device),
            "s2": torch.stack([x[3] for x in parts]).to(r.device),
        })
    return {
        "w13": torch.stack([x[0] for x in parts]).to(r.device, r.dtype),
        "w2": torch.stack([x[1] for x in parts]).to(r.device, r.dtype),
    }


def load_layer(ck: Checkpoint, prefix: str, kind: str, cfg: Qwen35Config, p: Plan, device, dtype) -> dict:
    r = _Rd(ck, prefix, device, dtype)
    d = {
        "kind": kind,
        "in_norm": r.norm1p("input_layernorm.weight"),
        "post_norm": r.norm1p("post_attention_layernorm.weight"),
    }
    d.update(load_attention(r, cfg, p) if kind == FULL else load_deltanet(r, cfg, p))
    d.update(load_moe_dense(r, cfg, p))
    d["experts"] = load_experts(r, p)
    return d


def load_weights(model_dir: str, cfg: Qwen35Config, p: Plan, device, dtype, with_mtp: bool = True) -> dict:
    ck = Checkpoint(model_dir)
    top = _Rd(ck, PREFIX, device, dtype)
    head = _Rd(ck, "", device, dtype)
    w = {
        "embed": top.w("embed_tokens.weight"),
        "final_norm": top.norm1p("norm.weight"),
        "lm_head": head.w("lm_head.weight", (p.vocab.start, p.vocab.stop)),
        "layers": [
            load_layer(ck, f"{PREFIX}layers.{i}.", cfg.layer_types[i], cfg, p, device, dtype)
            for i in range(cfg.layers)
        ],
        "mtp": None,
    }
    if with_mtp and ck.has("mtp.fc.weight"):
        m = _Rd(ck, "mtp.", device, dtype)
        w["mtp"] = {
            "fc": m.w("fc.weight"),
            "pre_fc_norm_embedding": m.norm1p("pre_fc_norm_embedding.weight"),
            "pre_fc_norm_hidden": m.norm1p("pre_fc_norm_hidden.weight"),
            "norm": m.norm1p("norm.weight"),
            "layer": load_layer(ck, "mtp.layers.0.", FULL, cfg, p, device, dtype),
        }
    ck.close()
    return w


# ============================================================================ random init
def _randn(shape, gen, device, dtype, std=0.02):
    """N(0, std) in ``dtype``, drawn in fp32 pieces of at most 2^28 elements (a 1 GB temporary) so
    that multi-GB weights do not need twice their size while they are made."""
    out = torch.empty(shape, device=device, dtype=dtype)
    flat = out.view(-1)
    step = 1 << 28
    for i in range(0, flat.numel(), step):
        n = min(step, flat.numel() - i)
        flat[i:i + n] = torch.randn(n, generator=gen, device=device, dtype=torch.float32) * std
    return out


def random_layer(kind: str, cfg: Qwen35Config, p: Plan, gen, device, dtype, experts_from: dict | None,
                 mtp_bf16_experts: bool = False) -> dict:
    """One rank's shard of a random-init layer, generated directly on ``device``.

    Dense weights are N(0, 0.02) in ``dtype``. MXFP4 expert codes are uniform random nibbles with
    e8m0 scale byte 120 (value spacing 2**-7), which has the spread of N(0, 0.02) weights after
    quantisation (RMS 0.023). ``experts_from`` reuses another layer's expert storage (same
    shapes); see ``random_weights``."""
    h, hd, vd, kd = cfg.hidden, cfg.head_dim, cfg.dn_v_dim, cfg.dn_k_dim
    one = lambda n: torch.ones(n, dtype=torch.float32, device=device)  # noqa: E731
    d = {"kind": kind, "in_norm": one(h), "post_norm": one(h)}
    if kind == FULL:
        nq, nkv = p.q.count, p.kv.count
        d.update(
            w_qkv=_randn((nq * 2 * hd + 2 * nkv * hd, h), gen, device, dtype),
            q_norm=one(hd), k_norm=one(hd),
            w_o=_randn((h, nq * hd), gen, device, dtype),
        )
    else:
        nk, nv = p.dn_k.count, p.dn_v.count
        c = 2 * nk * kd + nv * vd
        d.update(
            w_in=_randn((c + nv * vd + 2 * nv, h), gen, device, dtype),
            conv_w=_randn((c, cfg.conv_kernel), gen, device, dtype, std=0.2),
            A_log=torch.log(torch.rand(nv, generator=gen, device=device) * 15 + 1),
            dt_bias=torch.ones(nv, device=device),
            norm_w=torch.ones(vd, device=device, dtype=dtype),
            w_out=_randn((h, nv * vd), gen, device, dtype),
        )
    d.update(
        w_router=_randn((cfg.experts + 1, h), gen, device, dtype),
        w_sh13=_randn((2 * p.shared.count, h), gen, device, dtype),
        w_sh2=_randn((h, p.shared.count), gen, device, dtype),
    )
    fuse_router_shared(d)
    if experts_from is not None:
        d["experts"] = experts_from
        return d
    ne, inter = p.experts.count, cfg.moe_inter
    if mtp_bf16_experts:
        d["experts"] = {
            "w13": _randn((ne, 2 * inter, h), gen, device, dtype),
            "w2": _randn((ne, h, inter), gen, device, dtype),
        }
        return d
    u8 = dict(dtype=torch.uint8, device=device)
    d["experts"] = _device_experts({
        "w13": torch.randint(0, 256, (ne, 2 * inter, h // 2), generator=gen, **u8),
        "s13": torch.full((ne, 2 * inter, h // 32), 120, **u8),
        "w2": torch.randint(0, 256, (ne, h, inter // 2), generator=gen, **u8),
        "s2": torch.full((ne, h, inter // 32), 120, **u8),
    })
    return d


def expert_bytes_per_layer(cfg: Qwen35Config, p: Plan) -> int:
    per = 3 * cfg.hidden * cfg.moe_inter
    return p.experts.count * (per // 2 + per // 32)


def random_weights(cfg: Qwen35Config, p: Plan, device, dtype, seed: int = 0, with_mtp: bool = True,
                   distinct_expert_layers: int | None = None) -> dict:
    """Random-init weights of ``cfg`` for rank ``p.rank``.

    ``distinct_expert_layers`` bounds how many layers get their own routed-expert storage;
    layer ``i >= n`` reuses layer ``i - n``'s (same shapes, same HBM traffic per layer, as each
    layer's experts are far larger than L2). It exists for one case only: the full geometry on
    one GPU, whose 205 GB of MXFP4 experts exceed one GPU's 180 GB. ``None`` = all distinct."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1000003 + p.rank)
    layers = []
    n = cfg.layers if distinct_expert_layers is None else max(1, distinct_expert_layers)
    for i, kind in enumerate(cfg.layer_types):
        src = layers[i - n]["experts"] if i >= n else None
        layers.append(random_layer(kind, cfg, p, gen, device, dtype, src))
    w = {
        "embed": _randn((cfg.vocab, cfg.hidden), gen, device, dtype),
        "final_norm": torch.ones(cfg.hidden, dtype=torch.float32, device=device),
        "lm_head": _randn((p.vocab.count, cfg.hidden), gen, device, dtype),
        "layers": layers,
        "mtp": None,
    }
    if with_mtp and cfg.mtp_layers:
        one = torch.ones(cfg.hidden, dtype=torch.float32, device=device)
        w["mtp"] = {
            "fc": _randn((cfg.hidden, 2 * cfg.hidden), gen, device, dtype),
            "pre_fc_norm_embedding": one.clone(),
            "pre_fc_norm_hidden": one.clone(),
            "norm": one.clone(),
            "layer": random_layer(FULL, cfg, p, gen, device, dtype, None, mtp_bf16_experts=cfg.mtp_experts_bf16),
        }
    return w


# ============================================================================ tiny checkpoint
def _layer_tensors(prefix: str, kind: str, cfg: Qwen35Config, gen, quant_experts: bool) -> dict:
    h = cfg.hidden
    g = lambda *s: torch.randn(*s, generator=gen) * 0.02  # noqa: E731
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    t = {
        prefix + "input_layernorm.weight": bf(g(h)),
        prefix + "post_attention_layernorm.weight": bf(g(h)),
    }
    if kind == FULL:
        hd = cfg.head_dim
        t.update({
            prefix + "self_attn.q_proj.weight": bf(g(cfg.q_heads * hd * 2, h)),
            prefix + "self_attn.k_proj.weight": bf(g(cfg.kv_heads * hd, h)),
            prefix + "self_attn.v_proj.weight": bf(g(cfg.kv_heads * hd, h)),
            prefix + "self_attn.o_proj.weight": bf(g(h, cfg.q_heads * hd)),
            prefix + "self_attn.q_norm.weight": bf(g(hd)),
            prefix + "self_attn.k_norm.weight": bf(g(hd)),
        })
    else:
        t.update({
            prefix + "linear_attn.in_proj_qkv.weight": bf(g(cfg.dn_conv_dim, h)),
            prefix + "linear_attn.in_proj_z.weight": bf(g(cfg.dn_value_dim, h)),
            prefix + "linear_attn.in_proj_b.weight": bf(g(cfg.dn_v_heads, h)),
            prefix + "linear_attn.in_proj_a.weight": bf(g(cfg.dn_v_heads, h)),
            prefix + "linear_attn.conv1d.weight": bf(g(cfg.dn_conv_dim, 1, cfg.conv_kernel)),
            prefix + "linear_attn.A_log": bf(g(cfg.dn_v_heads)),
            prefix + "linear_attn.dt_bias": bf(g(cfg.dn_v_heads)),
            prefix + "linear_attn.norm.weight": bf(g(cfg.dn_v_dim)),
            prefix + "linear_attn.out_proj.weight": bf(g(h, cfg.dn_value_dim)),
        })
    t.update({
        prefix + "mlp.gate.weight": bf(g(cfg.experts, h)),
        prefix + "mlp.shared_expert_gate.weight": bf(g(1, h)),
        prefix + "mlp.shared_expert.gate_proj.weight": bf(g(cfg.shared_inter, h)),
        prefix + "mlp.shared_expert.up_proj.weight": bf(g(cfg.shared_inter, h)),
        prefix + "mlp.shared_expert.down_proj.weight": bf(g(h, cfg.shared_inter)),
    })
    for e in range(cfg.experts):
        b = f"{prefix}mlp.experts.{e}."
        for name, shape in (("gate_proj", (cfg.moe_inter, h)), ("up_proj", (cfg.moe_inter, h)),
                            ("down_proj", (h, cfg.moe_inter))):
            w = g(*shape)
            if quant_experts:
                codes, scales = mxfp4.quantize(w)
                t[b + name + ".weight"] = codes
                t[b + name + ".weight_scale"] = scales
            else:
                t[b + name + ".weight"] = bf(w)
    return t


def write_tiny_checkpoint(path: str, cfg: Qwen35Config, seed: int = 0, shards: int = 2) -> None:
    """Write a random-init checkpoint of ``cfg`` in the published tensor naming and layout:
    every tensor N(0, 0.02) from ``seed``; routed experts MXFP4 (and the MTP experts MXFP4 or
    bf16 per ``cfg.mtp_experts_bf16``); the rest bf16; ``shards`` files, no index."""
    os.makedirs(path, exist_ok=True)
    gen = torch.Generator().manual_seed(seed)
    g = lambda *s: torch.randn(*s, generator=gen) * 0.02  # noqa: E731
    bf = lambda t: t.to(torch.bfloat16)  # noqa: E731
    tensors = {
        PREFIX + "embed_tokens.weight": bf(g(cfg.vocab, cfg.hidden)),
        PREFIX + "norm.weight": bf(g(cfg.hidden)),
        "lm_head.weight": bf(g(cfg.vocab, cfg.hidden)),
    }
    for i, kind in enumerate(cfg.layer_types):
        tensors.update(_layer_tensors(f"{PREFIX}layers.{i}.", kind, cfg, gen, True))
    if cfg.mtp_layers:
        tensors.update({
            "mtp.fc.weight": bf(g(cfg.hidden, 2 * cfg.hidden)),
            "mtp.pre_fc_norm_embedding.weight": bf(g(cfg.hidden)),
            "mtp.pre_fc_norm_hidden.weight": bf(g(cfg.hidden)),
            "mtp.norm.weight": bf(g(cfg.hidden)),
        })
        tensors.update(_layer_tensors("mtp.layers.0.", FULL, cfg, gen, not cfg.mtp_experts_bf16))
    names = sorted(tensors)
    per = (len(names) + shards - 1) // shards
    for s in range(shards):
        part = {n: tensors[n] for n in names[s * per:(s + 1) * per]}
        save_file(part, os.path.join(path, f"model-{s + 1:05d}-of-{shards:05d}.safetensors"))
    hf = {"architectures": ["Qwen3_5MoeForConditionalGeneration"], "model_type": "qwen3_5_moe",
          "text_config": to_hf_text_config(cfg), "tie_word_embeddings": False,
          "qwen35_b200": json.loads(cfg.to_json())}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)


# ============================================================================ full-size checkpoint
def _layer_specs(prefix: str, kind: str, cfg: Qwen35Config) -> list[tuple[str, str, tuple[int, ...]]]:
    """(name, kind, shape) of one decoder layer's tensors in the published layout; kind is
    ``bf16``, ``codes`` (packed e2m1, uint8) or ``scales`` (e8m0, uint8)."""
    h = cfg.hidden
    out = [(prefix + "input_layernorm.weight", "bf16", (h,)),
           (prefix + "post_attention_layernorm.weight", "bf16", (h,))]
    if kind == FULL:
        hd = cfg.head_dim
        out += [(prefix + "self_attn.q_proj.weight", "bf16", (cfg.q_heads * hd * 2, h)),
                (prefix + "self_attn.k_proj.weight", "bf16", (cfg.kv_heads * hd, h)),
                (prefix + "self_attn.v_proj.weight", "bf16", (cfg.kv_heads * hd, h)),
                (prefix + "self_attn.o_proj.weight", "bf16", (h, cfg.q_heads * hd)),
                (prefix + "self_attn.q_norm.weight", "bf16", (hd,)),
                (prefix + "self_attn.k_norm.weight", "bf16", (hd,))]
    else:
        out += [(prefix + "linear_attn.in_proj_qkv.weight", "bf16", (cfg.dn_conv_dim, h)),
                (prefix + "linear_attn.in_proj_z.weight", "bf16", (cfg.dn_value_dim, h)),
                (prefix + "linear_attn.in_proj_b.weight", "bf16", (cfg.dn_v_heads, h)),
                (prefix + "linear_attn.in_proj_a.weight", "bf16", (cfg.dn_v_heads, h)),
                (prefix + "linear_attn.conv1d.weight", "bf16", (cfg.dn_conv_dim, 1, cfg.conv_kernel)),
                (prefix + "linear_attn.A_log", "bf16", (cfg.dn_v_heads,)),
                (prefix + "linear_attn.dt_bias", "bf16", (cfg.dn_v_heads,)),
                (prefix + "linear_attn.norm.weight", "bf16", (cfg.dn_v_dim,)),
                (prefix + "linear_attn.out_proj.weight", "bf16", (h, cfg.dn_value_dim))]
    out += [(prefix + "mlp.gate.weight", "bf16", (cfg.experts, h)),
            (prefix + "mlp.shared_expert_gate.weight", "bf16", (1, h)),
            (prefix + "mlp.shared_expert.gate_proj.weight", "bf16", (cfg.shared_inter, h)),
            (prefix + "mlp.shared_expert.up_proj.weight", "bf16", (cfg.shared_inter, h)),
            (prefix + "mlp.shared_expert.down_proj.weight", "bf16", (h, cfg.shared_inter))]
    for e in range(cfg.experts):
        b = f"{prefix}mlp.experts.{e}."
        for name, (rows, cols) in (("gate_proj", (cfg.moe_inter, h)), ("up_proj", (cfg.moe_inter, h)),
                                   ("down_proj", (h, cfg.moe_inter))):
            out.append((b + name + ".weight", "codes", (rows, cols // 2)))
            out.append((b + name + ".weight_scale", "scales", (rows, cols // 32)))
    return out


def checkpoint_shards(cfg: Qwen35Config) -> list[list[tuple[str, str, tuple[int, ...]]]]:
    """Tensor specs per shard of ``write_random_checkpoint``: shard 0 holds the embedding, the
    final norm and the LM head; shard ``1 + i`` holds decoder layer ``i``."""
    h = cfg.hidden
    shards = [[(PREFIX + "embed_tokens.weight", "bf16", (cfg.vocab, h)), (PREFIX + "norm.weight", "bf16", (h,)),
               ("lm_head.weight", "bf16", (cfg.vocab, h))]]
    for i, kind in enumerate(cfg.layer_types):
        shards.append(_layer_specs(f"{PREFIX}layers.{i}.", kind, cfg))
    return shards


def write_random_checkpoint(path: str, cfg: Qwen35Config, seed: int = 0, only: list[int] | None = None,
                            device: str | torch.device = "cpu", write_config: bool = True,
                            zero_codes: bool = False) -> list[str]:
    """Write a random-init checkpoint of ``cfg`` (any size, the full geometry included) in the
    published naming and layout, one safetensors file per shard of ``checkpoint_shards``:
    bf16 tensors N(0, 0.02); routed experts as packed e2m1 codes (uniform random bytes) with
    e8m0 scales 2^-7 .. 2^-5 (the block scales an N(0, 0.02) matrix quantises to). Tensors are
    generated one at a time on ``device`` and streamed to the file, so host memory stays at one
    tensor. ``only`` restricts the call to those shard indices (ranks can split the work); the
    shard's own seed makes its bytes independent of which process writes it. ``zero_codes``
    leaves the routed experts' code bytes as file holes (zeros, no disk blocks) for a disk that
    cannot hold ~190 GB of codes; readers still read every byte. Returns the paths written."""
    import struct

    os.makedirs(path, exist_ok=True)
    shards = checkpoint_shards(cfg)
    n = len(shards)
    written = []
    dev = torch.device(device)
    for s in (range(n) if only is None else only):
        specs = shards[s]
        gen = torch.Generator(device=dev).manual_seed(seed * 100_003 + s)
        header, off = {}, 0
        for name, kind, shape in specs:
            nbytes = int(torch.Size(shape).numel()) * (2 if kind == "bf16" else 1)
            header[name] = {"dtype": "BF16" if kind == "bf16" else "U8", "shape": list(shape),
                            "data_offsets": [off, off + nbytes]}
            off += nbytes
        hb = json.dumps(header, separators=(",", ":")).encode()
        hb += b" " * ((8 - len(hb) % 8) % 8)
        fn = os.path.join(path, f"model-{s + 1:05d}-of-{n:05d}.safetensors")
        tmp = fn + ".part"
        with open(tmp, "wb") as f:
            f.write(struct.pack("<Q", len(hb)))
            f.write(hb)
            for name, kind, shape in specs:
                if kind == "bf16":
                    t = (torch.randn(*shape, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
                elif kind == "codes" and zero_codes:
                    f.seek(int(torch.Size(shape).numel()), os.SEEK_CUR)  # a hole: reads as zeros
                    continue
                elif kind == "codes":
                    t = torch.randint(0, 256, shape, generator=gen, device=dev, dtype=torch.uint8)
                else:
                    t = torch.randint(120, 123, shape, generator=gen, device=dev, dtype=torch.uint8)
                f.write(t.contiguous().view(torch.uint8).cpu().numpy().tobytes())
            f.truncate(f.tell())  # a trailing hole still counts toward the file size
        os.replace(tmp, fn)
        written.append(fn)
    if write_config:
        hf = {"architectures": ["Qwen3_5MoeForConditionalGeneration"], "model_type": "qwen3_5_moe",
              "text_config": to_hf_text_config(cfg), "tie_word_embeddings": False,
              "qwen35_b200": json.loads(cfg.to_json())}
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(hf, f, indent=1)
    return written
