"""Plain PyTorch statements of every op, with the rounding points of the HuggingFace modeling
code (transformers ``models/qwen3_5_moe/modeling_qwen3_5_moe.py``; reference copy
``reference/modeling_qwen3_5_moe.py``).

These functions are the CPU execution path (hermetic tests, gloo tensor parallelism) and the
fp32 oracle every CUDA kernel in ``csrc/`` is tested against. They are never called on CUDA
tensors by the model runtime: ``ops.core`` routes CUDA tensors to the compiled extension.

Spec line references (reference copy of the HF file):
* RMSNorm ``x * (1 + w)`` ``:817-835``; gated RMSNorm ``w * norm(x) * silu(z)`` ``:185-200``
* gated DeltaNet ``:369-558``; recurrent rule ``:325-366``; causal conv update ``:220-238``
* gated attention with partial RoPE ``:568-718``
* router softmax/top-k ``:794-806``; experts ``:755-791``; sparse MoE block ``:809-815``
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..utils import mxfp4


# ----------------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w1p: torch.Tensor, eps: float) -> torch.Tensor:
    """``norm(x) * w1p`` in fp32, rounded once to ``x.dtype``; ``w1p`` is ``1 + w`` (fp32)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (y * w1p.float()).to(x.dtype)


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w1p: torch.Tensor, eps: float):
    """``residual + x`` (rounded to the residual dtype, like a bf16 add), then RMSNorm of it.
    Returns ``(new_residual, normed)``."""
    r = (residual.float() + x.float()).to(residual.dtype)
    return r, rmsnorm(r, w1p, eps)


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """DeltaNet output norm over the last dim: ``(w * norm(x).to(dtype)) * silu(z)``."""
    dt = x.dtype
    xf = x.float()
    y = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(dt)
    y = (w.to(dt) * y)
    return (y.float() * F.silu(z.float())).to(dt)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


# ----------------------------------------------------------------------------- dense
def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` with fp32 accumulation, rounded to ``x.dtype``."""
    if x.dtype in (torch.bfloat16, torch.float16) and x.device.type == "cpu":
        return (x.float() @ w.float().t()).to(x.dtype)
    return F.linear(x, w)


# ----------------------------------------------------------------------------- rope
def rope_cos_sin(positions: torch.Tensor, rot: int, theta: float, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.float32, device=positions.device) / rot))
    f = positions.float()[:, None] * inv[None, :]
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_partial_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x``: [T, heads, hd]; rotate the first ``cos.shape[-1]`` dims (rotate-half form)."""
    rot = cos.shape[-1]
    xr, xp = x[..., :rot], x[..., rot:]
    half = rot // 2
    rh = torch.cat([-xr[..., half:], xr[..., :half]], dim=-1)
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([xr * c + rh * s, xp], dim=-1)


# ----------------------------------------------------------------------------- attention
def attention_prefix(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_start: int,
                     causal: bool = True) -> torch.Tensor:
    """Causal GQA attention of ``q`` [Tq, Hq, D] at positions ``q_start..`` over ``k``/``v``
    [Tk, Hkv, D] at positions ``0..Tk-1`` (``Tk == q_start + Tq``). Softmax in fp32; the
    probabilities are rounded to the input dtype before the value product (HF eager path)."""
    tq, hq, d = q.shape
    tk, hkv, _ = k.shape
    rep = hq // hkv
    kk = k.repeat_interleave(rep, dim=1)
    vv = v.repeat_interleave(rep, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk.float()) / math.sqrt(d)
    qpos = torch.arange(q_start, q_start + tq, device=q.device)[:, None]
    kpos = torch.arange(tk, device=q.device)[None, :]
    if causal:  # (False: every key of the context visible, a calibration fault)
        s = s.masked_fill((kpos > qpos)[None], float("-inf"))
    p = torch.softmax(s, dim=-1).to(q.dtype)
    return torch.einsum("hqk,khd->qhd", p.float(), vv.float()).to(q.dtype)


# ----------------------------------------------------------------------------- deltanet
def causal_conv(x_seg: torch.Tensor, state: torch.Tensor, w: torch.Tensor):
    """Depthwise causal conv + SiLU for one sequence segment.

    ``x_seg`` [T, C]; ``state`` [C, K-1] (the previous K-1 inputs, oldest first); ``w`` [C, K].
    Returns (out [T, C], new_state [C, K-1])."""
    kk = w.shape[-1]
    ext = torch.cat([state.to(x_seg.dtype), x_seg.t()], dim=-1)  # [C, K-1+T]
    out = F.conv1d(ext.float()[None], w.float()[:, None, :], groups=w.shape[0])[0]  # [C, T]
    out = F.silu(out).to(x_seg.dtype).t()
    return out, ext[:, -(kk - 1):].clone()


def gated_delta_rule(q, k, v, g, beta, state):
    """Recurrent gated delta rule for one segment (fp32).

    ``q``,``k`` [T, H, dk] (already l2-normalised and repeated to value heads; ``q`` scaled by
    ``dk**-0.5``), ``v`` [T, H, dv], ``g`` (log decay) and ``beta`` [T, H], ``state``
    [H, dk, dv] fp32. Returns (out [T, H, dv] fp32, final state)."""
    s = state.float().clone()
    outs = []
    for t in range(q.shape[0]):
        s = s * torch.exp(g[t].float())[:, None, None]
        kv = torch.einsum("hkv,hk->hv", s, k[t].float())
        delta = (v[t].float() - kv) * beta[t].float()[:, None]
        s = s + k[t].float()[:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hkv,hk->hv", s, q[t].float()))
    return torch.stack(outs, 0), s


def deltanet_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """``beta = sigmoid(b)`` (in the activation dtype, as HF computes it), ``g = -exp(A_log) *
    softplus(a + dt_bias)`` in fp32."""
    beta = torch.sigmoid(b).float()
    g = -torch.exp(a_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g, beta


# ----------------------------------------------------------------------------- moe
def router_topk(logits: torch.Tensor, k: int):
    """Softmax over experts in fp32, top-k, renormalise. Returns (weights [T,k] in the logits
    dtype, indices [T,k] int64)."""
    p = torch.softmax(logits.float(), dim=-1)
    v, i = torch.topk(p, k, dim=-1)
    v = v / v.sum(-1, keepdim=True)
    return v.to(logits.dtype), i


def expert_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """One SwiGLU expert: ``w2 @ (silu(w1 x) * (w3 x))``; ``w13`` is ``[gate; up]`` rows."""
    gu = linear(x, w13)
    inter = gu.shape[-1] // 2
    h = (F.silu(gu[:, :inter].float()) * gu[:, inter:].float()).to(x.dtype)
    return linear(h, w2)


def routed_experts(h, topw, topi, experts: dict, first: int, count: int) -> torch.Tensor:
    """Sum over the top-k assignments that fall in local experts ``[first, first+count)``.

    ``experts`` holds either MXFP4 tensors (``w13``/``s13``/``w2``/``s2`` packed) or bf16
    (``w13``/``w2``) stacked over the local experts. Accumulated in fp32, rounded once."""
    out = torch.zeros(h.shape[0], h.shape[1], dtype=torch.float32, device=h.device)
    mxfp4_w = "s13" in experts
    for e in range(count):
        ge = first + e
        tok, slot = torch.where(topi == ge)
        if tok.numel() == 0:
            continue
        if mxfp4_w:
            w13 = mxfp4.dequantize(experts["w13"][e], experts["s13"][e], h.dtype)
            w2 = mxfp4.dequantize(experts["w2"][e], experts["s2"][e], h.dtype)
        else:
            w13, w2 = experts["w13"][e], experts["w2"][e]
        y = expert_mlp(h[tok], w13, w2)
        out.index_add_(0, tok, y.float() * topw[tok, slot].float()[:, None])
    return out.to(h.dtype)
