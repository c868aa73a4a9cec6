"""MXFP4 (OCP Microscaling, e2m1 elements with one e8m0 scale per 32) codec in PyTorch.

Checkpoint layout (reference ``reference/README.md:27-83``, ``mxfp4.py:1-51``): a ``[N, K]``
weight is stored as U8 ``[N, K/2]`` (two e2m1 codes per byte, the LOW nibble holds the EVEN
element along K) plus U8 ``[N, K/32]`` e8m0 scales (value ``2**(byte - 127)``). An e2m1 code is
``s e1 e0 m``: magnitudes ``0, .5, 1, 1.5, 2, 3, 4, 6`` and bit 3 is the sign.

``quantize`` follows the OCP MX v1.0 recipe: the block's shared exponent is
``floor(log2(amax)) - 2`` (2 is e2m1's largest exponent), elements are rounded to the nearest
representable value (ties to even) and saturated to +-6.
"""

from __future__ import annotations

import torch

E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
BLOCK = 32


def e2m1_lut(dtype=torch.float32, device=None) -> torch.Tensor:
    pos = torch.tensor(E2M1_VALUES, dtype=torch.float32)
    return torch.cat([pos, -pos]).to(dtype=dtype, device=device)


def dequantize(packed: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """``[..., N, K/2]`` codes + ``[..., N, K/32]`` scales -> ``[..., N, K]`` in ``dtype``.

    The product of an e2m1 value and a power of two is exact in bf16/f16/fp32, so the result
    does not depend on the order of the two steps."""
    lut = e2m1_lut(torch.float32, packed.device)
    lo = (packed & 0x0F).long()
    hi = (packed >> 4).long()
    vals = torch.stack([lut[lo], lut[hi]], dim=-1).flatten(-2)  # [..., N, K]
    exp = scales.to(torch.int32) - 127
    scale = torch.exp2(exp.to(torch.float32))
    k = vals.shape[-1]
    vals = vals.view(*vals.shape[:-1], k // BLOCK, BLOCK) * scale.unsqueeze(-1)
    return vals.view(*vals.shape[:-2], k).to(dtype)


def quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``[..., N, K]`` float -> (``[..., N, K/2]`` u8 codes, ``[..., N, K/32]`` u8 scales)."""
    if w.shape[-1] % BLOCK:
        raise ValueError(f"K={w.shape[-1]} is not a multiple of {BLOCK}")
    x = w.float().reshape(*w.shape[:-1], w.shape[-1] // BLOCK, BLOCK)
    amax = x.abs().amax(dim=-1, keepdim=True)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp_min(1e-38))) - 2, torch.zeros_like(amax))
    e = e.clamp(-127, 127)
    y = x / torch.exp2(e)
    mag = y.abs().clamp(max=6.0)
    grid = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=w.device)
    # nearest grid point; ties go to the even code (code 2k is even)
    d = (mag.unsqueeze(-1) - grid).abs()
    best = d.min(dim=-1, keepdim=True).values
    cand = (d <= best + 1e-7)
    codes = torch.arange(8, device=w.device)
    even_pref = torch.where(cand, (codes % 2) * 8 + codes, torch.full_like(codes, 1000))
    code = even_pref.argmin(dim=-1)
    code = code | ((y < 0) & (code > 0)).long() << 3
    code = code.reshape(*w.shape[:-1], w.shape[-1]).to(torch.uint8)
    packed = (code[..., 0::2] | (code[..., 1::2] << 4)).to(torch.uint8)
    scales = (e.squeeze(-1) + 127).to(torch.uint8)
    return packed.contiguous(), scales.contiguous()
