"""Multi-token prediction (MTP) speculative decoding.

The checkpoint's ``mtp.*`` block is one extra decoder layer (gated full attention + MoE) fed by
``fc(concat(rmsnorm(embed(token)), rmsnorm(hidden)))`` and followed by its own final norm; it
shares the target's embedding and LM head. It predicts the token after next: fed the token at
position ``p`` and the target's hidden state at ``p - 1``, it drafts the token at ``p + 1``.

One round per lane (``Model.speculative_decode``):

1. **draft** - ``k`` sequential steps of the MTP layer alone, seeded by the target's final-normed
   hidden of the last forwarded position and the last committed token; the MTP layer keeps its
   own paged KV cache (same block tables and positions as the target);
2. **verify** - one wide target forward over ``B x (k+1)`` rows (last committed token plus the
   drafts). DeltaNet layers run this forward without writing their state back, and keep their
   per-row inputs;
3. **accept** - greedy: the longest draft prefix that equals the target's argmax, plus the
   target's next token (``forced`` mode instead accepts each position with probability 0.7,
   so the verify path can be timed independently of random weights);
4. **commit** - DeltaNet state is advanced over exactly the accepted rows from the saved inputs
   (conv window and recurrent state end where the accepted prefix ends); target KV rows past the
   accepted prefix are never read and get overwritten; the MTP layer re-runs over the accepted
   rows with the target's hidden states ("catch-up"), so its KV cache matches the committed text.

Reference behaviour: ``mtp.py:115-817`` (``MTP``, ``draft``, ``verify_and_commit``, forced
drafts), ``graph_verify_wide.py`` (wide verify) and the rollback by replaying the accepted
prefix (``Model.deltanet_verify_rollback``).
"""

from __future__ import annotations

import random

import torch

from ..ops import core as ops
from .qwen35 import StepInputs


class MTPHead:
    def __init__(self, model, w: dict, k: int = 3, forced_accept: float | None = None, seed: int = 0):
        self.m = model
        self.w = w
        self.k = k
        self.forced_accept = forced_accept
        self.rng = random.Random(seed)
        cfg = model.cfg
        rows = model.num_blocks * model.block_size
        dev, dt = model.device, model.dtype
        self.k_cache = torch.zeros(rows, model.nkv, cfg.head_dim, dtype=dt, device=dev)
        self.v_cache = torch.zeros(rows, model.nkv, cfg.head_dim, dtype=dt, device=dev)
        self.seed_h = torch.zeros(model.max_batch, cfg.hidden, dtype=dt, device=dev)
        self.snap_h = torch.zeros(model.num_snapshots, cfg.hidden, dtype=dt, device=dev)
        self.rounds = 0
        self.accepted = 0
        self.drafted = 0

    # ------------------------------------------------------------------ state
    def begin(self, lane: int) -> None:
        self.seed_h[lane].zero_()

    def copy_block(self, d: int, s: int, filled: int) -> None:
        self.k_cache[d:d + filled].copy_(self.k_cache[s:s + filled])
        self.v_cache[d:d + filled].copy_(self.v_cache[s:s + filled])

    def save_snapshot(self, lane: int, snap: int) -> None:
        self.snap_h[snap].copy_(self.seed_h[lane])

    def load_snapshot(self, lane: int, snap: int) -> None:
        self.seed_h[lane].copy_(self.snap_h[snap])

    # ------------------------------------------------------------------ layer
    def combine(self, tokens: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
        eps = self.m.cfg.eps
        e = ops.rmsnorm(ops.embed(tokens, self.m.w["embed"]), self.w["pre_fc_norm_embedding"], eps)
        h = ops.rmsnorm(hidden, self.w["pre_fc_norm_hidden"], eps)
        return ops.linear(torch.cat([e, h], dim=-1), self.w["fc"])

    def layer(self, x_in: torch.Tensor, b: StepInputs) -> torch.Tensor:
        """The MTP decoder layer on residual input ``x_in``; returns its final-normed output."""
        m, L, eps = self.m, self.w["layer"], self.m.cfg.eps
        h = ops.rmsnorm(x_in, L["in_norm"], eps)
        a = m._attention_core(L, h, b, self.k_cache, self.v_cache)
        x, h = m.comm.allreduce_add_rmsnorm(a, x_in.clone(), L["post_norm"], eps)
        mo = m._moe(L, h)
        _, h = m.comm.allreduce_add_rmsnorm(mo, x, self.w["norm"], eps)
        return h

    def catch_up(self, b: StepInputs, h_all: torch.Tensor) -> None:
        """Fill the MTP KV cache for the rows of a target forward: row at position p pairs its
        token with the target hidden at p - 1 (the lane's seed for a segment's first row)."""
        cu, lanes = b.cu_h, b.seg_lane_h
        first = torch.tensor([cu[s] for s in range(len(lanes))], device=h_all.device)
        prev = torch.empty_like(h_all)
        prev[1:] = h_all[:-1]
        prev[first] = self.seed_h[torch.tensor(lanes, device=h_all.device)]
        self.layer(self.combine(b.tokens, prev), b)
        last = torch.tensor([cu[s + 1] - 1 for s in range(len(lanes))], device=h_all.device)
        self.seed_h[torch.tensor(lanes, device=h_all.device)] = h_all[last]

    # ------------------------------------------------------------------ draft
    def draft(self, lanes, tokens, positions) -> torch.Tensor:
        """``k`` draft tokens per lane, [B, k] on the device (no host sync)."""
        m = self.m
        dev = m.device
        B = len(lanes)
        lane_t = torch.tensor(lanes, device=dev)
        hidden = self.seed_h[lane_t]
        tok = torch.tensor([int(t) for t in tokens], dtype=torch.int64, device=dev)
        out = []
        for i in range(self.k):
            b = m.make_inputs([(l, [0], p + i) for l, p in zip(lanes, positions)])
            b.tokens = tok
            h = self.layer(self.combine(tok, hidden), b)
            tok = m.greedy(h)[0]
            out.append(tok)
            hidden = h
        self.drafted += B * self.k
        return torch.stack(out, dim=1)

    def accept(self, drafts: list[int], argmax: list[int]) -> int:
        n = 0
        if self.forced_accept is not None:
            while n < self.k and self.rng.random() < self.forced_accept:
                n += 1
            return n
        while n < self.k and drafts[n] == argmax[n]:
            n += 1
        return n


def attach(model, k: int = 3, forced_accept: float | None = None) -> MTPHead | None:
    """Create the MTP head from ``model.w["mtp"]`` (None when the weights have no MTP block)."""
    if model.w.get("mtp") is None:
        return None
    model.mtp = MTPHead(model, model.w["mtp"], k=k, forced_accept=forced_accept)
    return model.mtp
