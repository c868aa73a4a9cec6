"""Qwen3.5-MoE runtime: the ``Runner`` the scheduler drives.

One instance per rank. It owns the static pools and runs every forward as one varlen batch of
segments, so prefill, packed multi-request prefill, batched decode, mixed decode + prefill and
MTP verify are the same call with different segment lengths:

* paged KV pool per full-attention layer: ``[num_blocks * block_size, kv_heads_local, head_dim]``
  (block 0 is the pad sentinel, reference ``block_pool.py:38``);
* DeltaNet live state per lane: conv window ``[lanes, C_local, K-1]`` and fp32 recurrent state
  ``[lanes, v_heads_local, dk, dv]`` per linear-attention layer;
* snapshot pool (turn boundaries of the session cache): the same two states per slot, plus the
  cached next-token logits and the MTP seed hidden of that boundary.

Per-layer dataflow (``Model._forward``), with the TP collective fused into the next norm::

    x = embed(tokens); h = rmsnorm(x, in_norm[0])
    for each layer:
        partial = deltanet(h) | gated_attention(h)        # row-parallel partial sums
        x, h = allreduce_add_rmsnorm(partial, x, post_norm)   # prefill: out_proj GEMM fused in
        partial = moe(h)                                   # EP experts + TP shared expert
        x, h = allreduce_add_rmsnorm(partial, x, next in_norm | final_norm)
    logits = lm_head(h[logit rows])                        # vocab parallel, all-gathered

Reference parity: ``model.py:1344-4355`` (``Model``; the ``Runner`` methods ``begin``,
``prefill``, ``prefill_batch``, ``decode``, ``save_snapshot``/``load_snapshot``,
``attach_blocks``/``extend_blocks``/``copy_block``, ``sample_batch``, ``cache_node_logits``,
``score``) and ``scheduler.py:399-516`` (the ``Runner`` protocol).
"""

from __future__ import annotations

import os
from collections.abc import Sequence
from dataclasses import dataclass

import torch

from ..ops import core as ops
from ..parallel.comm import Comm
from ..utils import flags
from ..parallel.plan import Plan
from .config import FULL, Qwen35Config

RESERVED_BLOCK = 0


@dataclass
class _Deferred:
    """A mixer's output projection not yet run: ``x @ w^T`` is fused into the all-reduce."""

    x: torch.Tensor
    w: torch.Tensor


@dataclass
class StepInputs:
    """Device-side description of one varlen forward (plus host copies for the CPU path)."""

    tokens: torch.Tensor  # [T] int64
    positions: torch.Tensor  # [T] int32
    rows: torch.Tensor  # [T] int32 physical KV rows
    seg_lane: torch.Tensor  # [S] int32
    cu: torch.Tensor  # [S+1] int32
    seg_start: torch.Tensor  # [S] int32
    logit_rows: torch.Tensor  # [R] int64
    seg_lane_h: list[int]
    cu_h: list[int]
    seg_start_h: list[int]
    max_ctx: int = 0
    verify: bool = False  # MTP verify: DeltaNet layers keep their inputs and do not write state


class Model:
    """Per-rank Qwen3.5-MoE model with its static pools; implements the scheduler's Runner."""

    def __init__(
        self,
        cfg: Qwen35Config,
        weights: dict,
        plan: Plan,
        comm: Comm | None = None,
        device: torch.device | str = "cpu",
        dtype: torch.dtype = torch.bfloat16,
        max_batch: int = 8,
        max_seq: int = 4096,
        block_size: int = 16,
        num_blocks: int | None = None,
        num_snapshots: int = 16,
    ) -> None:
        self.cfg, self.w, self.plan = cfg, weights, plan
        self.comm = comm or Comm()
        self.device = torch.device(device)
        self.dtype = dtype
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.block_size = block_size
        self.max_blocks = (max_seq + block_size - 1) // block_size
        if num_blocks is None:
            num_blocks = max_batch * self.max_blocks + 1
        self.num_blocks = num_blocks
        self.num_snapshots = num_snapshots
        self.mtp = None  # set by models.mtp.attach
        self.full_slot = {i: j for j, i in enumerate(cfg.full_layers)}
        self.lin_slot = {i: j for j, i in enumerate(cfg.linear_layers)}
        p = plan
        self.nq, self.nkv = p.q.count, p.kv.count
        self.nk, self.nv = p.dn_k.count, p.dn_v.count
        self.conv_ch = 2 * self.nk * cfg.dn_k_dim + self.nv * cfg.dn_v_dim
        dev, dt = self.device, dtype
        rows = num_blocks * block_size
        self.k_cache = [torch.zeros(rows, self.nkv, cfg.head_dim, dtype=dt, device=dev) for _ in cfg.full_layers]
        self.v_cache = [torch.zeros(rows, self.nkv, cfg.head_dim, dtype=dt, device=dev) for _ in cfg.full_layers]
        nl, km1 = len(cfg.linear_layers), cfg.conv_kernel - 1
        self.conv_state = torch.zeros(nl, max_batch, self.conv_ch, km1, dtype=dt, device=dev)
        self.rec_state = torch.zeros(nl, max_batch, self.nv, cfg.dn_k_dim, cfg.dn_v_dim, dtype=torch.float32, device=dev)
        self.snap_conv = torch.zeros(nl, num_snapshots, self.conv_ch, km1, dtype=dt, device=dev)
        self.snap_rec = torch.zeros(nl, num_snapshots, self.nv, cfg.dn_k_dim, cfg.dn_v_dim, dtype=torch.float32, device=dev)
        self.snap_logits: dict[int, torch.Tensor] = {}
        self.tables: list[list[int]] = [[] for _ in range(max_batch)]
        self.table_dev = torch.zeros(max_batch, self.max_blocks, dtype=torch.int32, device=dev)
        self._dirty: set[int] = set(range(max_batch))
        self.last_hidden: torch.Tensor | None = None  # pre-final-norm hidden of the logit rows (MTP seed)
        self.fault: dict[str, object] = {}  # accuracy-gate calibration faults (serving.faults)
        self._vsave: dict = {}  # MTP verify: per DeltaNet layer (conv inputs, ab rows)
        self._h2d = 0  # bytes copied host -> device for step inputs (bench accounting)
        self._d2h = 0  # bytes read back device -> host (sampled ids)
        self.gpu_marks = None  # list -> CUDA events at each input upload ("in") and result read ("out")
        self.stamps = None  # utils.telemetry.Stamps -> in-graph clock stamps at layer boundaries
        self._defer_out = False  # set inside _layers while the out projections fuse into the all-reduce
        self.fuse_shared = bool(flags.get("QB_MOE_FUSE_SHARED"))  # shared expert added in the routed combine
        self.greedy_head = bool(flags.get("QB_GREEDY_HEAD"))  # greedy ids from gathered (max, index) pairs
        self.route_log: list | None = None  # list -> every MoE call's top-k expert ids, in call order (tests)
        self.status_watch = None  # utils.devstatus.StatusWatch (CUDA): polled by the scheduler / workers

    def _gpu_mark(self, tag: str) -> None:
        """Stream-ordered event where a step's device work starts (input upload) or ends (the
        result read): a benchmark sums these intervals as the device time of its steps."""
        if self.gpu_marks is not None and self.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.gpu_marks.append((tag, ev))

    def _stamp(self, tag: str) -> None:
        if self.stamps is not None:
            self.stamps.mark(tag)

    def _dstamp(self, tag: str) -> None:
        """A stamp inside a layer part (only when the installed ``Stamps`` asks for detail)."""
        if self.stamps is not None and self.stamps.detail:
            self.stamps.mark(tag)

    def io_bytes(self) -> tuple[int, int]:
        return self._h2d, self._d2h

    # ================================================================== Runner: lanes & blocks
    def begin(self, lane: int) -> None:
        for j in range(self.conv_state.shape[0]):
            self.conv_state[j, lane].zero_()
            self.rec_state[j, lane].zero_()
        self.tables[lane] = []
        self._dirty.add(lane)
        if self.mtp is not None:
            self.mtp.begin(lane)

    def lane_blocks(self, lane: int) -> tuple[int, ...]:
        return tuple(self.tables[lane])

    def lane_block_count(self, lane: int) -> int:
        return len(self.tables[lane])

    def attach_blocks(self, lane: int, blocks: Sequence[int]) -> None:
        if len(blocks) > self.max_blocks:
            raise ValueError(f"lane {lane}: {len(blocks)} blocks > max {self.max_blocks}")
        self.tables[lane] = list(blocks)
        self._dirty.add(lane)

    def extend_blocks(self, grants: Sequence[tuple[int, int]]) -> None:
        for lane, blk in grants:
            if len(self.tables[lane]) >= self.max_blocks:
                raise ValueError(f"lane {lane}: block table full ({self.max_blocks})")
            self.tables[lane].append(int(blk))
            self._dirty.add(lane)

    def copy_block(self, dst_block: int, src_block: int, filled: int) -> None:
        bs = self.block_size
        s, d = src_block * bs, dst_block * bs
        for kc, vc in zip(self.k_cache, self.v_cache):
            kc[d:d + filled].copy_(kc[s:s + filled])
            vc[d:d + filled].copy_(vc[s:s + filled])
        if self.mtp is not None:
            self.mtp.copy_block(d, s, filled)

    def _sync_tables(self) -> None:
        if not self._dirty:
            return
        for lane in sorted(self._dirty):
            t = self.tables[lane]
            row = torch.zeros(self.max_blocks, dtype=torch.int32)
            if t:
                row[: len(t)] = torch.tensor(t, dtype=torch.int32)
            self.table_dev[lane].copy_(row.to(self.device), non_blocking=True)
            self._h2d += row.numel() * 4
        self._dirty.clear()

    # ================================================================== Runner: snapshots
    def save_snapshot(self, lane: int, snap: int) -> None:
        self.snap_conv[:, snap].copy_(self.conv_state[:, lane])
        self.snap_rec[:, snap].copy_(self.rec_state[:, lane])
        if self.mtp is not None:
            self.mtp.save_snapshot(lane, snap)

    def load_snapshot(self, lane: int, snap: int) -> None:
        self.conv_state[:, lane].copy_(self.snap_conv[:, snap])
        self.rec_state[:, lane].copy_(self.snap_rec[:, snap])
        if self.mtp is not None:
            self.mtp.load_snapshot(lane, snap)

    def cache_node_logits(self, snap: int, logits) -> None:
        self.snap_logits[snap] = logits.detach().clone()

    def cached_node_logits(self, snap: int):
        return self.snap_logits[snap]

    # ================================================================== inputs
    def _row(self, lane: int, pos: int) -> int:
        blk = pos // self.block_size
        t = self.tables[lane]
        if blk >= len(t):
            raise IndexError(f"lane {lane}: position {pos} has no block (table has {len(t)})")
        return t[blk] * self.block_size + pos % self.block_size

    def make_inputs(self, segs: Sequence[tuple[int, Sequence[int], int]], logit_rows: Sequence[int] | None = None) -> StepInputs:
        """``segs`` = ``(lane, ids, start)`` per segment; logits default to each segment's last row."""
        toks, pos, rows, lanes, cu, starts, last = [], [], [], [], [0], [], []
        for lane, ids, start in segs:
            n = len(ids)
            if n == 0:
                raise ValueError("empty segment")
            if start + n > self.max_seq:
                raise ValueError(f"lane {lane}: {start + n} tokens > max_seq {self.max_seq}")
            toks.extend(int(t) for t in ids)
            pos.extend(range(start, start + n))
            rows.extend(self._row(lane, p) for p in range(start, start + n))
            lanes.append(lane)
            starts.append(start)
            cu.append(cu[-1] + n)
            last.append(cu[-1] - 1)
        if logit_rows is None:
            logit_rows = last
        self._gpu_mark("in")
        dev = self.device
        i32 = torch.int32
        packed = torch.tensor(pos + rows + lanes + cu + starts, dtype=i32)
        if dev.type == "cuda":
            packed = packed.pin_memory().to(dev, non_blocking=True)
            tok = torch.tensor(toks, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            lr = torch.tensor(list(logit_rows), dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
            self._h2d += packed.numel() * 4 + tok.numel() * 8 + lr.numel() * 8
        else:
            tok = torch.tensor(toks, dtype=torch.int64)
            lr = torch.tensor(list(logit_rows), dtype=torch.int64)
        t, s = len(toks), len(lanes)
        o = 0
        positions = packed[o:o + t]; o += t  # noqa: E702
        prow = packed[o:o + t]; o += t  # noqa: E702
        seg_lane = packed[o:o + s]; o += s  # noqa: E702
        cu_d = packed[o:o + s + 1]; o += s + 1  # noqa: E702
        seg_start = packed[o:o + s]
        self._sync_tables()
        max_ctx = max(st + (cu[i + 1] - cu[i]) for i, st in enumerate(starts))
        return StepInputs(tok, positions, prow, seg_lane, cu_d, seg_start, lr, lanes, cu, starts, max_ctx)

    # ================================================================== layers
    def _deltanet(self, i: int, L: dict, h: torch.Tensor, b: StepInputs) -> torch.Tensor:
        cfg = self.cfg
        j = self.lin_slot[i]
        nk, nv, dk, dv = self.nk, self.nv, cfg.dn_k_dim, cfg.dn_v_dim
        c = self.conv_ch
        proj = ops.linear(h, L["w_in"])  # [T, c + nv*dv + 2nv]
        self._dstamp("dn.in_proj")
        if (h.is_cuda and not b.verify and b.cu_h is not None and len(b.cu_h) - 1 == h.shape[0]
                and not self.fault.get("skip_deltanet_gate")):
            # decode (one token per lane): conv, delta step and gated norm in one kernel
            normed = ops.deltanet_decode(proj, self.conv_state[j], L["conv_w"], L["A_log"], L["dt_bias"],
                                         self.rec_state[j], L["norm_w"], b.seg_lane, nk, nv, dk, dv, cfg.eps,
                                         b.seg_lane_h)
            self._dstamp("dn.decode_mixer")
            return self._out_proj(normed, L["w_out"])
        commit = not b.verify
        if b.verify:  # keep the per-row inputs: the accepted prefix is committed later
            self._vsave[j] = (proj[:, :c].clone(), proj[:, c + nv * dv:].clone())
        qkv = ops.causal_conv_varlen(proj[:, :c], self.conv_state[j], L["conv_w"], b.seg_lane, b.cu,
                                     b.seg_lane_h, b.cu_h, commit=commit)
        self._dstamp("dn.conv")
        z = proj[:, c:c + nv * dv]
        ab = proj[:, c + nv * dv:]
        core = ops.gated_delta_varlen(qkv, ab, L["A_log"], L["dt_bias"], self.rec_state[j], b.seg_lane, b.cu,
                                      nk, nv, dk, dv, b.seg_lane_h, b.cu_h, commit=commit)
        self._dstamp("dn.recurrence")
        if self.fault.get("skip_deltanet_gate"):
            normed = ops.rmsnorm(core, torch.ones(dv, device=h.device), cfg.eps).reshape(-1, nv * dv)
        else:
            normed = ops.gated_rmsnorm(core, z.reshape(-1, nv, dv), L["norm_w"], cfg.eps).reshape(-1, nv * dv)
        self._dstamp("dn.gated_norm")
        return self._out_proj(normed, L["w_out"])

    def _attention(self, i: int, L: dict, h: torch.Tensor, b: StepInputs) -> torch.Tensor:
        j = self.full_slot[i]
        return self._attention_core(L, h, b, self.k_cache[j], self.v_cache[j], j)

    def _attention_core(self, L: dict, h: torch.Tensor, b: StepInputs, k_cache, v_cache,
                        j: int | None = None) -> torch.Tensor:
        cfg = self.cfg
        hd, nq, nkv = cfg.head_dim, self.nq, self.nkv
        qkv = ops.linear(h, L["w_qkv"])
        self._dstamp("attn.qkv_proj")
        t = qkv.shape[0]
        qg = qkv[:, : nq * 2 * hd].reshape(t, nq, 2 * hd)
        q, gate = qg[..., :hd], qg[..., hd:]
        k = qkv[:, nq * 2 * hd: nq * 2 * hd + nkv * hd].reshape(t, nkv, hd)
        v = qkv[:, nq * 2 * hd + nkv * hd:].reshape(t, nkv, hd)
        theta = float(self.fault.get("rope_base", cfg.rope_theta))
        q = ops.qk_norm_rope_kv_write(q, k, v, L["q_norm"], L["k_norm"], b.positions, b.rows,
                                      k_cache, v_cache, cfg.rotary_dim, theta, cfg.eps)
        if j is not None and self.fault.get("fp8_kv_no_scale"):
            rows = b.rows.long()  # the rows just written, truncated through e4m3 without a scale
            k_cache[rows] = k_cache[rows].to(torch.float8_e4m3fn).to(k_cache.dtype)
            v_cache[rows] = v_cache[rows].to(torch.float8_e4m3fn).to(v_cache.dtype)
        self._dstamp("attn.norm_rope_kv")
        o = ops.attention_varlen(q, k_cache, v_cache, self.table_dev, b.seg_lane, b.cu,
                                 b.seg_start, self.block_size, b.seg_lane_h, b.cu_h, b.seg_start_h,
                                 self.tables if h.device.type == "cpu" else None, b.positions, b.max_ctx,
                                 causal=not (j is not None and self.fault.get("flip_causal_mask")
                                             and j == int(self.fault.get("flip_causal_mask_layer", 0))))
        self._dstamp("attn.core")
        o = ops.sigmoid_gate_mul(o.reshape(t, nq * hd), gate.reshape(t, nq * hd))
        self._dstamp("attn.gate")
        return self._out_proj(o, L["w_o"])

    def _out_proj(self, x: torch.Tensor, w: torch.Tensor):
        """The mixer's row-parallel output projection, or (x, w) left for the all-reduce that
        follows when it fuses the two (GEMM -> reduce-scatter over peer memory)."""
        if self._defer_out:
            return _Deferred(x, w)
        return ops.linear(x, w)

    def _moe(self, L: dict, h: torch.Tensor) -> torch.Tensor:
        cfg, p = self.cfg, self.plan
        if "w_rsh" in L:  # router and shared gate|up in one GEMM
            rs = ops.linear(h, L["w_rsh"])
            rl, g13 = rs[:, : cfg.experts + 1], rs[:, L["rsh_off"]:]
        else:
            rl, g13 = ops.linear(h, L["w_router"]), None  # [T, E+1]: router logits | shared-expert gate logit
        self._dstamp("moe.router_proj")
        topw, topi = ops.router_topk(rl[:, : cfg.experts], cfg.top_k)
        self._dstamp("moe.topk")
        if self.route_log is not None:
            self.route_log.append(topi)
        drop = self.fault.get("drop_expert")
        if drop is not None:
            topw = torch.where(topi == int(drop), torch.zeros_like(topw), topw)
        if g13 is None:
            g13 = ops.linear(h, L["w_sh13"])
        sh = ops.linear(ops.silu_mul(g13), L["w_sh2"])
        self._dstamp("moe.shared")
        if not self.fuse_shared:
            routed = ops.moe_routed(h, topw, topi, L["experts"], p.experts.start, p.experts.count)
            self._dstamp("moe.routed")
            return ops.shared_gate_combine(routed, sh, rl[:, cfg.experts])
        # routed experts; their combine also adds sigmoid(gate) x the shared expert's rows
        out = ops.moe_routed(h, topw, topi, L["experts"], p.experts.start, p.experts.count, shared=sh,
                             gate=rl[:, cfg.experts])
        self._dstamp("moe.routed")
        return out

    def _layers(self, x: torch.Tensor, b: StepInputs) -> tuple[torch.Tensor, torch.Tensor]:
        cfg, comm, layers = self.cfg, self.comm, self.w["layers"]
        h = ops.rmsnorm(x, layers[0]["in_norm"], cfg.eps)
        self._stamp("embed")
        fuse_out = hasattr(comm, "fuses_linear") and comm.fuses_linear(x.shape[0])
        for i, L in enumerate(layers):
            full = L["kind"] == FULL
            self._defer_out = fuse_out
            try:
                mix = self._attention(i, L, h, b) if full else self._deltanet(i, L, h, b)
            finally:
                self._defer_out = False
            self._stamp("attention" if full else "deltanet")
            # the residual after this all-reduce is read only by the next one (QB_SP_RES_LOCAL lets
            # sequence-parallel sizes keep it on each rank's own rows)
            if isinstance(mix, _Deferred):
                x, h = comm.linear_allreduce_add_rmsnorm(mix.x, mix.w, x, L["post_norm"], cfg.eps, res_local=True)
            else:
                x, h = comm.allreduce_add_rmsnorm(mix, x, L["post_norm"], cfg.eps, res_local=True)
            self._stamp("allreduce")
            m = self._moe(L, h)
            self._stamp("moe")
            nxt = layers[i + 1]["in_norm"] if i + 1 < len(layers) else self.w["final_norm"]
            # before another layer, h only feeds its input projection: that GEMM may do the
            # all-gather itself (QB_AG_GEMM; the residual then stays on this rank's rows until the
            # next all-reduce, which reads only those)
            last = i + 1 == len(layers)  # the forward's last residual is read as a whole (MTP seed rows)
            x, h = comm.allreduce_add_rmsnorm(m, x, nxt, cfg.eps, gather_out=not last, res_local=not last)
            self._stamp("allreduce")
        return x, h

    def _forward(self, b: StepInputs) -> torch.Tensor:
        """Runs every layer over the batch; returns the final-normed hidden of the logit rows and
        keeps the matching pre-norm residual in ``last_hidden`` (the MTP seed)."""
        self._stamp("start")
        x = ops.embed(b.tokens, self.w["embed"])
        x, h = self._layers(x, b)
        self.last_hidden = x.index_select(0, b.logit_rows)
        self.last_h_all = h
        return h.index_select(0, b.logit_rows)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """Full-vocab logits [R, V] (vocab-parallel GEMM, then all-gathered over ranks)."""
        local = ops.linear(h, self.w["lm_head"])
        out = self.comm.all_gather_last(local)
        self._stamp("lm_head")
        return out

    def greedy(self, h: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Greedy next-token ids of the rows of ``h`` through the vocabulary-parallel head: every
        rank takes the (max, index) of its own vocabulary slice and only those pairs cross the
        ranks (8 bytes per row and rank instead of each row's full logits); the largest value
        wins, the lowest index on a tie, which is exactly the argmax of the gathered rows.
        Returns (ids [R] int64, this rank's logits slice [R, V / world]); ``full_rows`` gathers
        the full logits of the rows that need them. With ``QB_GREEDY_HEAD=0`` the rows are
        all-gathered first (the slice is then the full rows). Reference behaviour:
        ``mtp.py:640-658`` (``greedy_token``)."""
        if not self.greedy_head:
            lg = self.logits(h)
            return ops.argmax_rows(lg)[1], lg
        local = ops.linear(h, self.w["lm_head"])
        ids = self.comm.argmax_gather(local, self.plan.vocab.start)
        self._stamp("lm_head")
        return ids, local

    def full_rows(self, local: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits of rows of a ``greedy`` slice (a collective: every rank calls
        it with the same rows)."""
        return self.comm.all_gather_last(local) if self.greedy_head else local

    # ================================================================== Runner: forwards
    @torch.inference_mode()
    def forward(self, segs, logit_rows=None) -> torch.Tensor:
        b = self.make_inputs(segs, logit_rows)
        lg = self.logits(self._forward(b))
        if self.mtp is not None:
            self.mtp.catch_up(b, self.last_h_all)
        return lg

    # ================================================================== MTP speculative decode
    @torch.inference_mode()
    def speculative_decode(self, lanes, tokens, positions, budgets, stops) -> list[list[int]]:
        """One MTP round per lane (see ``models.mtp``): draft k, verify k+1 rows in one forward,
        accept, commit DeltaNet state over the accepted rows, re-run the MTP layer on them."""
        mtp = self.mtp
        k = mtp.k
        B = len(lanes)
        drafts = mtp.draft(lanes, tokens, positions)  # [B, k]
        segs = [(l, [0] * (k + 1), p) for l, p in zip(lanes, positions)]
        b = self.make_inputs(segs, logit_rows=list(range(B * (k + 1))))
        tok0 = torch.tensor([int(t) for t in tokens], dtype=torch.int64, device=self.device)
        b.tokens = torch.cat([tok0[:, None], drafts], dim=1).reshape(-1)
        b.verify = True
        self._vsave = {}
        h = self._forward(b)
        am = self.greedy(h)[0].view(B, k + 1)
        self._gpu_mark("out")
        am_h, dr_h = am.tolist(), drafts.tolist()  # the round's one host sync
        self._d2h += 8 * B * (2 * k + 1)
        ns = [mtp.accept(dr_h[i], am_h[i]) for i in range(B)]
        mtp.rounds += B
        mtp.accepted += sum(ns)
        self._commit_verify(b, lanes, positions, ns, k)
        out = []
        for i in range(B):
            toks = dr_h[i][:ns[i]] + [am_h[i][ns[i]]]
            st = set(stops[i])
            cut = next((j for j, t in enumerate(toks) if t in st), None)
            if cut is not None:
                toks = toks[:cut + 1]
            out.append(toks[:max(1, budgets[i])])
        return out

    def _commit_verify(self, b: StepInputs, lanes, positions, ns, k) -> None:
        """Advance DeltaNet state over each lane's accepted rows (the committed token plus the
        accepted drafts) from the verify forward's saved inputs, then run the MTP catch-up."""
        dev = self.device
        idx, cu, seg_l = [], [0], []
        for i, (l, n) in enumerate(zip(lanes, ns)):
            idx.extend(range(i * (k + 1), i * (k + 1) + n + 1))
            cu.append(cu[-1] + n + 1)
            seg_l.append(l)
        it = torch.tensor(idx, dtype=torch.long, device=dev)
        seg_lane_d = torch.tensor(seg_l, dtype=torch.int32, device=dev)
        cu_d = torch.tensor(cu, dtype=torch.int32, device=dev)
        cfg = self.cfg
        for i, L in enumerate(self.w["layers"]):
            if L["kind"] == FULL:
                continue
            j = self.lin_slot[i]
            conv_in, ab = self._vsave[j]
            qkv = ops.causal_conv_varlen(conv_in.index_select(0, it), self.conv_state[j], L["conv_w"], seg_lane_d,
                                         cu_d, seg_l, cu, commit=True)
            ops.gated_delta_varlen(qkv, ab.index_select(0, it), L["A_log"], L["dt_bias"], self.rec_state[j],
                                   seg_lane_d, cu_d, self.nk, self.nv, cfg.dn_k_dim, cfg.dn_v_dim, seg_l, cu,
                                   commit=True)
        self._vsave = {}
        if self.mtp is not None:
            acc_segs = [(l, [0] * (n + 1), p) for l, n, p in zip(lanes, ns, positions)]
            ab_in = self.make_inputs(acc_segs)
            ab_in.tokens = b.tokens.index_select(0, it)
            self.mtp.catch_up(ab_in, self.last_h_all.index_select(0, it))

    def _commit_verify_device(self, b: StepInputs, n: torch.Tensor, k: int) -> None:
        """``_commit_verify`` with fixed shapes, for a captured graph: ``n`` [B] (device, int64)
        accepted drafts per lane of the verify batch ``b`` (B segments of k+1 rows). The accepted
        rows are compacted on the device into a full-size batch whose tail is padding (the kernels
        bound their work by the device segment table); the MTP catch-up runs over all k+1 rows of
        every lane (KV rows past the accepted prefix are rewritten before any read) and the seed
        hidden of each lane becomes the one of its last accepted row."""
        B = n.shape[0]
        R = B * (k + 1)
        dev = self.device
        cu = torch.zeros(B + 1, dtype=torch.int64, device=dev)
        cu[1:] = torch.cumsum(n + 1, 0)
        r = torch.arange(R, device=dev)
        lane_of = torch.searchsorted(cu[1:], r, right=True).clamp_(max=B - 1)
        src = (lane_of * (k + 1) + (r - cu[lane_of])).clamp_(0, R - 1)
        cu32 = cu.to(torch.int32)
        cfg = self.cfg
        for i, L in enumerate(self.w["layers"]):
            if L["kind"] == FULL:
                continue
            j = self.lin_slot[i]
            conv_in, ab = self._vsave[j]
            qkv = ops.causal_conv_varlen(conv_in.index_select(0, src), self.conv_state[j], L["conv_w"], b.seg_lane,
                                         cu32, b.seg_lane_h, b.cu_h, commit=True)
            ops.gated_delta_varlen(qkv, ab.index_select(0, src), L["A_log"], L["dt_bias"], self.rec_state[j],
                                   b.seg_lane, cu32, self.nk, self.nv, cfg.dn_k_dim, cfg.dn_v_dim, b.seg_lane_h,
                                   b.cu_h, commit=True)
        self._vsave = {}
        mtp = self.mtp
        if mtp is not None:
            h_all = self.last_h_all
            first = torch.arange(0, R, k + 1, device=dev)
            prev = torch.empty_like(h_all)
            prev[1:] = h_all[:-1]
            lanes = b.seg_lane.long()
            prev[first] = mtp.seed_h.index_select(0, lanes)
            mtp.layer(mtp.combine(b.tokens, prev), b)
            mtp.seed_h.index_copy_(0, lanes, h_all.index_select(0, first + n))

    def prefill(self, lane: int, ids: Sequence[int], start: int):
        return self.forward([(lane, ids, start)])[0:1]

    def prefill_batch(self, calls: Sequence[tuple[int, Sequence[int], int]]) -> list:
        if not calls:
            return []
        lg = self.forward(list(calls))
        return [lg[i:i + 1] for i in range(len(calls))]

    def decode(self, lanes: Sequence[int], tokens: Sequence[int], positions: Sequence[int]):
        return self.forward([(l, [t], p) for l, t, p in zip(lanes, tokens, positions)])

    # ------------------------------------------------------------------ one-step overlap
    @torch.inference_mode()
    def decode_launch(self, lanes, tokens, positions, src_rows, keep_rows=()):
        """A decode step whose result is read later (``decode_collect``): a token of -1 takes the
        previous launch's greedy id at row ``src_rows[i]`` on the device, so the host never has to
        see it first. The step's greedy ids are copied to pinned host memory behind an event; the
        logits rows in ``keep_rows`` are kept (the node logits of lanes that finish here)."""
        host = [int(t) if t >= 0 else 0 for t in tokens]
        b = self.make_inputs([(l, [t], p) for l, t, p in zip(lanes, host, positions)])
        self._feed_back(b.tokens, tokens, src_rows)
        ids, local = self.greedy(self._forward(b))
        if self.mtp is not None:
            self.mtp.catch_up(b, self.last_h_all)
        return self._launch_tail(ids, local, len(lanes), keep_rows)

    def _dev_index(self, xs) -> torch.Tensor:
        t = torch.tensor(list(xs), dtype=torch.long)
        if self.device.type == "cuda":
            return t.pin_memory().to(self.device, non_blocking=True)
        return t

    def _feed_back(self, tokens_dev: torch.Tensor, tokens, src_rows) -> None:
        rows = [i for i, t in enumerate(tokens) if t < 0]
        if not rows:
            return
        src = [src_rows[i] for i in rows]
        self._h2d += 16 * len(rows)
        tokens_dev.index_copy_(0, self._dev_index(rows), self._launch_ids.index_select(0, self._dev_index(src)))

    def _launch_tail(self, ids: torch.Tensor, local: torch.Tensor, n: int, keep_rows):
        """Greedy ids of a launched step (``greedy``) to pinned host memory behind an event; the
        full logits of the ``keep_rows`` gathered (a collective on every rank)."""
        self._launch_ids = ids
        kept = {}
        if keep_rows:
            sel = self.full_rows(local.index_select(0, self._dev_index(keep_rows)))
            kept = {r: sel[i:i + 1] for i, r in enumerate(keep_rows)}
        if self.device.type == "cuda":
            host = torch.empty(n, dtype=torch.int64).pin_memory()
            host.copy_(ids, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
        else:  # a copy: ids may be a replayed bucket's static output, which the next replay rewrites
            host, ev = ids.clone(), None
        return (host, ev, kept, n)

    def decode_collect(self, handle) -> list[int]:
        host, ev, _, n = handle
        if ev is not None:
            ev.synchronize()
        self._d2h += 8 * n
        return [int(x) for x in host.tolist()]

    def decode_kept(self, handle) -> dict:
        return handle[2]

    def decode_mixed(self, lanes, tokens, positions, prefill_calls):
        segs = [(l, [t], p) for l, t, p in zip(lanes, tokens, positions)] + list(prefill_calls)
        lg = self.forward(segs)
        n = len(lanes)
        return lg[:n], [lg[n + i:n + i + 1] for i in range(len(prefill_calls))]

    def decode_row(self, logits, row: int):
        return logits[row:row + 1]

    def decode_tokens_per_step(self) -> int:
        return 1 if self.mtp is None else self.mtp.k + 1

    @torch.inference_mode()
    def score(self, lane: int, ids: Sequence[int], continuation_start: int):
        """Logits predicting ``ids[continuation_start:]`` (rows ``continuation_start-1 ..``)."""
        rows = list(range(max(continuation_start - 1, 0), len(ids) - 1))
        if not rows:
            return torch.empty(0, self.cfg.vocab)
        return self.forward([(lane, ids, 0)], logit_rows=rows)

    def sample_batch(self, logits, temperatures: Sequence[float], generator=None) -> list[int]:
        temps = list(temperatures)
        am = ops.argmax_rows(logits)[1] if logits.shape[0] else None
        self._gpu_mark("out")
        out = am.tolist() if am is not None else []
        self._d2h += 8 * len(out)
        for i, t in enumerate(temps):
            if t and t > 0:
                p = torch.softmax(logits[i].float() / t, dim=-1)
                out[i] = int(torch.multinomial(p, 1, generator=generator).item())
        return [int(x) for x in out]

    def warmup(self) -> None:
        pass

    # ================================================================== convenience
    @torch.inference_mode()
    def generate(self, ids: Sequence[int], max_new: int, lane: int = 0, stop: Sequence[int] = ()) -> list[int]:
        """Single-sequence greedy generation on ``lane`` with private block bookkeeping
        (blocks ``1 + lane * max_blocks ..``); used by tests and examples, not by serving."""
        self.begin(lane)
        need = (len(ids) + max_new + self.block_size - 1) // self.block_size
        base = 1 + lane * self.max_blocks
        if base + need > self.num_blocks:
            raise ValueError("pool too small for generate()")
        self.attach_blocks(lane, list(range(base, base + need)))
        lg = self.prefill(lane, ids, 0)
        out: list[int] = []
        pos = len(ids)
        for _ in range(max_new):
            tok = self.sample_batch(lg, [0.0])[0]
            out.append(tok)
            if tok in stop:
                break
            lg = self.decode([lane], [tok], [pos])
            pos += 1
        return out


def env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) not in ("0", "", "false", "False")
