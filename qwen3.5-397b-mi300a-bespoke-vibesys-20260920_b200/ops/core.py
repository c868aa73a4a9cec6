"""Entry points of every op the model runtime issues.

CUDA tensors go to the compiled sm_100a extension (``ops._ext``; sources in ``csrc/``). If the
extension is missing on a CUDA tensor the call raises: there is no silent eager fallback.
CPU tensors use the PyTorch statements in ``ops.reference`` (hermetic tests, gloo ranks).

Varlen conventions shared by the sequence ops: the batch is a concatenation of segments; a
segment is ``cu[s]..cu[s+1]`` rows of lane ``seg_lane[s]`` whose first row is at absolute
position ``seg_start[s]``. Lane state (conv window, recurrent state, block table) is indexed by
lane. ``rows[t]`` is the physical paged-KV row of token ``t``.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import ext
from ..utils import flags


def _cuda(x: torch.Tensor) -> bool:
    return x.is_cuda


# ----------------------------------------------------------------------------- norms
def rmsnorm(x, w1p, eps):
    if _cuda(x):
        return ext().rmsnorm(x, w1p, eps)
    return ref.rmsnorm(x, w1p, eps)


def add_rmsnorm(x, residual, w1p, eps):
    """Returns (residual + x, rmsnorm(residual + x)); on CUDA the residual is updated in place."""
    if _cuda(x):
        normed = torch.empty_like(residual)
        ext().add_rmsnorm(x, residual, w1p, normed, eps)
        return residual, normed
    return ref.add_rmsnorm(x, residual, w1p, eps)


def gated_rmsnorm(x, z, w, eps):
    if _cuda(x):
        return ext().gated_rmsnorm(x, z, w, eps)
    return ref.gated_rmsnorm(x, z, w, eps)


# ----------------------------------------------------------------------------- dense
def linear(x, w, out=None):
    """``x @ w.T`` (fp32 accumulate). CUDA: tcgen05 GEMM with the weight as the M operand. ``x``
    may be the owner-only rows of a sequence-parallel all-reduce (``parallel.symm.GatheredRows``):
    then the GEMM gathers them from every rank over NVLink itself."""
    if getattr(x, "gathered", False):
        assert out is None
        return x.linear(w)
    if _cuda(x):
        return ext().linear(x, w, out)
    y = ref.linear(x, w)
    if out is not None:
        out.copy_(y)
        return out
    return y


def silu_mul(gu):
    """``silu(gu[:, :n]) * gu[:, n:]`` rounded to the input dtype."""
    if _cuda(gu):
        return ext().silu_mul(gu)
    n = gu.shape[-1] // 2
    return (F.silu(gu[..., :n].float()) * gu[..., n:].float()).to(gu.dtype)


def embed(tokens, table):
    if _cuda(tokens):
        return ext().embed(tokens, table)
    return table[tokens]


def argmax_rows(logits):
    if _cuda(logits):
        return ext().argmax_rows(logits)
    v, i = logits.float().max(dim=-1)
    return v, i


def deltanet_decode(proj, conv_state, conv_w, a_log, dt_bias, rec_state, norm_w, seg_lane, nk, nv, dk, dv, eps,
                    seg_lane_h=None):
    """DeltaNet token mixer for a batch of one token per lane, from the input projection ``proj``
    ([T, conv channels | z | b | a]) to the gated-normed heads [T, nv*dv]: causal conv + SiLU,
    q/k l2norm, gated delta step and gated RMSNorm, the lane's conv window and fp32 state
    continued and updated. One fused kernel on CUDA (dk = dv = 128, conv kernel 4); elsewhere the
    separate ops. Reference behaviour: ``deltanet_fused.py`` decode step, ``model.py:3596``."""
    if _cuda(proj) and dk == 128 and dv == 128 and conv_w.shape[1] == 4:
        return ext().deltanet_decode(proj, conv_state, conv_w, a_log, dt_bias, rec_state, norm_w, seg_lane,
                                     nk, nv, dk, dv, eps)
    t = proj.shape[0]
    c = 2 * nk * dk + nv * dv
    cu_h = list(range(t + 1))
    lanes_h = seg_lane.tolist() if seg_lane_h is None else list(seg_lane_h)
    cu = torch.arange(t + 1, dtype=torch.int32, device=proj.device)
    qkv = causal_conv_varlen(proj[:, :c], conv_state, conv_w, seg_lane, cu, lanes_h, cu_h)
    core = gated_delta_varlen(qkv, proj[:, c + nv * dv:], a_log, dt_bias, rec_state, seg_lane, cu, nk, nv, dk, dv,
                              lanes_h, cu_h)
    z = proj[:, c:c + nv * dv].reshape(t, nv, dv)
    return gated_rmsnorm(core, z, norm_w, eps).reshape(t, nv * dv)


def stamp(buf: torch.Tensor, slot: int) -> None:
    """``buf[slot]`` = the device clock (ns, ``%globaltimer``) when the stream reaches this point;
    a one-thread kernel, so it can sit inside a captured CUDA graph. On CPU: the host clock."""
    if _cuda(buf):
        ext().stamp(buf, slot)
    else:
        buf[slot] = time.perf_counter_ns()


# ----------------------------------------------------------------------------- deltanet
def causal_conv_varlen(x, conv_state, w, seg_lane, cu, seg_lane_h=None, cu_h=None, commit=True):
    """Depthwise causal conv + SiLU over each segment, continuing from ``conv_state[lane]``
    ([lanes, C, K-1]) and, when ``commit``, updating it. ``x`` [T, C] (may be a column slice)."""
    if _cuda(x):
        return ext().causal_conv_varlen(x, conv_state, w, seg_lane, cu, commit)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    lanes = seg_lane_h if seg_lane_h is not None else seg_lane.tolist()
    cus = cu_h if cu_h is not None else cu.tolist()
    for s, lane in enumerate(lanes):
        a, b = cus[s], cus[s + 1]
        if b == a:  # an empty segment leaves its lane's window as it is
            continue
        o, st = ref.causal_conv(x[a:b], conv_state[lane], w)
        out[a:b] = o
        if commit:
            conv_state[lane].copy_(st)
    return out


def gated_delta_varlen(qkv, ab, a_log, dt_bias, rec_state, seg_lane, cu, nk, nv, dk, dv,
                       seg_lane_h=None, cu_h=None, commit=True):
    """Gated delta rule over each segment with the DeltaNet glue fused in.

    ``qkv`` [T, 2*nk*dk + nv*dv] (conv output: q | k | v), ``ab`` [T, 2*nv] (``b`` then ``a``
    projections). Per row: ``beta = sigmoid(b)``, ``g = -exp(A_log) * softplus(a + dt_bias)``,
    q/k l2-normalised, ``q *= dk**-0.5``, key heads repeated to value heads. ``rec_state``
    [lanes, nv, dk, dv] fp32 is continued and updated. Returns [T, nv, dv] in ``qkv.dtype``."""
    if _cuda(qkv):
        mode = dn_prefill_mode(nv, cu_h)
        plan = dn_chunk_plan(cu_h, dk, dv, qkv.device, mode)
        if plan is not None:
            chunks, seg0 = plan
            fn = ext().gated_delta_tc if mode == "tc" else ext().gated_delta_chunked
            return fn(qkv, ab, a_log, dt_bias, rec_state, seg_lane, chunks, seg0, nk, nv, dk, dv, commit)
        return ext().gated_delta_varlen(qkv, ab, a_log, dt_bias, rec_state, seg_lane, cu, nk, nv, dk, dv, commit)
    t = qkv.shape[0]
    q = qkv[:, : nk * dk].reshape(t, nk, dk)
    k = qkv[:, nk * dk: 2 * nk * dk].reshape(t, nk, dk)
    v = qkv[:, 2 * nk * dk:].reshape(t, nv, dv).float()
    g, beta = ref.deltanet_gates(ab[:, nv:], ab[:, :nv], a_log, dt_bias)
    rep = nv // nk
    # l2norm runs in the activation dtype, as in the HF modeling code
    q = ref.l2norm(q).float().repeat_interleave(rep, dim=1) * dk ** -0.5
    k = ref.l2norm(k).float().repeat_interleave(rep, dim=1)
    out = torch.empty(t, nv, dv, dtype=torch.float32, device=qkv.device)
    lanes = seg_lane_h if seg_lane_h is not None else seg_lane.tolist()
    cus = cu_h if cu_h is not None else cu.tolist()
    for s, lane in enumerate(lanes):
        a, b = cus[s], cus[s + 1]
        o, st = ref.gated_delta_rule(q[a:b], k[a:b], v[a:b], g[a:b], beta[a:b], rec_state[lane])
        out[a:b] = o
        if commit:
            rec_state[lane].copy_(st)
    return out.to(qkv.dtype)


# ----------------------------------------------------------------------------- attention
def qk_norm_rope_kv_write(q, k, v, q_norm, k_norm, positions, rows, k_cache, v_cache, rot, theta, eps):
    """Per-head RMSNorm of q and k, partial RoPE on the first ``rot`` dims, and the paged KV
    write of (k, v) at physical ``rows``. Returns the normalised, rotated q [T, Hq, D]."""
    if _cuda(q):
        return ext().qk_norm_rope_kv_write(q, k, v, q_norm, k_norm, positions, rows, k_cache, v_cache,
                                           rot, theta, eps)
    qn = ref.rmsnorm(q, q_norm, eps)
    kn = ref.rmsnorm(k, k_norm, eps)
    cos, sin = ref.rope_cos_sin(positions, rot, theta, q.dtype)
    qn = ref.apply_partial_rope(qn, cos, sin)
    kn = ref.apply_partial_rope(kn, cos, sin)
    k_cache[rows.long()] = kn.to(k_cache.dtype)
    v_cache[rows.long()] = v.to(v_cache.dtype)
    return qn


def attention_varlen(q, k_cache, v_cache, block_table, seg_lane, cu, seg_start, block_size,
                     seg_lane_h=None, cu_h=None, seg_start_h=None, tables_h=None, positions=None, max_ctx=None,
                     causal=True):
    """Causal GQA attention of each segment's queries over its lane's paged context
    ``[0, seg_start + len)``. ``q`` [T, Hq, D]; caches [rows, Hkv, D]. Returns [T, Hq, D].
    On CUDA ``positions`` ([T] absolute positions) and ``max_ctx`` (longest context) are used.
    ``causal=False`` (the ``flip_causal_mask`` calibration fault) runs the PyTorch form with every
    key of the segment's context visible."""
    if _cuda(q) and causal:
        plan = fa_plan(q, k_cache, cu_h, block_size, max_ctx)
        if plan is not None:
            tiles, splits = plan
            return ext().attention_fa(q, k_cache, v_cache, block_table, seg_lane, positions, tiles, block_size, splits)
        return ext().attention_varlen(q, k_cache, v_cache, block_table, seg_lane, cu, positions, block_size,
                                      int(max_ctx))
    out = torch.empty_like(q)
    lanes = seg_lane_h if seg_lane_h is not None else seg_lane.tolist()
    cus = cu_h if cu_h is not None else cu.tolist()
    starts = seg_start_h if seg_start_h is not None else seg_start.tolist()
    for s, lane in enumerate(lanes):
        a, b = cus[s], cus[s + 1]
        n = starts[s] + (b - a)
        if tables_h is not None:
            blocks = tables_h[lane]
        else:
            blocks = block_table[lane].tolist()
        nb = (n + block_size - 1) // block_size
        rows = torch.tensor([blk * block_size + o for blk in blocks[:nb] for o in range(block_size)][:n],
                            dtype=torch.long, device=q.device)
        out[a:b] = ref.attention_prefix(q[a:b], k_cache[rows], v_cache[rows], starts[s], causal)
    return out


DN_CHUNK = 64
DN_CHUNK_MIN = 64
_dn_chunk_cache: dict = {}
# Device tables read by a captured CUDA graph must outlive it: entries used during a capture are
# kept here for good, the bounded caches evict only tables no graph refers to.
_captured_tables: dict = {}


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def _cache_put(cache: dict, tag: tuple, key, value) -> None:
    if _capturing():
        _captured_tables[tag + key] = value
        return
    if len(cache) >= 256:
        cache.pop(next(iter(cache)))
    cache[key] = value


DN_TC_MAX_HEADS = 32
DN_TC_MIN_TOKENS = 128


def dn_prefill_mode(nv: int, cu_h=None) -> str:
    """The DeltaNet prefill path for ``nv`` value heads on this rank (``QB_DN_PREFILL``). ``auto``:
    the tensor-core chunked form up to ``DN_TC_MAX_HEADS`` heads (from 2-way tensor parallelism
    on; at 8 heads it measured 2.5-3.3x faster than the token recurrence for 800-4096 tokens) and,
    at more heads, for batches whose longest segment has at least ``DN_TC_MIN_TOKENS`` tokens
    (64 heads: 0.95 vs 1.79 ms for 4096 tokens, 0.26 vs 0.36 for 800, 0.097 vs 0.123 for 256,
    0.061 vs 0.069 for 128; shorter segments keep the fp32 recurrence)."""
    mode = flags.get("QB_DN_PREFILL")
    if mode == "auto":
        if nv <= DN_TC_MAX_HEADS:
            return "tc"
        longest = max((cu_h[i + 1] - cu_h[i] for i in range(len(cu_h) - 1)), default=0) if cu_h else 0
        return "tc" if longest >= DN_TC_MIN_TOKENS else "recurrence"
    return mode


def dn_chunk_plan(cu_h, dk, dv, device, mode=None):
    """(device chunk table [n, 3] = (segment, first row, rows), device first-chunk index per
    segment [S + 1]) for the chunked delta rule, or None (the token-serial kernel runs).

    ``mode`` (``dn_prefill_mode``): ``tc`` runs the chunked form with the state in tensor memory
    and its products on tcgen05 (serial depth: chunks, not tokens); ``chunked_fp32`` the same
    identities on CUDA cores in fp32 (exact formulation, slower than the token kernel);
    ``recurrence`` always the fp32 token recurrence. Only batches whose longest segment reaches
    a chunk, and head size 128."""
    mode = mode or flags.get("QB_DN_PREFILL")
    if cu_h is None or dk != 128 or dv != 128 or mode not in ("tc", "chunked_fp32"):
        return None
    lens = [cu_h[i + 1] - cu_h[i] for i in range(len(cu_h) - 1)]
    if not lens or max(lens) < DN_CHUNK_MIN:
        return None
    key = (tuple(cu_h), device)
    hit = _dn_chunk_cache.get(key) or _captured_tables.get(("dn",) + key)
    if hit is None:
        rows, seg0 = [], [0]
        for s, n in enumerate(lens):
            for r in range(0, n, DN_CHUNK):
                rows.append([s, cu_h[s] + r, min(DN_CHUNK, n - r)])
            seg0.append(len(rows))
        hit = (torch.tensor(rows, dtype=torch.int32).to(device), torch.tensor(seg0, dtype=torch.int32).to(device))
        _cache_put(_dn_chunk_cache, ("dn",), key, hit)
    elif _capturing():
        _captured_tables[("dn",) + key] = hit
    return hit


_FA_SMS = 148
_fa_tiles_cache: dict = {}


def fa_plan(q, k_cache, cu_h, block_size, max_ctx):
    """(device tile list, key splits) for the tcgen05 flash-attention kernel, or None when the
    shape is outside what it supports (then the CUDA-core split-K kernel runs).

    Every tile is (segment, first row, rows) with rows <= 128 / G, so a tile's G query heads x
    rows fill the 128 MMA rows. When there are fewer (tile, kv head) CTAs than SMs (decode), each
    tile's key range is split so that one wave covers the GPU; the partials are merged by a
    second kernel. The tile tensor is cached per (segments, G): a CUDA-graph capture then reads a
    persistent device tensor instead of recording a copy from a temporary host buffer."""
    if cu_h is None or block_size != 16 or not flags.get("QB_FA"):
        return None
    g = q.shape[1] // k_cache.shape[1]
    if 128 % g or q.shape[2] not in (64, 128, 256) or len(cu_h) < 2:
        return None
    key = (tuple(cu_h), g, q.device)
    tiles = _fa_tiles_cache.get(key)
    if tiles is None:
        tiles = _captured_tables.get(("fa",) + key)
    if tiles is None:
        host = torch.tensor(fa_tiles(cu_h, g), dtype=torch.int32)
        tiles = host.to(q.device)
        _cache_put(_fa_tiles_cache, ("fa",), key, tiles)
    elif _capturing():
        _captured_tables[("fa",) + key] = tiles
    base = tiles.shape[0] * k_cache.shape[1]
    splits = 1
    forced = flags.get("QB_FA_SPLITS")
    if forced > 0:
        splits = max(1, min(forced, (int(max_ctx) + 63) // 64, 128))
    elif base < _FA_SMS:
        splits = max(1, min(_FA_SMS // base, (int(max_ctx) + 63) // 64, 128))
    return tiles, splits


def fa_tiles(cu_h, g: int) -> list[list[int]]:
    """[segment, first row, rows] per 128/g-token query tile of every segment."""
    qt = 128 // g
    out = []
    for s in range(len(cu_h) - 1):
        a, b = cu_h[s], cu_h[s + 1]
        for r in range(a, b, qt):
            out.append([s, r, min(qt, b - r)])
    return out


def sigmoid_gate_mul(x, gate):
    if _cuda(x):
        return ext().sigmoid_gate_mul(x, gate)
    return (x.float() * torch.sigmoid(gate.float())).to(x.dtype)


# ----------------------------------------------------------------------------- moe
def router_topk(logits, k):
    """Softmax / top-k / renormalise over the first ``E`` columns; returns (w [T,k] fp32,
    idx [T,k] int32)."""
    if _cuda(logits):
        return ext().router_topk(logits, k)
    w, i = ref.router_topk(logits, k)
    return w.float(), i.int()


def mx_scale_chunks(s: torch.Tensor, gate_up: bool) -> torch.Tensor:
    """Weight e8m0 scales [E, rows, K/32] -> the tensor-memory chunk layout of the block-scaled
    MMA: [E, rows/128, K/128, 512] bytes, one 512-byte chunk per (128-row weight tile, 4 K-blocks),
    line r (16 bytes) = the 4 scales of tile rows r, r+32, r+64, r+96. For gate_up a tile's rows
    are 64 gate rows followed by the matching 64 up rows (the epilogue pairs them)."""
    E, rows, kb = s.shape
    nt = rows // 128
    if gate_up:
        half = rows // 2
        t = torch.arange(nt, device=s.device)[:, None]
        r = torch.arange(128, device=s.device)[None, :]
        order = torch.where(r < 64, t * 64 + r, half + t * 64 + (r - 64)).reshape(-1)
        s = s[:, order, :]
    x = s.reshape(E, nt, 4, 32, kb // 4, 4)         # [E, tile, c, r0, k-chunk, j]
    return x.permute(0, 1, 4, 3, 2, 5).contiguous().reshape(E, nt, kb // 4, 512)


def mx_tile_codes(w: torch.Tensor, gate_up: bool) -> torch.Tensor:
    """Packed e2m1 codes [E, rows, K/2] -> the same bytes with every (128-row weight tile, 128-K
    stage) block contiguous: [E, rows/128, K/128, 128 rows, 64 bytes], returned in the original
    shape. One TMA box of the block-scaled kernel then reads 4 KB of consecutive memory instead
    of 64 rows of 64 bytes each 2 KB apart. For gate_up a tile's rows are 64 gate rows followed
    by the matching 64 up rows (as for the scale chunks)."""
    E, rows, kb2 = w.shape
    nt, ks = rows // 128, kb2 // 64
    if gate_up:
        t = w.view(E, 2, nt, 64, ks, 64).permute(0, 2, 4, 1, 3, 5)  # [E, tile, stage, gate|up, r, byte]
    else:
        t = w.view(E, nt, 128, ks, 64).permute(0, 1, 3, 2, 4)       # [E, tile, stage, r, byte]
    return t.contiguous().view(E, rows, kb2)


def prepare_experts(experts: dict, keep_rows: bool = False) -> dict:
    """Add the layouts the block-scaled CUDA path reads: chunked scales (``s13c``/``s2c``) and
    tile-contiguous codes. Without ``keep_rows`` the row-major scales are dropped and the codes
    replaced in place (``tiled``); with it (the CPU reference and the f16-decode path read the
    row-major forms) the tiled codes are kept beside them as ``w13t``/``w2t``."""
    if "s13" in experts and "s13c" not in experts and experts["s13"].is_cuda:
        experts["s13c"] = mx_scale_chunks(experts["s13"], True)
        experts["s2c"] = mx_scale_chunks(experts["s2"], False)
        if not flags.get("QB_MX_TILED"):
            if not keep_rows:
                del experts["s13"], experts["s2"]
            return experts
        w13t, w2t = mx_tile_codes(experts["w13"], True), mx_tile_codes(experts["w2"], False)
        if keep_rows:
            experts["w13t"], experts["w2t"] = w13t, w2t
        else:
            del experts["s13"], experts["s2"]
            experts["w13"], experts["w2"], experts["tiled"] = w13t, w2t, True
    return experts


def moe_impl() -> str:
    """``mx`` (block-scaled MMA, default) or ``f16`` (codes decoded to f16 by the converter warps)."""
    return flags.get("QB_MOE_IMPL")


def moe_routed(h, topw, topi, experts, first, count, shared=None, gate=None):
    """Sum of this rank's experts' weighted outputs for each row (zero for rows routed only to
    other ranks' experts). fp32 accumulation, rounded once to ``h.dtype``. With ``shared`` and
    ``gate`` (the shared expert's rows and gate logits): ``+ sigmoid(gate) * shared``, as
    ``shared_gate_combine`` gives it; the block-scaled path adds it in its combine kernel."""
    if _cuda(h):
        if "s13c" in experts and (moe_impl() == "mx" or "s13" not in experts):
            w13, w2, tiled = (experts["w13t"], experts["w2t"], True) if "w13t" in experts else \
                (experts["w13"], experts["w2"], bool(experts.get("tiled", False)))
            return ext().moe_routed_mx(h, topw, topi, w13, experts["s13c"], w2, experts["s2c"], first, count,
                                       tiled, shared, gate)
        if "s13" in experts and moe_impl() == "mx" and h.shape[1] % 128 == 0 \
                and experts["w2"].shape[2] * 2 % 128 == 0:
            prepare_experts(experts, keep_rows=True)
            return moe_routed(h, topw, topi, experts, first, count, shared, gate)
        if shared is not None:
            return shared_gate_combine(moe_routed(h, topw, topi, experts, first, count), shared, gate)
        if "s13" in experts:
            return ext().moe_routed_fp4(h, topw, topi, experts["w13"], experts["s13"], experts["w2"], experts["s2"],
                                        first, count)
        return ext().moe_routed_bf16(h, topw, topi, experts["w13"], experts["w2"], first, count)
    routed = ref.routed_experts(h, topw, topi.long(), experts, first, count)
    return routed if shared is None else shared_gate_combine(routed, shared, gate)


def shared_gate_combine(routed, shared, gate_logit):
    """``routed + sigmoid(gate_logit) * shared``."""
    if _cuda(routed):
        return ext().shared_gate_combine(routed, shared, gate_logit)
    return (routed.float() + torch.sigmoid(gate_logit.float())[:, None] * shared.float()).to(routed.dtype)
