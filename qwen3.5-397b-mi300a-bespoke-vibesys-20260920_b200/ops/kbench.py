"""Kernel micro-benchmarks at the full model's shapes, with roofline fractions.

    python -m qwen35_b200.ops.kbench [--case moe|gemm|attn_prefill|attn_decode|deltanet|model|all]
                                     [--tokens N] [--ctx N] [--lanes N] [--iters N]

Each case builds random inputs of one hot op at the Qwen3.5-397B-A17B geometry (one GPU, TP=1
shard sizes unless noted), warms up, then times ``--iters`` launches with CUDA events on the
launching stream, synchronising before and after. Inputs are far larger than the 126 MB L2
where the case is bandwidth-bound (weights, KV cache), so nothing is served from a warm L2.
Reported per case: mean time per call, achieved bytes/s and FLOP/s from the algorithmic
counts, and the fraction of the measured peaks (``MEASURED_PEAKS.json`` at the repository root
when present: STREAM-style copy bandwidth and cuBLAS bf16 GEMM throughput).

The same command with one case and a small ``--iters`` is the capture target for ncu; the
summaries under ``profiles/`` name the exact command lines.

Reference counterparts (behaviour, not code): ``mxfp4_gemv.py`` / ``moe_hip.py`` /
``prefill_moe.py`` (routed experts), ``skinny_gemm.py`` (dense GEMMs), ``varlen_prefill_attn.py``
and ``decode_attn_v2.py`` (attention), ``deltanet_fused.py`` (gated delta rule).
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import core as ops
from ._ext import ext
from ..utils import flags

HERE = os.path.dirname(os.path.abspath(__file__))
_DEFAULT_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks() -> dict:
    """Measured roofline denominators; the documented fallback when the file is absent."""
    for p in (os.path.join(HERE, "..", "..", "MEASURED_PEAKS.json"), "MEASURED_PEAKS.json"):
        if os.path.exists(p):
            with open(p) as f:
                d = json.load(f)
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(_DEFAULT_PEAKS, source="fallback")


def _time(fn, iters: int) -> float:
    """Mean milliseconds per call (CUDA events, synchronised on both sides)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _report(name: str, ms: float, bytes_: float, flops: float, pk: dict, **extra) -> dict:
    gbs = bytes_ / ms / 1e6
    tfs = flops / ms / 1e9
    row = {"case": name, "ms": round(ms, 4), "GB_s": round(gbs, 1), "TFLOP_s": round(tfs, 2),
           "hbm_frac": round(gbs / pk["hbm_gbs"], 3), "tensor_frac": round(tfs / pk["bf16_tflops"], 3),
           "peaks": pk["source"], **extra}
    print(json.dumps(row), flush=True)
    return row


def _g(seed: int) -> torch.Generator:
    return torch.Generator(device="cuda").manual_seed(seed)


def case_moe(tokens: int, iters: int, pk: dict, experts: int = 512, top_k: int = 10, hidden: int = 4096,
             inter: int = 1024) -> dict:
    """Routed MXFP4 experts (gate_up + SiLU*mul + down + weighted combine) for ``tokens`` rows
    with uniform random routing; bytes = packed weights + scales of every expert hit."""
    dev = "cuda"
    g = _g(0)
    ex = {"w13": torch.randint(0, 256, (experts, 2 * inter, hidden // 2), device=dev, dtype=torch.uint8, generator=g),
          "s13": torch.full((experts, 2 * inter, hidden // 32), 120, device=dev, dtype=torch.uint8),
          "w2": torch.randint(0, 256, (experts, hidden, inter // 2), device=dev, dtype=torch.uint8, generator=g),
          "s2": torch.full((experts, hidden, inter // 32), 120, device=dev, dtype=torch.uint8)}
    h = torch.randn(tokens, hidden, device=dev, generator=g).to(torch.bfloat16)
    lg = torch.randn(tokens, experts, device=dev, generator=g).to(torch.bfloat16)
    tw, ti = ops.router_topk(lg, top_k)
    active = int((torch.bincount(ti.flatten().long(), minlength=experts) > 0).sum())
    per_expert = (2 * inter * hidden + hidden * inter) // 2 * (1 + 1 / 16)
    probe = flags.get("QB_MX_PROBE")
    if probe:
        ops.moe_routed(h, tw, ti, ex, 0, experts)  # the experts' layouts are prepared on first use
        torch.cuda.synchronize()
        ext().mx_probe()
    ms = _time(lambda: ops.moe_routed(h, tw, ti, ex, 0, experts), iters)
    flops = 2 * tokens * top_k * 3 * hidden * inter
    extra = {}
    if probe:  # share of each single-thread role's cycles spent waiting
        p = ext().mx_probe().tolist()
        extra = {"producer_wait_free_stage": round(p[0] / max(1, p[1]), 3),
                 "mma_wait_full_stage": round(p[2] / max(1, p[3]), 3),
                 "mma_wait_accumulator": round(p[4] / max(1, p[3]), 3),
                 "producer_issue_cycles_per_stage": round(p[5] / max(1, p[7]), 1),
                 "mma_issue_cycles_per_stage": round(p[6] / max(1, p[7]), 1),
                 "producer_cycles_per_stage": round(p[1] / max(1, p[7]), 1)}
    return _report(f"moe_T{tokens}", ms, active * per_expert, flops, pk, active_experts=active, **extra)


def case_gemm(tokens: int, iters: int, pk: dict, n: int = 12288, k: int = 4096, name: str = "") -> dict:
    """Dense bf16 GEMM y = x W^T (the fused q/k/v/gate projection width at TP=1 by default)."""
    g = _g(1)
    # enough weight copies cycled (>= 4, >= 384 MB) that consecutive calls never hit a warm L2
    copies = max(4, -(-(384 << 20) // (2 * n * k)))
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn(tokens, k, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(tokens, n, device="cuda", dtype=torch.bfloat16)
    i = [0]

    def fn():
        ops.linear(x, ws[i[0] % copies], out)
        i[0] += 1

    ms = _time(fn, max(iters, copies))
    return _report(f"gemm{name}_T{tokens}_N{n}_K{k}", ms, 2 * (n * k + tokens * (k + n)), 2 * tokens * n * k, pk)


# every dense projection of the full model at TP=1: (name, N, K)
MODEL_GEMMS = (("_dn_in", 20608, 4096), ("_dn_out", 4096, 8192), ("_attn_qkv", 17408, 4096),
               ("_attn_o", 4096, 8192), ("_router", 513, 4096), ("_sh13", 2048, 4096), ("_sh2", 4096, 1024))


def case_gemm_shapes(tokens: int, iters: int, pk: dict) -> list:
    return [case_gemm(tokens, iters, pk, n, k, name) for name, n, k in MODEL_GEMMS]


def _paged_kv(lanes: int, ctx: int, nkv: int, hd: int, bs: int = 16, seed: int = 2):
    g = _g(seed)
    per = (ctx + 64 + bs - 1) // bs
    nblocks = 1 + lanes * per
    kc = torch.randn(nblocks * bs, nkv, hd, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(nblocks * bs, nkv, hd, device="cuda", generator=g).to(torch.bfloat16)
    table = (torch.arange(lanes * per, dtype=torch.int32).view(lanes, per) + 1).cuda()
    return kc, vc, table


def case_attn_prefill(tokens: int, ctx: int, iters: int, pk: dict, nq: int = 32, nkv: int = 2, hd: int = 256) -> dict:
    """One prompt chunk of ``tokens`` rows continuing ``ctx`` cached tokens (tcgen05 flash
    attention). FLOPs count the causal QK^T and PV products actually needed."""
    bs = 16
    kc, vc, table = _paged_kv(1, ctx + tokens, nkv, hd)
    q = torch.randn(tokens, nq, hd, device="cuda", generator=_g(3)).to(torch.bfloat16)
    i32 = dict(dtype=torch.int32, device="cuda")
    pos = torch.arange(ctx, ctx + tokens, **i32)
    lanes, cu, starts = [0], [0, tokens], [ctx]
    args = (torch.tensor(lanes, **i32), torch.tensor(cu, **i32), torch.tensor(starts, **i32), bs, lanes, cu, starts,
            None)
    ms = _time(lambda: ops.attention_varlen(q, kc, vc, table, *args, positions=pos, max_ctx=ctx + tokens), iters)
    keys = tokens * ctx + tokens * (tokens + 1) / 2
    flops = 4 * nq * hd * keys
    kv_bytes = 2 * (ctx + tokens) * nkv * hd * 2
    return _report(f"attn_prefill_T{tokens}_ctx{ctx}", ms, kv_bytes + 2 * q.numel() * 2, flops, pk)


def case_attn_decode(lanes: int, ctx: int, iters: int, pk: dict, nq: int = 32, nkv: int = 2, hd: int = 256) -> dict:
    """``lanes`` decode rows at context ``ctx`` each (split-K paged attention); bytes = the KV
    cache read."""
    bs = 16
    kc, vc, table = _paged_kv(lanes, ctx, nkv, hd)
    q = torch.randn(lanes, nq, hd, device="cuda", generator=_g(4)).to(torch.bfloat16)
    i32 = dict(dtype=torch.int32, device="cuda")
    pos = torch.full((lanes,), ctx - 1, **i32)
    ln, cu, st = list(range(lanes)), list(range(lanes + 1)), [ctx - 1] * lanes
    args = (torch.tensor(ln, **i32), torch.tensor(cu, **i32), torch.tensor(st, **i32), bs, ln, cu, st, None)
    ms = _time(lambda: ops.attention_varlen(q, kc, vc, table, *args, positions=pos, max_ctx=ctx), iters)
    kv_bytes = 2 * lanes * ctx * nkv * hd * 2
    return _report(f"attn_decode_B{lanes}_ctx{ctx}", ms, kv_bytes, 4 * lanes * nq * hd * ctx, pk)


def case_deltanet(tokens: int, lanes: int, iters: int, pk: dict, nk: int = 16, nv: int = 64, dk: int = 128,
                  dv: int = 128) -> dict:
    """Gated delta rule over ``lanes`` segments of ``tokens`` rows each (fp32 state
    [nv, dk, dv] per lane read and written once); FLOPs ~ 4 * dk * dv per head per row (the
    token recurrence's count; the chunked form used for long segments does more arithmetic in
    parallel). The host segment table is passed, as the model does, so routing matches it."""
    C = 2 * nk * dk + nv * dv
    g = _g(5)
    qkv = torch.randn(lanes * tokens, C, device="cuda", generator=g).to(torch.bfloat16)
    ab = torch.randn(lanes * tokens, 2 * nv, device="cuda", generator=g).to(torch.bfloat16)
    a_log = torch.log(torch.rand(nv, device="cuda", generator=g) * 15 + 1)
    dtb = torch.rand(nv, device="cuda", generator=g)
    rs = torch.randn(lanes, nv, dk, dv, device="cuda", generator=g) * 0.1
    i32 = dict(dtype=torch.int32, device="cuda")
    seg = torch.arange(lanes, **i32)
    cu = torch.arange(0, lanes * tokens + 1, tokens, **i32)
    seg_h, cu_h = list(range(lanes)), list(range(0, lanes * tokens + 1, tokens))
    ms = _time(lambda: ops.gated_delta_varlen(qkv, ab, a_log, dtb, rs, seg, cu, nk, nv, dk, dv, seg_h, cu_h), iters)
    bytes_ = 2 * rs.numel() * 4 + qkv.numel() * 2 + lanes * tokens * nv * dv * 2
    flops = 4 * lanes * tokens * nv * dk * dv
    return _report(f"deltanet_T{tokens}_B{lanes}", ms, bytes_, flops, pk)


def case_conv(tokens: int, iters: int, pk: dict) -> dict:
    """The DeltaNet causal conv + SiLU of a prefill over ``tokens`` rows of one lane: the conv
    channels (2 x 16 x 128 + 64 x 128) read as a column slice of the input projection's output
    rows, as in the model."""
    C, W = 2 * 16 * 128 + 64 * 128, 20608
    g = torch.Generator(device="cuda").manual_seed(3)
    proj = torch.randn(tokens, W, device="cuda", generator=g).to(torch.bfloat16)
    w = (0.3 * torch.randn(C, 4, device="cuda", generator=g)).to(torch.bfloat16)
    st = torch.zeros(2, C, 3, device="cuda", dtype=torch.bfloat16)
    seg = torch.tensor([0], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, tokens], dtype=torch.int32, device="cuda")
    ms = _time(lambda: ops.causal_conv_varlen(proj[:, :C], st, w, seg, cu, [0], [0, tokens], commit=False), iters)
    byts = 2 * tokens * C * 2  # inputs read once, outputs written once
    row = {"case": f"conv_T{tokens}", "ms": round(ms, 4), "GB_s": round(byts / ms / 1e6, 1),
           "hbm_frac": round(byts / ms / 1e6 / pk["hbm_gbs"], 3), "peaks": pk["source"]}
    print(json.dumps(row), flush=True)
    return row


def case_deltanet_decode(lanes: int, iters: int, pk: dict, nk: int = 16, nv: int = 64, dk: int = 128,
                         dv: int = 128, layers: int = 8) -> dict:
    """The fused one-token-per-lane DeltaNet mixer (conv, l2norm, gated delta step, gated
    RMSNorm) from the input projection's output. ``layers`` distinct state pools are cycled so
    that every call streams its lanes' fp32 states from HBM (as consecutive layers do); bytes =
    state read + write, conv windows, projection row in, normed row out."""
    C = 2 * nk * dk + nv * dv
    g = _g(6)
    proj = torch.randn(lanes, C + nv * dv + 2 * nv, device="cuda", generator=g).to(torch.bfloat16)
    conv_w = (0.3 * torch.randn(C, 4, device="cuda", generator=g)).to(torch.bfloat16)
    a_log = torch.log(torch.rand(nv, device="cuda", generator=g) * 15 + 1)
    dtb = torch.rand(nv, device="cuda", generator=g)
    norm_w = torch.ones(dv, device="cuda", dtype=torch.bfloat16)
    pools = [(torch.randn(lanes, C, 3, device="cuda", generator=g).to(torch.bfloat16),
              0.1 * torch.randn(lanes, nv, dk, dv, device="cuda", generator=g)) for _ in range(layers)]
    seg = torch.arange(lanes, dtype=torch.int32, device="cuda")
    i = [0]

    def fn():
        cs, rs = pools[i[0] % layers]
        ops.deltanet_decode(proj, cs, conv_w, a_log, dtb, rs, norm_w, seg, nk, nv, dk, dv, 1e-6)
        i[0] += 1

    ms = _time(fn, max(iters, layers))
    bytes_ = 2 * lanes * nv * dk * dv * 4 + 2 * lanes * C * 3 * 2 + proj.numel() * 2 + lanes * nv * dv * 2
    return _report(f"deltanet_decode_B{lanes}", ms, bytes_, 4 * lanes * nv * dk * dv, pk)


def case_model(tokens: int, ctx: int, lanes: int = 32, shard: int = 1) -> dict:
    """Whole-model steps at the full geometry on one GPU (random weights; experts of the first
    layers reused by the rest, as the one-GPU benchmark does): one prefill of ``tokens`` new
    tokens continuing ``ctx`` cached ones, and one ``lanes``-row decode step at context
    ``max(ctx, 2048)``. Prints the step times (CUDA events) and the per-kernel share of device
    time (torch profiler, a separate run). Every decode lane feeds the same token id, so the
    routed experts of a decode step are those of one token (ten per layer): the step is a lower
    bound of a chat decode step, whose distinct tokens reach ~240 experts per layer.

    ``shard`` N > 1: rank 0's shard of N-way tensor + expert parallelism (its heads, its expert
    range, its vocabulary slice, all layers' experts distinct) on this one GPU with every
    collective replaced by the local identity: the per-rank compute of an N-GPU step, without
    its NVLink traffic (``parallel.bench_collectives`` times that part)."""
    import collections

    from ..parallel.comm import Comm
    from ..serving.engine import PoolSpec, build_model

    dev = torch.device("cuda", 0)
    spec = PoolSpec(lanes=lanes + 1, max_seq=16384, kv_tokens=(lanes + 1) * 9600, snapshots=8)  # + pad lane
    m, _ = build_model("full", 0, shard, dev, spec, graphs=False, comm=Comm() if shard > 1 else None)
    per = 600
    for lane in range(lanes):
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + lane * per, 1 + (lane + 1) * per)))
    ids = [(i * 7919) % 150000 for i in range(tokens)]
    res = {}

    def prefill():
        m.forward([(0, ids, ctx)])

    def decode():
        m.decode(list(range(lanes)), [5] * lanes, [max(ctx, 2048) + lane for lane in range(lanes)])

    for f in (prefill, decode):
        ms = _time(f, 1)
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            f()
            torch.cuda.synchronize()
        agg = collections.defaultdict(lambda: [0, 0.0])
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                agg[ev.name.split("(")[0][:60]][0] += 1
                agg[ev.name.split("(")[0][:60]][1] += getattr(ev, "device_time_total", 0.0)
        tot = sum(v[1] for v in agg.values()) or 1.0
        top = sorted(agg.items(), key=lambda kv: -kv[1][1])[:20]
        # kernel_ms: the step's kernels back to back; ms - kernel_ms: device idle inside the step
        # (host launch cost the GPU waited for)
        row = {"case": f"model_{f.__name__}", "shard": shard, "tokens": tokens if f is prefill else lanes,
               "ctx": ctx, "ms": round(ms, 2), "kernel_ms": round(tot / 1e3, 2),
               "launches": sum(n for n, _ in agg.values()),
               "kernels": [(k, n, round(t / tot, 3), round(t / 1e3, 3)) for k, (n, t) in top]}
        print(json.dumps(row), flush=True)
        res[f.__name__] = row
    # the same decode step replayed from a CUDA graph, and its per-part device time from clock
    # stamps inside a separate diagnostic capture
    from ..serving.graphs import GraphRunner

    g = GraphRunner(m, buckets=(lanes,))
    g.prepare()
    for lane in range(lanes):  # capture and validation ran on reset lanes: attach the blocks again
        m.begin(lane)
        m.attach_blocks(lane, list(range(1 + lane * per, 1 + (lane + 1) * per)))
    pos = [max(ctx, 2048) + lane for lane in range(lanes)]
    ms = _time(lambda: g.decode(list(range(lanes)), [5] * lanes, pos), 5)
    replay_ms = _time(lambda: g._b[lanes].graph.replay(), 5) if lanes in g._b else None
    att = g.attribution(lanes, replays=5)
    tot = att.get("total", 0.0) or 1.0
    row = {"case": "model_decode_graph", "lanes": lanes, "ctx": max(ctx, 2048), "ms": round(ms, 2),
           "replay_ms": round(replay_ms, 2) if replay_ms is not None else None,
           "parts_ms": {k: round(v, 3) for k, v in sorted(att.items())},
           "parts_share": {k: round(v / tot, 3) for k, v in sorted(att.items()) if k != "total"}}
    print(json.dumps(row), flush=True)
    res["decode_graph"] = row
    att = g.attribution(lanes, replays=5, detail=True)
    row = {"case": "model_decode_graph_detail", "lanes": lanes,
           "parts_ms": {k: round(v, 3) for k, v in sorted(att.items(), key=lambda kv: -kv[1])}}
    print(json.dumps(row), flush=True)
    g.release()
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all",
                    choices=["moe", "gemm", "gemm_shapes", "attn_prefill", "attn_decode", "deltanet",
                             "deltanet_decode", "model", "conv", "all"])
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--lanes", type=int, default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--shard", type=int, default=1,
                    help="model case: time rank 0's shard of N-way parallelism on this GPU (collectives local)")
    ap.add_argument("--heads", type=int, nargs=2, default=None, metavar=("NK", "NV"),
                    help="deltanet cases: key and value heads (default the full geometry's 16 64; one "
                         "rank of N-way tensor parallelism has 16/N and 64/N)")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("kbench needs a CUDA device")
    pk = peaks()
    run = []
    if a.case in ("moe", "all"):
        for t in ([a.tokens] if a.tokens else [32, 800, 2048]):
            run.append(case_moe(t, a.iters, pk))
    if a.case in ("gemm", "all"):
        for t in ([a.tokens] if a.tokens else [32, 2048]):
            run.append(case_gemm(t, a.iters, pk))
    if a.case == "gemm_shapes":
        for t in ([a.tokens] if a.tokens else [1, 32, 800]):
            run.extend(case_gemm_shapes(t, a.iters, pk))
    if a.case in ("attn_prefill", "all"):
        run.append(case_attn_prefill(a.tokens or 800, a.ctx if a.ctx is not None else 6000, a.iters, pk))
    if a.case in ("attn_decode", "all"):
        run.append(case_attn_decode(a.lanes or 32, a.ctx or 6000, a.iters, pk))
    if a.case == "conv":
        return [case_conv(a.tokens or 2048, a.iters, pk)]
    if a.case == "model":
        return case_model(a.tokens or 800, a.ctx if a.ctx is not None else 6000, a.lanes or 32, a.shard)
    if a.case in ("deltanet_decode", "all"):
        run.append(case_deltanet_decode(a.lanes or 32, a.iters, pk))
    if a.case in ("deltanet", "all"):
        hk = dict(nk=a.heads[0], nv=a.heads[1]) if a.heads else {}
        run.append(case_deltanet(a.tokens or 1, a.lanes or 32, a.iters, pk, **hk))
        if a.case == "all":
            run.append(case_deltanet(800, 1, a.iters, pk))
    return run


if __name__ == "__main__":
    main()
