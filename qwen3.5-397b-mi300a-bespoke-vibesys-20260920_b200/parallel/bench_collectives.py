"""Fused-collective sweep: all-reduce + residual + RMSNorm at hidden 4096 over token counts:
the one-shot peer-memory kernel, the sequence-parallel kernel (reduce-scatter + add + RMSNorm +
all-gather), the automatic choice between them (`fused`), and NCCL all-reduce (fp32) followed by
the add+norm kernel.

    torchrun --nproc-per-node N -m qwen35_b200.parallel.bench_collectives [--tokens 1 16 ...]

Times each variant with CUDA events over many back-to-back calls (max over ranks), and reports
microseconds per call, bus bandwidth (2 (N-1)/N x bytes / time, the NCCL convention) and the
fraction of the NVLink roofline of `fused`: an all-reduce without in-switch reduction must move
2 (N-1)/N x the message bytes through every GPU's links, at 770 GB/s measured per-direction
peer bandwidth. `nvls` (when the fabric has multicast): the switch-reduced kernel, whose
roofline is (1 + 1/N) x the message bytes into every GPU (its reduced rows, then every result
row).

``--case ep``: expert-parallel MoE (dispatch -> block-scaled expert GEMMs -> combine over peer
memory, ``parallel.ep``) at the full geometry (512 experts top-10, hidden 4096, expert width
1024, random MXFP4 codes, uniform random routing) against the replicated form the tensor-parallel
model uses (NCCL all-gather of the tokens, every rank's experts on all tokens, NCCL reduce-scatter
of the partial sums). Roofline of a call: the slower of this rank's active expert weights over
HBM (measured copy bandwidth) and its dispatch + combine bytes over NVLink (770 GB/s).

``--case ag_gemm``: the all-reduce after the MoE with the next layer's input projection: the
owner-only all-reduce + the GEMM that gathers the rows over NVLink itself, against the full
sequence-parallel all-reduce + plain GEMM and NCCL + GEMM.

``--case sp_gemm``: the prefill out-projection (o_proj, K = 8192 / N per rank) with its
all-reduce + residual + RMSNorm: the fused GEMM -> reduce-scatter (the GEMM epilogue stores rows
into their owners' symmetric slots, then the sequence-parallel kernel reduces and gathers)
against the GEMM followed by the sequence-parallel kernel and by NCCL. Roofline of a call: the
slower of the GEMM's FLOPs at the measured bf16 peak and the 3 (N-1)/N x message bytes every GPU
takes in over NVLink (partials, then the result rows) at 770 GB/s.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def ep_sweep(args, rank, world, dev) -> list[dict]:
    from ..ops import core as ops
    from ..ops.kbench import peaks
    from .ep import EPComm

    E, k, H, I = 512, 10, args.hidden, 1024
    per = E // world
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    u8 = dict(dtype=torch.uint8, device=dev)
    experts = {"w13": torch.randint(0, 256, (per, 2 * I, H // 2), generator=g, **u8),
               "s13": torch.full((per, 2 * I, H // 32), 120, **u8),
               "w2": torch.randint(0, 256, (per, H, I // 2), generator=g, **u8),
               "s2": torch.full((per, H, I // 32), 120, **u8)}
    ops.prepare_experts(experts)
    cap = max(max(args.tokens) // world, 1)
    ep = EPComm(rank, world, dev, cap=cap, hidden=H, top_k=k, experts=E)
    hbm = peaks()["hbm_gbs"]
    rows = []
    for N in args.tokens:
        T = max(N // world, 1)
        h = torch.randn(T, H, device=dev, generator=g).bfloat16()
        tw, ti = ops.router_topk(torch.randn(T, E, device=dev, generator=g).bfloat16(), k)

        def ep_call():
            ep.moe(h, tw, ti, experts)

        def replicated():
            hs = torch.empty(T * world, H, device=dev, dtype=torch.bfloat16)
            dist.all_gather_into_tensor(hs, h)
            ws = torch.empty(T * world, k, device=dev)
            dist.all_gather_into_tensor(ws, tw)
            iss = torch.empty(T * world, k, device=dev, dtype=torch.int32)
            dist.all_gather_into_tensor(iss, ti)
            y = ops.moe_routed(hs, ws, iss, experts, rank * per, per).float()
            out = torch.empty(T, H, device=dev)
            dist.reduce_scatter_tensor(out, y)

        out = {"case": "ep", "tokens": T * world, "tokens_per_rank": T, "n_gpus": world}
        for name, fn in (("ep", ep_call), ("replicated", replicated)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.ep_iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = torch.tensor([s.elapsed_time(e) * 1e3 / args.ep_iters], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            out[name + "_us"] = round(us.item(), 1)
        # bytes: rows this rank sends to other ranks (dispatch) and reads back (combine)
        owner = ti.long() // per
        sent = sum(int(((owner == d).any(dim=1)).sum()) for d in range(world) if d != rank)
        link_bytes = 2 * sent * H * 2
        # this rank's active experts: any token of any rank may route to them (uniform routing)
        hits = torch.zeros(E, dtype=torch.int64, device=dev)
        ti_all = torch.empty(T * world, k, device=dev, dtype=torch.int32)
        dist.all_gather_into_tensor(ti_all, ti)
        hits.index_add_(0, ti_all.long().flatten(), torch.ones(ti_all.numel(), dtype=torch.int64, device=dev))
        active = int((hits[rank * per:(rank + 1) * per] > 0).sum())
        wbytes = active * (3 * H * I // 2) * (1 + 1 / 16)
        roof_us = max(wbytes / (hbm * 1e3), link_bytes / (PEER_GBS * 1e3))
        out.update(link_bytes=link_bytes, active_experts=active, roofline_us=round(roof_us, 1),
                   ep_busbw_gbs=round(link_bytes / out["ep_us"] / 1e3, 1),
                   ep_frac_of_roofline=round(roof_us / out["ep_us"], 3))
        rows.append(out)
    ep.close()
    return rows


def sp_gemm_sweep(args, rank, world, dev) -> list[dict]:
    from ..ops import core as ops
    from ..ops.kbench import peaks
    from .symm import SymmComm

    H, K = args.hidden, 8192 // world
    tokens = [t for t in args.tokens if t % world == 0]
    symm = SymmComm(rank, world, dev, max_rows=512, hidden=H, sp_rows=max(tokens))
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    wo = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
    w = torch.ones(H, device=dev)
    tflops = peaks()["bf16_tflops"]
    rows = []
    for T in tokens:
        x = torch.randn(T, K, device=dev, generator=g).bfloat16()
        res = torch.zeros(T, H, device=dev).bfloat16()

        def fused():
            symm.linear_allreduce_add_rmsnorm(x, wo, res, w, 1e-6)

        def gemm_sp():
            symm.allreduce_add_rmsnorm(ops.linear(x, wo), res, w, 1e-6, kind="sp")

        def gemm_nccl():
            y = ops.linear(x, wo).float()
            dist.all_reduce(y)
            ops.add_rmsnorm(y.bfloat16(), res, w, 1e-6)

        def gemm():
            ops.linear(x, wo)

        out = {"case": "sp_gemm", "tokens": T, "K": K, "n_gpus": world, "fused_path": symm.fuses_linear(T)}
        for name, fn in (("fused", fused), ("gemm_sp", gemm_sp), ("gemm_nccl", gemm_nccl), ("gemm_only", gemm)):
            for _ in range(5):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.ep_iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = torch.tensor([s.elapsed_time(e) * 1e3 / args.ep_iters], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            out[name + "_us"] = round(us.item(), 1)
        link_bytes = 3 * (world - 1) / world * T * H * 2
        roof_us = max(2 * T * H * K / (tflops * 1e6), link_bytes / (PEER_GBS * 1e3))
        out.update(roofline_us=round(roof_us, 1), fused_frac_of_roofline=round(roof_us / out["fused_us"], 3))
        rows.append(out)
    symm.close()
    return rows


def ag_gemm_sweep(args, rank, world, dev) -> list[dict]:
    """All-reduce + add + RMSNorm followed by the next layer's input projection (DeltaNet in_proj,
    K = hidden, N = its 20608 output columns / N ranks): the owner-only all-reduce with the
    gathering GEMM (rows pulled over NVLink inside the GEMM) against the full sequence-parallel
    all-reduce (push all-gather) + the plain GEMM, and NCCL all-reduce + norm + GEMM."""
    from ..ops import core as ops
    from ..ops.kbench import peaks
    from .symm import SymmComm

    H = args.hidden
    N = (20608 // world + 127) // 128 * 128
    tokens = list(args.tokens)
    symm = SymmComm(rank, world, dev, max_rows=512, hidden=H, sp_rows=max(tokens))
    g = torch.Generator(device=dev).manual_seed(9 + rank)
    wi = (torch.randn(N, H, device=dev, generator=g) * 0.02).bfloat16()
    w = torch.ones(H, device=dev)
    tflops = peaks()["bf16_tflops"]
    rows = []
    for T in tokens:
        x = torch.randn(T, H, device=dev, generator=g).bfloat16()
        res = torch.zeros(T, H, device=dev).bfloat16()

        def fused():
            _, gat = symm.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="sp", gather_out=True)
            ops.linear(gat, wi)

        def sp_then_gemm():
            _, h = symm.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="sp")
            ops.linear(h, wi)

        def nccl_then_gemm():
            y = x.float()
            dist.all_reduce(y)
            _, h = ops.add_rmsnorm(y.bfloat16(), res, w, 1e-6)
            ops.linear(h, wi)

        def gemm():
            ops.linear(x, wi)

        out = {"case": "ag_gemm", "tokens": T, "N": N, "n_gpus": world}
        for name, fn in (("fused", fused), ("sp_gemm", sp_then_gemm), ("nccl_gemm", nccl_then_gemm),
                         ("gemm_only", gemm)):
            for _ in range(5):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.ep_iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = torch.tensor([s.elapsed_time(e) * 1e3 / args.ep_iters], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            out[name + "_us"] = round(us.item(), 1)
        # bytes into each GPU over NVLink: its share of the reduce-scatter and the gathered rows
        link_bytes = 2 * (world - 1) / world * T * H * 2
        roof_us = max(2 * T * H * N / (tflops * 1e6), link_bytes / (PEER_GBS * 1e3))
        out.update(roofline_us=round(roof_us, 1), fused_frac_of_roofline=round(roof_us / out["fused_us"], 3))
        rows.append(out)
    symm.close()
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=[1, 4, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096])
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--case", default="allreduce", choices=["allreduce", "ep", "sp_gemm", "ag_gemm"])
    ap.add_argument("--ep-iters", type=int, default=20)
    args = ap.parse_args()
    from ..ops import core as ops
    from . import comm as commmod
    from .symm import SymmComm

    rank, world = commmod.init("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    if args.case in ("ep", "sp_gemm", "ag_gemm"):
        if args.tokens == ap.get_default("tokens"):
            args.tokens = [8, 64, 512, 2048, 8192] if args.case == "ep" else [1024, 2048, 4096, 8192, 16384]
        rows = {"ep": ep_sweep, "sp_gemm": sp_gemm_sweep, "ag_gemm": ag_gemm_sweep}[args.case](args, rank, world, dev)
        if rank == 0:
            for r in rows:
                print(json.dumps(r))
        dist.destroy_process_group()
        return
    H = args.hidden
    symm = SymmComm(rank, world, dev, max_rows=min(512, max(args.tokens)), hidden=H, sp_rows=max(args.tokens))
    have_nvls = symm.enable_nvls(rows_cap=max(args.tokens), min_rows=1 << 30)  # only when asked by kind
    w = torch.ones(H, device=dev)
    rows_out = []
    for T in args.tokens:
        x = torch.randn(T, H, device=dev).bfloat16()
        res = torch.zeros(T, H, device=dev).bfloat16()

        def fused():
            symm.allreduce_add_rmsnorm(x, res, w, 1e-6)

        def oneshot():
            symm.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="oneshot")

        def sp():
            symm.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="sp")

        def nccl():
            y = x.float()
            dist.all_reduce(y)
            ops.add_rmsnorm(y.bfloat16(), res, w, 1e-6)

        def nvls():
            symm.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="nvls")

        out = {"tokens": T, "bytes": T * H * 2}
        variants = [("fused", fused), ("nccl", nccl), ("sp", sp)]
        if have_nvls:
            variants.append(("nvls", nvls))
        if T <= symm.max_rows:
            variants.append(("oneshot", oneshot))
        for name, fn in variants:
            for _ in range(10):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = torch.tensor([s.elapsed_time(e) * 1e3 / args.iters], device=dev)
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            us = us.item()
            b = T * H * 2
            out[name + "_us"] = round(us, 2)
            out[name + "_busbw_gbs"] = round(2 * (world - 1) / world * b / us / 1e3, 1)
        # bytes every rank must move for an all-reduce without in-switch reduction: 2 (W-1)/W x payload
        roof_us = 2 * (world - 1) / world * out["bytes"] / (PEER_GBS * 1e3)
        out["roofline_us"] = round(roof_us, 2)
        out["fused_frac_of_roofline"] = round(roof_us / out["fused_us"], 3)
        if have_nvls:  # with in-switch reduction a GPU takes in its reduced rows and every result row
            nv_roof = (1 + 1 / world) * out["bytes"] / (PEER_GBS * 1e3)
            out["nvls_roofline_us"] = round(nv_roof, 2)
            out["nvls_frac_of_roofline"] = round(nv_roof / out["nvls_us"], 3)
        rows_out.append(out)
    if rank == 0:
        for r in rows_out:
            print(json.dumps(r))
    symm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
