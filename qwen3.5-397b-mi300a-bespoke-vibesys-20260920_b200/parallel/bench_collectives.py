"""Fused-collective sweep: all-reduce + residual + RMSNorm at hidden 4096 over token counts:
the one-shot peer-memory kernel, the sequence-parallel kernel (reduce-scatter + add + RMSNorm +
all-gather), the automatic choice between them (`fused`), and NCCL all-reduce (fp32) followed by
the add+norm kernel.

    torchrun --nproc-per-node N -m qwen35_b200.parallel.bench_collectives [--tokens 1 16 ...]

Times each variant with CUDA events over many back-to-back calls (max over ranks), and reports
microseconds per call, bus bandwidth (2 (N-1)/N x bytes / time, the NCCL convention) and the
fraction of the NVLink roofline of `fused`: an all-reduce without in-switch reduction must move
2 (N-1)/N x the message bytes through every GPU's links, at 770 GB/s measured per-direction
peer bandwidth.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=[1, 4, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096])
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--hidden", type=int, default=4096)
    args = ap.parse_args()
    from ..ops import core as ops
    from . import comm as commmod
    from .symm import SymmComm

    rank, world = commmod.init("nccl")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    H = args.hidden
    symm = SymmComm(rank, world, dev, max_rows=min(512, max(args.tokens)), hidden=H, sp_rows=max(args.tokens))
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

        out = {"tokens": T, "bytes": T * H * 2}
        variants = [("fused", fused), ("nccl", nccl), ("sp", sp)]
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
        rows_out.append(out)
    if rank == 0:
        for r in rows_out:
            print(json.dumps(r))
    symm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
