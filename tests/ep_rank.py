"""One rank of the 2-GPU expert-parallel MoE check (see test_symm_gpu.py)."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import datetime

    import torch
    import torch.distributed as dist

    from qwen35_b200.ops import core as ops
    from qwen35_b200.ops._ext import ext
    from qwen35_b200.parallel.ep import EPComm
    from qwen35_b200.utils import mxfp4

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    E, k, H, I = 32, 4, 512, 256
    g = torch.Generator(device=dev).manual_seed(7)  # the same experts on every rank
    w13, s13 = mxfp4.quantize(torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02)
    w2, s2 = mxfp4.quantize(torch.randn(E, H, I, device=dev, generator=g) * 0.02)
    full = {"w13": w13, "s13": s13, "w2": w2, "s2": s2}
    per = E // world
    mine = {"w13": w13[rank * per:(rank + 1) * per].contiguous(), "s13": s13[rank * per:(rank + 1) * per].contiguous(),
            "w2": w2[rank * per:(rank + 1) * per].contiguous(), "s2": s2[rank * per:(rank + 1) * per].contiguous()}
    ep = EPComm(rank, world, dev, cap=256, hidden=H, top_k=k, experts=E)
    gt = torch.Generator(device=dev).manual_seed(100 + rank)
    for it, T in enumerate([37 if rank == 0 else 100, 1, 256, 0 if rank == 1 else 5, 64, 64]):
        h = torch.randn(T, H, device=dev, generator=gt).bfloat16()
        tw, ti = ops.router_topk(torch.randn(T, E, device=dev, generator=gt).bfloat16(), k)
        y = ep.moe(h, tw, ti, mine)
        ref = ops.moe_routed(h, tw, ti, {kk: v.clone() for kk, v in full.items()}, 0, E)
        torch.cuda.synchronize()
        if T:
            err = (y.float() - ref.float()).abs().max().item()
            assert err <= 2e-2 * ref.float().abs().max().item() + 2e-3, (it, T, err)
    st = ext().status(torch.empty(1, device=dev)).tolist()
    assert st[0] == 0, st
    dist.barrier()
    ep.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
