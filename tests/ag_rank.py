"""One rank of the multi-GPU all-gather -> GEMM check (see test_symm_gpu.py): the owner-only
sequence-parallel all-reduce followed by the gathering GEMM against the full all-reduce followed
by the plain GEMM, over consecutive calls of different sizes (both slot parities, uneven splits)."""

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
    from qwen35_b200.parallel.symm import SymmComm

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    H = 1024
    s = SymmComm(rank, world, dev, max_rows=64, hidden=H, timeout_s=10.0, sp_rows=4096)
    g = torch.Generator(device=dev).manual_seed(200 + rank)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).float()
    W = (0.05 * torch.randn(1000, H, device=dev, generator=torch.Generator(device=dev).manual_seed(3))).bfloat16()
    dist.broadcast(w, 0)
    worst = 0.0
    for it, rows in enumerate((700, 2048, 3001, 1024, 4096, 257, 2048)):
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        base = torch.randn(rows, H, device=dev, generator=torch.Generator(device=dev).manual_seed(it)).bfloat16()
        r1, n1 = s.allreduce_add_rmsnorm(x, base.clone(), w, 1e-6, kind="sp")
        y1 = ops.linear(n1, W)
        r2, gat = s.allreduce_add_rmsnorm(x, base.clone(), w, 1e-6, kind="sp", gather_out=True)
        assert getattr(gat, "gathered", False)
        y2 = ops.linear(gat, W)
        torch.cuda.synchronize()
        per = -(-rows // world)
        a, b = min(rows, rank * per), min(rows, (rank + 1) * per)
        assert torch.equal(r1[a:b], r2[a:b]), it  # this rank's residual rows
        d = (y1.float() - y2.float()).abs().max().item()
        worst = max(worst, d)
        assert d <= 1e-2 * y1.float().abs().max().item() + 1e-3, (rows, d)
    st = ext().status(torch.empty(1, device=dev)).tolist()
    assert st[0] == 0, st
    dist.barrier()
    if rank == 0:
        print(f"ag ok world={world} worst_abs_diff={worst:.3g}", flush=True)
    s.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
