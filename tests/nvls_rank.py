"""One rank of the multi-GPU NVLS all-reduce + add + RMSNorm check (see test_symm_gpu.py).
Exit code 3: the fabric has no multicast support (the test skips)."""

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
    H = 4096
    s = SymmComm(rank, world, dev, max_rows=256, hidden=H, timeout_s=10.0, sp_rows=4096)
    if not s.enable_nvls(rows_cap=4096, min_rows=1024):
        s.close()
        dist.destroy_process_group()
        sys.exit(3)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).float()
    dist.broadcast(w, 0)
    worst = 0.0
    # many consecutive calls (slot parity, counter targets), uneven splits over ranks
    for it, rows in enumerate((1, 7, 1000, 1024, 2048, 4095, 4096, 33, 3000, 4096, 1, 2)):
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        base = torch.randn(rows, H, device=dev, generator=torch.Generator(device=dev).manual_seed(it)).bfloat16()
        r1, n1 = s.allreduce_add_rmsnorm(x, base.clone(), w, 1e-6, kind="nvls")
        y = x.float()
        dist.all_reduce(y)
        r2, n2 = ops.add_rmsnorm(y.bfloat16(), base.clone(), w, 1e-6)
        torch.cuda.synchronize()
        # the switch sums in fp32 and returns the sum as bf16 with its own rounding: the sum may be
        # one bf16 step of itself away from NCCL's, and the residual add rounds once more
        d = (r1.float() - r2.float()).abs()
        tol = 2 ** -7 * (y.abs() + r2.float().abs()) + 1e-6
        assert bool((d <= tol).all()), (rows, d.max().item())
        worst = max(worst, d.max().item())
        assert (n1.float() - n2.float()).abs().max().item() < 2e-2 * n2.float().abs().max().item() + 1e-3
        # every rank holds identical bits
        h = torch.tensor([float(r1.float().sum()), float(n1.float().sum())], device=dev, dtype=torch.float64)
        hs = [torch.zeros_like(h) for _ in range(world)]
        dist.all_gather(hs, h)
        assert all(torch.equal(hs[0], t) for t in hs), hs
    # graph capture + replay
    x = torch.randn(2048, H, device=dev, generator=g).bfloat16()
    res = torch.zeros(2048, H, device=dev).bfloat16()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        s.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="nvls")
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        s.allreduce_add_rmsnorm(x, res, w, 1e-6, kind="nvls")
    res.zero_()
    for _ in range(4):
        gr.replay()
    torch.cuda.synchronize()
    y = x.float()
    dist.all_reduce(y)
    exp = torch.zeros(2048, H, device=dev)
    for _ in range(4):
        exp = (exp + y.bfloat16().float()).bfloat16().float()
    assert (res.float() - exp).abs().max().item() < 2e-2 * exp.abs().max().item() + 2e-2
    st_word = ext().status(torch.empty(1, device=dev)).tolist()
    assert st_word[0] == 0, st_word
    if rank == 0:
        print(f"nvls ok world={world} worst_abs_diff={worst:.3g}", flush=True)
    del gr
    s.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
