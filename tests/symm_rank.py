"""One rank of the two-GPU fused all-reduce check (see test_symm_gpu.py)."""

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
    s = SymmComm(rank, world, dev, max_rows=512, hidden=H, timeout_s=10.0, sp_rows=2048)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    w = (1 + 0.1 * torch.randn(H, device=dev, generator=g)).float()
    dist.broadcast(w, 0)
    # both kernels on every size they take (odd counts split unevenly over ranks)
    cases = [(1, "auto"), (7, "auto"), (32, "auto"), (32, "sp"), (300, "oneshot"), (512, "auto"), (3, "sp"),
             (3, "auto"), (1000, "auto"), (2048, "auto"), (65, "sp"), (2047, "sp")]
    for it, (rows, kind) in enumerate(cases):
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        base = torch.randn(rows, H, device=dev, generator=torch.Generator(device=dev).manual_seed(it)).bfloat16()
        r1 = base.clone()
        r1, n1 = s.allreduce_add_rmsnorm(x, r1, w, 1e-6, kind=kind)
        y = x.float()
        dist.all_reduce(y)
        r2, n2 = ops.add_rmsnorm(y.bfloat16(), base.clone(), w, 1e-6)
        torch.cuda.synchronize()
        assert torch.equal(r1, r2), (it, (r1.float() - r2.float()).abs().max().item())
        assert (n1.float() - n2.float()).abs().max().item() < 1e-2 * n2.float().abs().max().item() + 1e-3
    # the projection fused in (GEMM -> reduce-scatter over peer memory): same bits as the
    # projection followed by the sequence-parallel kernel, over consecutive calls of both kinds
    K = 1024
    wo = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
    for it, rows in enumerate((1000, 2047, 513, 2048, 1001)):
        assert s.fuses_linear(rows), rows
        xo = torch.randn(rows, K, device=dev, generator=g).bfloat16()
        base = torch.randn(rows, H, device=dev, generator=torch.Generator(device=dev).manual_seed(50 + it)).bfloat16()
        r1, n1 = s.linear_allreduce_add_rmsnorm(xo, wo, base.clone(), w, 1e-6)
        r2, n2 = s.allreduce_add_rmsnorm(ops.linear(xo, wo), base.clone(), w, 1e-6, kind="sp")
        torch.cuda.synchronize()
        assert torch.equal(r1, r2), (rows, (r1.float() - r2.float()).abs().max().item())
        assert torch.equal(n1, n2), (rows, (n1.float() - n2.float()).abs().max().item())
    assert not s.fuses_linear(100)
    # residual kept on each rank's own rows: the normed rows equal the full gather's on every row,
    # the residual on this rank's range, over consecutive calls of both kernels
    for it, rows in enumerate((1000, 2047, 2048)):
        x = torch.randn(rows, H, device=dev, generator=g).bfloat16()
        base = torch.randn(rows, H, device=dev, generator=torch.Generator(device=dev).manual_seed(70 + it)).bfloat16()
        r1, n1 = s.allreduce_add_rmsnorm(x, base.clone(), w, 1e-6, kind="sp")
        r2, n2 = s.allreduce_add_rmsnorm(x, base.clone(), w, 1e-6, kind="sp", res_local=True)
        xo = torch.randn(rows, K, device=dev, generator=g).bfloat16()
        r3, n3 = s.linear_allreduce_add_rmsnorm(xo, wo, base.clone(), w, 1e-6)
        r4, n4 = s.linear_allreduce_add_rmsnorm(xo, wo, base.clone(), w, 1e-6, res_local=True)
        torch.cuda.synchronize()
        per = -(-rows // world)
        a, b = min(rows, rank * per), min(rows, (rank + 1) * per)
        assert torch.equal(n1, n2) and torch.equal(r1[a:b], r2[a:b]), (rows, "sp")
        assert torch.equal(n3, n4) and torch.equal(r3[a:b], r4[a:b]), (rows, "linear")
    # graph capture + replay
    x = torch.randn(16, H, device=dev, generator=g).bfloat16()
    res = torch.zeros(16, H, device=dev).bfloat16()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        s.allreduce_add_rmsnorm(x, res, w, 1e-6)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        out = s.allreduce_add_rmsnorm(x, res, w, 1e-6)
    res.zero_()
    for _ in range(5):
        gr.replay()
    torch.cuda.synchronize()
    y = x.float()
    dist.all_reduce(y)
    exp = torch.zeros(16, H, device=dev)
    for _ in range(5):
        exp = (exp + y.bfloat16().float()).bfloat16().float()
    assert (res.float() - exp).abs().max().item() < 1e-2 * exp.abs().max().item() + 1e-2
    st_word = ext().status(torch.empty(1, device=dev)).tolist()
    assert st_word[0] == 0, st_word
    del gr
    s.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
