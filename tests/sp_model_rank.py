"""One rank of the two-GPU check that the tiny model's prefill gives the same logits with the
out projections fused into the sequence-parallel all-reduce as without (see test_symm_gpu.py)."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), QB_SYMM_MAX_ROWS="256", QB_SP_MAX_ROWS="2048")
    import datetime

    import torch
    import torch.distributed as dist

    from qwen35_b200.ops._ext import ext
    from qwen35_b200.serving.engine import PoolSpec, build_model

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    m, _ = build_model("tiny", rank, world, dev, PoolSpec(lanes=2, max_seq=2048, kv_tokens=4096), graphs=False)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(10, 4000, (1500,), generator=g).tolist()
    out = {}
    # (out projection fused into the reduce-scatter, all-gather fused into the next input projection,
    # residual kept on each rank's own rows)
    modes = ((False, False, False), (True, False, False), (True, True, False), (False, True, False),
             (True, False, True), (False, False, True), (True, True, True))
    for fused, ag, rl in modes:
        m.comm.sp_gemm, m.comm.ag_gemm, m.comm.sp_res_local = fused, ag, rl
        assert m.comm.fuses_linear(len(ids)) == fused
        m.begin(0)
        m.attach_blocks(0, list(range(1, 1 + (len(ids) + 15) // 16)))
        out[(fused, ag, rl)] = m.forward([(0, ids, 0)]).clone()
        # a decode step after it (one-shot path, the fused flags do not apply)
        out[(fused, ag, rl, "d")] = m.forward([(0, [int(out[(fused, ag, rl)].argmax())], len(ids))]).clone()
    torch.cuda.synchronize()
    base = out[(False, False, False)]
    for fused, ag, rl in modes[1:]:
        got = out[(fused, ag, rl)]
        if ag:  # the gathering GEMM tiles tokens per owner: same products, equal up to accumulation
            assert (got.float() - base.float()).abs().max().item() <= 2e-2 * base.float().abs().max().item(), \
                (fused, ag, rl)
        else:  # fewer copies, the same arithmetic: the same bits
            assert torch.equal(base, got), ((fused, ag, rl), (base - got).abs().max().item())
            assert torch.equal(out[(False, False, False, "d")], out[(fused, ag, rl, "d")])
    assert ext().status(torch.empty(1, device=dev)).tolist()[0] == 0
    m.comm.symm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]))
