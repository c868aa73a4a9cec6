"""Host side of the prefill GEMM -> reduce-scatter fusion (CPU): which sizes take it, how the
region is sized, and that the model's deferred out projections give the same logits."""

import torch

from qwen35_b200.ops import core as ops
from qwen35_b200.parallel.comm import Comm
from qwen35_b200.parallel.symm import SymmComm


def _symm(world, max_rows=512, sp_rows=4096):
    fake = [0] * world  # bases are never dereferenced on the host
    return SymmComm(0, world, "cpu", max_rows, 4096, bases=fake, sp_rows=sp_rows, sp_bases=fake)


def test_fused_sizes_follow_the_sequence_parallel_choice():
    s2, s8 = _symm(2), _symm(8)
    assert not s2.fuses_linear(1) and not s2.fuses_linear(512)  # one-shot sizes
    assert s2.fuses_linear(513) and s2.fuses_linear(4096) and not s2.fuses_linear(4097)
    assert not s8.fuses_linear(146) and s8.fuses_linear(147)  # 147 x 7 rows > 1024
    assert not _symm(2, sp_rows=0).fuses_linear(2048)


def test_nvls_choice_by_world_size():
    from qwen35_b200.serving.engine import nvls_min_rows

    assert nvls_min_rows(-1, 8) == 1024  # measured ahead of the sequence-parallel kernel from 1024 rows
    assert nvls_min_rows(-1, 4) == 0 and nvls_min_rows(-1, 2) == 0  # never ahead at 2 and 4 ranks
    assert nvls_min_rows(0, 8) == 0 and nvls_min_rows(512, 2) == 512  # an explicit flag wins


def test_partial_slots_hold_whole_rank_ranges():
    s = _symm(8, sp_rows=1001)
    per = -(-1001 // 8)
    assert s.sp_slot_elems == per * 8 * 4096  # rows [o per, (o+1) per) of every owner fit


class _FusingComm(Comm):
    """World-1 comm that claims the fused path; runs it as projection + all-reduce."""

    def __init__(self):
        super().__init__()
        self.calls = 0

    def fuses_linear(self, rows):
        return True

    def linear_allreduce_add_rmsnorm(self, x, w, residual, w1p, eps, res_local=False):
        self.calls += 1
        return self.allreduce_add_rmsnorm(ops.linear(x, w), residual, w1p, eps, res_local=res_local)


def test_deferred_out_projection_gives_the_same_logits():
    from qwen35_b200.serving.engine import PoolSpec, build_model

    spec = PoolSpec(lanes=2, max_seq=64, kv_tokens=128)
    ids = list(range(300, 340))
    logits = []
    for comm in (None, _FusingComm()):
        m, _ = build_model("tiny", 0, 1, torch.device("cpu"), spec, dtype=torch.float32, graphs=False, comm=comm)
        m.begin(0)
        m.attach_blocks(0, [1, 2, 3])
        logits.append(m.forward([(0, ids, 0)]))
        if comm is not None:
            assert comm.calls == m.cfg.layers  # every mixer's out projection went through it
    assert torch.equal(logits[0], logits[1])
