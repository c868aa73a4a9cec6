"""Child process of test_bounds_gpu.py: loads the debug build (QB_BOUNDS=1) and checks that
(1) a tiny-model prefill + decode leaves the status word clear (no index out of range, every
scratch canary intact) and (2) an out-of-range token id and an out-of-range lane are caught: the
status word names the site, the value and the capacity, and the access is skipped. The "out of
range" values are out of the range the kernels are told (narrowed views) but inside the memory
actually allocated, so even a kernel without the checks would touch only valid memory."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> None:
    assert os.environ.get("QB_BOUNDS") == "1"
    import torch

    from qwen35_b200.ops import _ext
    from qwen35_b200.ops import core as ops
    from qwen35_b200.serving.engine import PoolSpec, build_model

    assert "_build_bounds" in (_ext.so_path() or ""), _ext.so_path()
    ext = _ext.ext()
    dev = torch.device("cuda", 0)
    probe = torch.empty(1, device=dev)
    ext.clear_status(probe)
    # (1) normal operation: nothing recorded
    m, _ = build_model("tiny", 0, 1, dev, PoolSpec(lanes=2, max_seq=512, kv_tokens=2048, snapshots=2), graphs=False)
    out = m.generate(list(range(3, 300)), 8)
    torch.cuda.synchronize()
    st = ext.status(probe).tolist()
    assert st == [0, 0, 0, 0], st
    assert len(out) == 8
    # (2a) token id past the table the kernel is given
    V, H = 1000, 256
    big = torch.randn(V + 8, H, device=dev).bfloat16()
    tok = torch.tensor([3, V + 2], device=dev, dtype=torch.int64)
    e = ops.embed(tok, big[:V])
    torch.cuda.synchronize()
    st = ext.status(probe).tolist()
    assert st == [7, 1, V + 2, V], st
    assert torch.equal(e[0], big[3])
    ext.clear_status(probe)
    # (2b) lane past the conv state the kernel is given
    lanes, C = 3, 64
    state = torch.zeros(lanes + 2, C, 3, device=dev).bfloat16()
    x = torch.randn(5, C, device=dev).bfloat16()
    w = torch.randn(C, 4, device=dev).bfloat16()
    seg_lane = torch.tensor([lanes + 1], device=dev, dtype=torch.int32)
    cu = torch.tensor([0, 5], device=dev, dtype=torch.int32)
    ops.causal_conv_varlen(x, state[:lanes], w, seg_lane, cu, commit=True)
    torch.cuda.synchronize()
    st = ext.status(probe).tolist()
    assert st == [7, 4, lanes + 1, lanes], st
    assert state.float().abs().sum().item() == 0.0  # the state write was skipped too
    ext.clear_status(probe)
    print("bounds ok", flush=True)


if __name__ == "__main__":
    main()
