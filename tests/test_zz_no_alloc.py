"""The allocation-free attention entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory (graph-captured regions that must not reach an
allocator, plugins inside a framework that owns all device memory, plain C callers without
PyTorch). ``qb_attention_varlen_noalloc`` serves them: its split-K scratch is a fixed device
array inside the library. This file checks it against a plain fp32 PyTorch attention (and the
regular ``attention_varlen`` entry point) on calls in a row (the scratch keeps the previous
call's contents, so the later calls show nothing stale leaks through), including the
single-split path that uses no scratch, and that bad arguments and an oversized request are
refused before launch.
It is named so that pytest collects it after every other test file.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

QB_NOALLOC_ERR_TOO_LARGE = -2
QB_NOALLOC_ERR_ARGS = -3


def _lib():
    from qwen35_b200.ops._ext import ext, so_path

    ext()  # load the extension (and its torch dependencies) into the process first
    lib = ctypes.CDLL(so_path())
    f = lib.qb_attention_varlen_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 7 + \
        [ctypes.c_void_p, ctypes.c_void_p]
    lib.qb_attention_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return lib


def _case(seed, nq=16, nkv=1, hd=256, bs=16, ctx=(5, 77, 700, 1500)):
    g = torch.Generator(device="cuda").manual_seed(seed)
    lanes = len(ctx)
    mb = max((c + bs - 1) // bs for c in ctx) + 1
    nblocks = 1 + lanes * mb
    kc = torch.randn(nblocks * bs, nkv, hd, generator=g, device="cuda").bfloat16()
    vc = torch.randn(nblocks * bs, nkv, hd, generator=g, device="cuda").bfloat16()
    perm = (torch.randperm(nblocks - 1, generator=g, device="cuda") + 1).int()
    table = perm[: lanes * mb].view(lanes, mb).contiguous()
    # lanes 0,1,3 decode one row each; lane 2 has a 3-row chunk
    segs = [(0, ctx[0] - 1, 1), (1, ctx[1] - 1, 1), (2, ctx[2] - 3, 3), (3, ctx[3] - 1, 1)]
    pos, seg_lane, cu = [], [], [0]
    for lane, st, n in segs:
        pos += list(range(st, st + n))
        seg_lane.append(lane)
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device="cuda")
    T = len(pos)
    q = torch.randn(T, nq, hd, generator=g, device="cuda").bfloat16()
    return dict(q=q, kc=kc, vc=vc, table=table, mb=mb, pos=torch.tensor(pos, **i32),
                seg_lane=torch.tensor(seg_lane, **i32), cu=torch.tensor(cu, **i32), T=T, nq=nq, nkv=nkv, hd=hd,
                bs=bs, max_ctx=max(ctx))


def _call(lib, c, out, splits):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.qb_attention_varlen_noalloc(
        c["q"].data_ptr(), c["kc"].data_ptr(), c["vc"].data_ptr(), c["table"].data_ptr(), c["mb"],
        c["pos"].data_ptr(), c["seg_lane"].data_ptr(), c["cu"].data_ptr(), c["seg_lane"].numel(), c["T"], c["nq"],
        c["nkv"], c["hd"], c["bs"], splits, out.data_ptr(), stream)


def _oracle(c):
    """Plain PyTorch fp32 attention of every query row over its lane's context, gathered from
    the paged cache through the block table (``ops.reference.attention_prefix`` on fp32 inputs)."""
    from qwen35_b200.ops.reference import attention_prefix

    out = torch.empty(c["T"], c["nq"], c["hd"], dtype=torch.float32, device="cuda")
    cu, lanes, pos = c["cu"].tolist(), c["seg_lane"].tolist(), c["pos"].tolist()
    bs = c["bs"]
    for s, lane in enumerate(lanes):
        r0, r1 = cu[s], cu[s + 1]
        ctx = pos[r1 - 1] + 1
        blocks = c["table"][lane, : (ctx + bs - 1) // bs].long()
        rows = (blocks[:, None] * bs + torch.arange(bs, device="cuda")[None]).reshape(-1)[:ctx]
        k, v = c["kc"][rows].float(), c["vc"][rows].float()
        out[r0:r1] = attention_prefix(c["q"][r0:r1].float(), k, v, pos[r0])
    return out


def test_noalloc_matches_fp32_attention_twice():
    """Two calls in a row (different data and split counts) and a single-split call, each
    against the fp32 PyTorch statement of the op; the split-K calls also equal the regular
    entry point's result."""
    from qwen35_b200.ops._ext import ext

    lib = _lib()
    assert lib.qb_attention_noalloc_scratch_bytes() == 16 << 20
    for seed, splits in ((1, 8), (2, 3), (4, 1)):
        c = _case(seed)
        out = torch.full_like(c["q"], float("nan"))
        rc = _call(lib, c, out, splits)
        assert rc == 0, rc
        torch.cuda.synchronize()
        ref = _oracle(c)
        err = (out.float() - ref).abs().max().item()
        assert err <= 2e-2 + 1e-2 * ref.abs().max().item(), (splits, err)
        exp = ext().attention_varlen(c["q"], c["kc"], c["vc"], c["table"], c["seg_lane"], c["cu"], c["pos"],
                                     c["bs"], c["max_ctx"])
        torch.cuda.synchronize()
        assert (out.float() - exp.float()).abs().max().item() <= 2e-2 + 2e-2 * exp.float().abs().max().item()


def test_noalloc_rejects_bad_arguments_without_launching():
    lib = _lib()
    c = _case(5)
    out = torch.full_like(c["q"], 7.0)
    # nq not a multiple of nkv; 32 query heads per KV head (one CTA takes 16); head_dim 96;
    # block size 0 (the checks run before any pointer is read)
    for over in ({"nq": 15, "nkv": 2}, {"nq": 32, "nkv": 1}, {"hd": 96}, {"bs": 0}):
        bad = dict(c, **over)
        assert _call(lib, bad, out, 4) == QB_NOALLOC_ERR_ARGS, over
    for splits in (0, 65):
        assert _call(lib, c, out, splits) == QB_NOALLOC_ERR_ARGS
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing ran


def test_noalloc_rejects_oversized_scratch():
    lib = _lib()
    c = _case(3)
    big_rows = (16 << 20) // (c["nq"] * 64 * (c["hd"] + 2) * 4) + 1
    c["T"] = big_rows  # rows * nq * splits * (hd + 2) * 4 bytes > 16 MiB with 64 splits
    out = torch.empty(1, device="cuda")
    assert _call(lib, c, out, 64) == QB_NOALLOC_ERR_TOO_LARGE
