"""Every sm_100a kernel against the plain PyTorch fp32 statement of the same op (``ops.reference``)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from qwen35_b200.ops import core as ops  # noqa: E402
from qwen35_b200.ops import reference as ref  # noqa: E402
from qwen35_b200.ops._ext import ext  # noqa: E402
from qwen35_b200.utils import mxfp4  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16


def rnd(*shape, scale=1.0, dtype=BF, seed=None):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed if seed is not None else hash(shape) % 10007)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(dtype)


def close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    tol = atol + rtol * b.abs().max().item()
    assert err <= tol, f"max err {err} > {tol}"


def status_ok():
    st = ext().status(torch.empty(1, device=DEV))
    assert int(st.abs().sum()) == 0, st.tolist()


@pytest.mark.parametrize("T,N,K", [(1, 128, 64), (7, 200, 256), (16, 384, 4096), (33, 256, 512), (100, 1024, 1024),
                                   (300, 640, 4096), (1000, 256, 128), (64, 4096, 4096), (800, 384, 1024),
                                   (513, 256, 512)])
def test_linear(T, N, K):
    x = rnd(T, K, scale=1.0, seed=T)
    w = rnd(N, K, scale=0.05, seed=N + K)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    close(y, x.float() @ w.float().t(), rtol=1e-2, atol=1e-2)
    status_ok()


@pytest.mark.parametrize("T,N,K", [(32, 20608, 4096), (32, 4096, 8192), (32, 513, 4096), (1, 2048, 4096),
                                   (17, 4096, 1024), (64, 1000, 2048)])
def test_linear_streamk(T, N, K):
    """Decode shapes whose tiles do not divide over the SMs: stream-K partials and their fixup,
    three calls in a row (the arrival counters re-arm themselves) and a graph replay."""
    x = rnd(T, K, scale=1.0, seed=T + 1)
    w = rnd(N, K, scale=0.05, seed=N)
    ref = x.float() @ w.float().t()
    for _ in range(3):
        y = ops.linear(x, w)
        torch.cuda.synchronize()
        close(y, ref, rtol=1e-2, atol=1e-2)
    out = torch.empty(T, N, dtype=BF, device=DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.linear(x, w, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.linear(x, w, out=out)
    out.zero_()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    close(out, ref, rtol=1e-2, atol=1e-2)
    status_ok()


def test_linear_strided_input_and_output():
    base = rnd(40, 512, seed=3)
    x = base[:, 128:384]  # row stride 512, 256 columns
    w = rnd(192, 256, scale=0.05, seed=4)
    out = torch.zeros(40, 320, dtype=BF, device=DEV)
    ops.linear(x, w, out=out[:, 64:256])
    torch.cuda.synchronize()
    close(out[:, 64:256], x.float() @ w.float().t(), rtol=1e-2, atol=1e-2)
    assert out[:, :64].abs().sum() == 0 and out[:, 256:].abs().sum() == 0


def test_norms_and_glue():
    x = rnd(37, 4096, seed=1)
    res = rnd(37, 4096, seed=2)
    w = (1 + 0.1 * torch.randn(4096, device=DEV)).float()
    close(ops.rmsnorm(x, w, 1e-6), ref.rmsnorm(x, w, 1e-6))
    r0 = res.clone()
    r1, n1 = ops.add_rmsnorm(x, r0, w, 1e-6)
    rr, nn = ref.add_rmsnorm(x, res, w, 1e-6)
    close(r1, rr, atol=1e-2)
    close(n1, nn)
    core = rnd(37, 8, 128, seed=5)
    zz = rnd(37, 8 * 128 + 64, seed=6)[:, :8 * 128].reshape(37, 8, 128)
    gw = rnd(128, seed=7)
    close(ops.gated_rmsnorm(core, zz, gw, 1e-6), ref.gated_rmsnorm(core, zz, gw, 1e-6))
    gu = rnd(9, 2 * 1024, seed=8)
    close(ops.silu_mul(gu), torch.nn.functional.silu(gu[:, :1024].float()) * gu[:, 1024:].float())
    g = rnd(9, 2048, seed=9)
    y = rnd(9, 1024, seed=10)
    close(ops.sigmoid_gate_mul(y, g[:, :1024]), y.float() * torch.sigmoid(g[:, :1024].float()))
    rl = rnd(9, 4096, seed=11)
    sh = rnd(9, 4096, seed=12)
    gl = rnd(9, 513, seed=13)
    close(ops.shared_gate_combine(rl, sh, gl[:, 512]), rl.float() + torch.sigmoid(gl[:, 512:513].float()) * sh.float())
    status_ok()


def test_embed_argmax():
    table = rnd(1000, 256, seed=14)
    tok = torch.randint(0, 1000, (33,), device=DEV)
    assert torch.equal(ops.embed(tok, table), table[tok])
    lg = rnd(5, 248320, seed=15)
    v, i = ops.argmax_rows(lg)
    assert torch.equal(i, lg.float().argmax(-1))
    lg2 = lg.float()
    lg2[:, 7] = 1e9
    lg2[:, 9] = 1e9
    assert ops.argmax_rows(lg2)[1].tolist() == [7] * 5  # ties -> lowest index


@pytest.mark.parametrize("E,k", [(512, 10), (32, 4)])
def test_router_topk(E, k):
    lg = rnd(50, E + 1, seed=E)
    w, i = ops.router_topk(lg[:, :E], k)
    rw, ri = ref.router_topk(lg[:, :E], k)
    assert torch.equal(i.long().sort(-1).values, ri.sort(-1).values)
    close(w.sort(-1).values, rw.float().sort(-1).values, atol=1e-2)


@pytest.mark.parametrize("nq,nkv,hd,rot", [(8, 1, 256, 64), (32, 2, 256, 64), (2, 1, 64, 16)])
def test_qk_norm_rope_kv_write(nq, nkv, hd, rot):
    T = 11
    qkv = rnd(T, nq * 2 * hd + 2 * nkv * hd, seed=hd)
    qg = qkv[:, : nq * 2 * hd].reshape(T, nq, 2 * hd)
    q = qg[..., :hd]
    k = qkv[:, nq * 2 * hd: nq * 2 * hd + nkv * hd].reshape(T, nkv, hd)
    v = qkv[:, nq * 2 * hd + nkv * hd:].reshape(T, nkv, hd)
    qn = (1 + 0.1 * torch.randn(hd, device=DEV)).float()
    kn = (1 + 0.1 * torch.randn(hd, device=DEV)).float()
    pos = torch.tensor([0, 1, 5, 17, 100, 1000, 4095, 8000, 12, 13, 65535], dtype=torch.int32, device=DEV)
    rows = torch.randperm(64, device=DEV)[:T].int()
    kc = torch.zeros(64, nkv, hd, dtype=BF, device=DEV)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone(), vc.clone()
    qo = ops.qk_norm_rope_kv_write(q, k, v, qn, kn, pos, rows, kc, vc, rot, 1e7, 1e-6)
    # oracle on CPU (same math)
    qr = ops.qk_norm_rope_kv_write(q.cpu(), k.cpu(), v.cpu(), qn.cpu(), kn.cpu(), pos.cpu(), rows.cpu(),
                                   kc2.cpu(), vc2.cpu(), rot, 1e7, 1e-6)
    kref = kc2.cpu()
    kref[rows.long().cpu()] = ref.apply_partial_rope(ref.rmsnorm(k.cpu(), kn.cpu(), 1e-6),
                                                     *ref.rope_cos_sin(pos.cpu(), rot, 1e7, BF))
    close(qo.cpu(), qr, atol=2e-2)
    close(kc.cpu(), kref, atol=2e-2)
    assert torch.equal(vc[rows.long()].cpu(), v.cpu())


def _paged(ctx_lens, nkv, hd, bs=16, seed=0):
    lanes = len(ctx_lens)
    max_blocks = max((c + bs - 1) // bs for c in ctx_lens) + 1
    nblocks = 1 + lanes * max_blocks
    kc = rnd(nblocks * bs, nkv, hd, seed=seed)
    vc = rnd(nblocks * bs, nkv, hd, seed=seed + 1)
    perm = torch.randperm(nblocks - 1) + 1
    table = torch.zeros(lanes, max_blocks, dtype=torch.int32)
    for l in range(lanes):
        table[l] = perm[l * max_blocks:(l + 1) * max_blocks].int()
    return kc, vc, table.to(DEV), max_blocks


@pytest.mark.parametrize("nq,nkv,hd", [(16, 1, 256), (4, 1, 256), (4, 2, 64)])
def test_attention_decode_and_prefill(nq, nkv, hd):
    bs = 16
    ctx = [1, 37, 300, 2049]
    kc, vc, table, mb = _paged(ctx, nkv, hd, bs, seed=nq)
    # segments: lanes 0,1 decode one token; lane 2 prefill 5 tokens; lane 3 decode
    segs = [(0, ctx[0] - 1, 1), (1, ctx[1] - 1, 1), (2, ctx[2] - 5, 5), (3, ctx[3] - 1, 1)]
    T = sum(s[2] for s in segs)
    q = rnd(T, nq, hd, seed=99)
    pos, lanes, cu, starts = [], [], [0], []
    for lane, st, n in segs:
        pos += list(range(st, st + n))
        lanes.append(lane)
        starts.append(st)
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device=DEV)
    out = ops.attention_varlen(q, kc, vc, table, torch.tensor(lanes, **i32), torch.tensor(cu, **i32),
                               torch.tensor(starts, **i32), bs, positions=torch.tensor(pos, **i32),
                               max_ctx=max(ctx))
    exp = ops.attention_varlen(q.cpu(), kc.cpu(), vc.cpu(), table.cpu(), torch.tensor(lanes), torch.tensor(cu),
                               torch.tensor(starts), bs, lanes, cu, starts, table.cpu().tolist())
    close(out.cpu(), exp, atol=2e-2)


def test_causal_conv_and_delta_rule():
    nk, nv, dk, dv, K = 2, 8, 128, 128, 4
    C = 2 * nk * dk + nv * dv
    lanes = 3
    segs = [(0, 1), (2, 17), (1, 5)]
    T = sum(n for _, n in segs)
    x = rnd(T, C + 64, seed=21)[:, :C]
    w = rnd(C, K, scale=0.3, seed=22)
    st = rnd(lanes, C, K - 1, seed=23)
    st2 = st.clone().cpu()
    cu = [0]
    for _, n in segs:
        cu.append(cu[-1] + n)
    ln = [l for l, _ in segs]
    i32 = dict(dtype=torch.int32, device=DEV)
    out = ops.causal_conv_varlen(x, st, w, torch.tensor(ln, **i32), torch.tensor(cu, **i32))
    exp = ops.causal_conv_varlen(x.cpu(), st2, w.cpu(), torch.tensor(ln), torch.tensor(cu), ln, cu)
    close(out.cpu(), exp, atol=2e-2)
    close(st.cpu(), st2, atol=0)
    # runs of tokens crossing several segments, an empty segment among them (one lane per segment)
    segs_b = [(0, 37), (1, 0), (2, 20), (3, 3)]
    cub = [0]
    for _, n in segs_b:
        cub.append(cub[-1] + n)
    xb = rnd(cub[-1], C, seed=31)
    stb = rnd(len(segs_b), C, K - 1, seed=32)
    stb2 = stb.clone().cpu()
    lnb = [l for l, _ in segs_b]
    outb = ops.causal_conv_varlen(xb, stb, w, torch.tensor(lnb, **i32), torch.tensor(cub, **i32))
    expb = ops.causal_conv_varlen(xb.cpu(), stb2, w.cpu(), torch.tensor(lnb), torch.tensor(cub), lnb, cub)
    close(outb.cpu(), expb, atol=2e-2)
    close(stb.cpu(), stb2, atol=0)
    # delta rule on the conv output
    ab = rnd(T, 2 * nv, seed=24)
    a_log = torch.log(torch.rand(nv, device=DEV) * 15 + 1)
    dtb = torch.rand(nv, device=DEV)
    rs = torch.randn(lanes, nv, dk, dv, device=DEV) * 0.1
    rs2 = rs.clone().cpu()
    o = ops.gated_delta_varlen(out, ab, a_log, dtb, rs, torch.tensor(ln, **i32), torch.tensor(cu, **i32), nk, nv, dk, dv)
    oe = ops.gated_delta_varlen(out.cpu(), ab.cpu(), a_log.cpu(), dtb.cpu(), rs2, torch.tensor(ln), torch.tensor(cu),
                                nk, nv, dk, dv, ln, cu)
    close(o.cpu(), oe, atol=2e-2)
    close(rs.cpu(), rs2, rtol=1e-2, atol=1e-3)  # bf16 l2norm rounding emulation


@pytest.mark.parametrize("T,E,k,H,I", [(3, 32, 4, 256, 128), (40, 64, 8, 512, 256), (5, 512, 10, 4096, 1024),
                                       (300, 64, 4, 1024, 256)])
@pytest.mark.parametrize("impl", ["mx", "f16"])
def test_moe_routed_mxfp4(T, E, k, H, I, impl, monkeypatch):
    """Both CUDA paths (block-scaled MMA with hi/lo e4m3 activations, and f16 decode) against
    the fp32 dequantised reference."""
    monkeypatch.setenv("QB_MOE_IMPL", impl)
    torch.manual_seed(T + E)
    h = rnd(T, H, seed=T)
    if E * I * H <= 2 ** 24:
        w13, s13 = mxfp4.quantize(torch.randn(E, 2 * I, H, device=DEV) * 0.02)
        w2, s2 = mxfp4.quantize(torch.randn(E, H, I, device=DEV) * 0.02)
    else:  # random codes and scales (quantising 4 GB of fp32 weights would not fit)
        u8 = dict(dtype=torch.uint8, device=DEV)
        w13 = torch.randint(0, 256, (E, 2 * I, H // 2), **u8)
        s13 = torch.randint(116, 124, (E, 2 * I, H // 32), **u8)
        w2 = torch.randint(0, 256, (E, H, I // 2), **u8)
        s2 = torch.randint(116, 124, (E, H, I // 32), **u8)
    lg = rnd(T, E, seed=T + 1)
    topw, topi = ops.router_topk(lg, k)
    experts = {"w13": w13, "s13": s13, "w2": w2, "s2": s2}
    first, count = (E // 4, E // 2) if E >= 64 else (0, E)
    out = ops.moe_routed(h, topw, topi, experts, first, count)
    torch.cuda.synchronize()
    exp = ref.routed_experts(h, topw, topi.long(), experts, first, count)
    close(out, exp, rtol=3e-2, atol=3e-3)
    # the shared expert added in the combine: the same bits as the separate gate-and-add kernel
    sh = rnd(T, H, seed=T + 2)
    gl = rnd(T, 3, seed=T + 3)[:, 1]  # a strided column, as the router projection gives it
    fused = ops.moe_routed(h, topw, topi, experts, first, count, shared=sh, gate=gl)
    apart = ops.shared_gate_combine(ops.moe_routed(h, topw, topi, experts, first, count), sh, gl)
    torch.cuda.synchronize()
    assert torch.equal(fused, apart), (fused.float() - apart.float()).abs().max().item()
    status_ok()


def test_tiny_model_gpu_matches_cpu_reference(tiny_dir):
    from qwen35_b200.models.config import load_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import load_weights
    from qwen35_b200.parallel.plan import plan

    cfg = load_config(tiny_dir)
    p = plan(cfg, 0, 1)
    mg = Model(cfg, load_weights(tiny_dir, cfg, p, DEV, BF), p, device=DEV, dtype=BF, max_batch=2, max_seq=512)
    mc = Model(cfg, load_weights(tiny_dir, cfg, p, "cpu", torch.float32), p, device="cpu", dtype=torch.float32,
               max_batch=2, max_seq=512)
    ids = list(range(5, 105))
    mg.begin(0); mc.begin(0)
    mg.attach_blocks(0, list(range(1, 9))); mc.attach_blocks(0, list(range(1, 9)))
    a = mg.prefill(0, ids, 0).float().cpu()
    b = mc.prefill(0, ids, 0)
    cos = torch.nn.functional.cosine_similarity(a, b).item()
    assert cos > 0.99, cos
    status_ok()


@pytest.mark.parametrize("T,E,k,H,I", [(3, 32, 4, 256, 128), (40, 64, 8, 512, 256), (9, 128, 10, 4096, 1024)])
def test_moe_routed_bf16_experts(T, E, k, H, I):
    h = rnd(T, H, seed=T + 7)
    experts = {"w13": rnd(E, 2 * I, H, scale=0.02, seed=E), "w2": rnd(E, H, I, scale=0.02, seed=E + 1)}
    topw, topi = ops.router_topk(rnd(T, E, seed=T + 8), k)
    out = ops.moe_routed(h, topw, topi, experts, 0, E)
    torch.cuda.synchronize()
    exp = ref.routed_experts(h, topw, topi.long(), experts, 0, E)
    close(out, exp, rtol=3e-2, atol=3e-3)
    status_ok()


def test_mtp_round_on_gpu_equals_plain_decode():
    """Speculative rounds (draft, wide verify, DeltaNet commit of the accepted rows) emit the
    plain model's greedy tokens. The verify forward runs other kernels than one-row decode
    (flash attention, wider GEMM and MoE tiles), so bf16 summation order differs; on random
    weights a near-tie can flip. Each emitted token is therefore checked teacher-forced: it is
    the plain model's top-1 on its own prefix, up to a bf16 margin."""
    from qwen35_b200.models import mtp as mtpmod
    from qwen35_b200.models.config import tiny_config
    from qwen35_b200.models.qwen35 import Model
    from qwen35_b200.models.weights import random_weights
    from qwen35_b200.parallel.plan import plan

    cfg = tiny_config()
    p = plan(cfg, 0, 1)
    w = random_weights(cfg, p, torch.device(DEV), BF, seed=3, with_mtp=True)
    ids = list(range(11, 91))

    def fresh(spec):
        m = Model(cfg, w, p, device=DEV, dtype=BF, max_batch=2, max_seq=512)
        if spec:
            mtpmod.attach(m, k=3)
        m.begin(0)
        m.attach_blocks(0, list(range(1, 20)))
        return m, m.prefill(0, ids, 0)

    plain, lg = fresh(False)
    ref, t = [], int(lg.float().argmax())
    for j in range(40):  # the plain model's greedy continuation, used as oracle drafts
        ref.append(t)
        t = int(plain.decode([0], [t], [len(ids) + j]).float().argmax())

    m, lg = fresh(True)
    head = m.mtp
    calls = [0]

    def oracle_draft(lanes, tokens, positions):
        j = positions[0] - len(ids)
        d = [ref[min(j + 1 + i, len(ref) - 1)] for i in range(head.k)]
        calls[0] += 1
        if calls[0] % 2 == 0:  # every other round: last draft wrong -> partial acceptance
            d[-1] = (d[-1] + 1) % cfg.vocab
        head.drafted += head.k
        return torch.tensor([d], device=DEV)

    head.draft = oracle_draft
    tok, pos, got = int(lg.float().argmax()), len(ids), []
    while len(got) < 16:
        new = m.speculative_decode([0], [tok], [pos], [16 - len(got)], [[]])[0]
        got += [tok] + new[:-1]
        pos += len(new)
        tok = new[-1]
    got = got[:16]
    assert head.accepted > 0
    plain, lg = fresh(False)
    for j, t in enumerate(got):
        lg = lg.float().flatten()
        top = lg.max().item()
        assert lg[t].item() >= top - 3e-2 * max(1.0, abs(top)), (j, t, lg[t].item(), top)
        lg = plain.decode([0], [t], [len(ids) + j])
    status_ok()


@pytest.mark.parametrize("nq,nkv,hd", [(32, 2, 256), (4, 1, 256), (8, 2, 64), (16, 1, 128)])
def test_flash_attention_prefill(nq, nkv, hd):
    """tcgen05 prefill attention: prompt chunks continuing a cached prefix, several segments."""
    bs = 16
    ctx = [300, 77, 1000, 130]
    kc, vc, table, mb = _paged([c + 8 for c in ctx], nkv, hd, bs, seed=hd + nq)
    segs = [(0, 0, 300), (1, 40, 37), (2, 700, 300), (3, 129, 1)]  # (lane, start, rows)
    T = sum(s[2] for s in segs)
    q = rnd(T, nq, hd, seed=5 + hd)
    pos, lanes, cu, starts = [], [], [0], []
    for lane, st, n in segs:
        pos += list(range(st, st + n))
        lanes.append(lane)
        starts.append(st)
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device=DEV)
    assert ops.fa_plan(q, kc, cu, bs, max(ctx)) is not None
    out = ops.attention_varlen(q, kc, vc, table, torch.tensor(lanes, **i32), torch.tensor(cu, **i32),
                               torch.tensor(starts, **i32), bs, lanes, cu, starts, None,
                               positions=torch.tensor(pos, **i32), max_ctx=max(ctx))
    torch.cuda.synchronize()
    exp = ops.attention_varlen(q.cpu(), kc.cpu(), vc.cpu(), table.cpu(), torch.tensor(lanes), torch.tensor(cu),
                               torch.tensor(starts), bs, lanes, cu, starts, table.cpu().tolist())
    close(out.cpu(), exp, atol=2e-2)
    status_ok()


@pytest.mark.parametrize("nq,nkv,hd", [(32, 2, 256), (8, 2, 64), (16, 1, 128)])
def test_flash_attention_decode_splits(nq, nkv, hd):
    """Decode-shaped batches through the tcgen05 kernel with key-range splits: one-row lanes with
    short and long contexts (some splits get no keys) and a 4-row verify-style segment."""
    bs = 16
    ctx = [1, 20, 700, 3000, 64]
    kc, vc, table, mb = _paged([c + 4 for c in ctx], nkv, hd, bs, seed=hd + 7)
    segs = [(0, 0, 1), (1, 19, 1), (2, 699, 1), (3, 2996, 4), (4, 63, 1)]  # (lane, start, rows)
    T = sum(s[2] for s in segs)
    q = rnd(T, nq, hd, seed=11 + hd)
    pos, lanes, cu, starts = [], [], [0], []
    for lane, st, n in segs:
        pos += list(range(st, st + n))
        lanes.append(lane)
        starts.append(st)
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device=DEV)
    plan = ops.fa_plan(q, kc, cu, bs, max(ctx))
    assert plan is not None and plan[1] > 1
    out = ops.attention_varlen(q, kc, vc, table, torch.tensor(lanes, **i32), torch.tensor(cu, **i32),
                               torch.tensor(starts, **i32), bs, lanes, cu, starts, None,
                               positions=torch.tensor(pos, **i32), max_ctx=max(ctx))
    torch.cuda.synchronize()
    exp = ops.attention_varlen(q.cpu(), kc.cpu(), vc.cpu(), table.cpu(), torch.tensor(lanes), torch.tensor(cu),
                               torch.tensor(starts), bs, lanes, cu, starts, table.cpu().tolist())
    close(out.cpu(), exp, atol=2e-2)
    status_ok()


@pytest.mark.parametrize("mode,vsplit", [("tc", "1"), ("tc", "2"), ("tc", "0"), ("chunked_fp32", "0")])
def test_chunked_delta_rule_matches_recurrence(monkeypatch, mode, vsplit):
    """Chunked (WY) delta rule on prefill-sized segments vs the fp32 token recurrence (PyTorch on
    the host): outputs and the carried state, several segments (one shorter than a chunk, one of
    a single row, one spanning four chunks). ``tc`` keeps the state in tensor memory and rounds
    the MMA operands to bf16 (fp32 accumulate), hence its wider tolerance; its state kernel runs
    with whole heads per CTA and with heads split over two CTAs by value columns."""
    monkeypatch.setenv("QB_DN_PREFILL", mode)
    monkeypatch.setenv("QB_DN_VSPLIT", vsplit)  # state CTAs per value head: 1, 2 (64 columns each), 0 auto
    nk, nv, dk, dv = 2, 8, 128, 128
    C = 2 * nk * dk + nv * dv
    lanes = 4
    segs = [(0, 200), (2, 64), (1, 1), (3, 130), (4, 256)]
    lanes = 5
    T = sum(n for _, n in segs)
    cu = [0]
    for _, n in segs:
        cu.append(cu[-1] + n)
    ln = [l for l, _ in segs]
    qkv = rnd(T, C, seed=31)
    ab = rnd(T, 2 * nv, seed=32)
    a_log = torch.log(torch.rand(nv, device=DEV) * 15 + 1)
    dtb = torch.rand(nv, device=DEV)
    rs = torch.randn(lanes, nv, dk, dv, device=DEV) * 0.1
    rs2 = rs.clone().cpu()
    i32 = dict(dtype=torch.int32, device=DEV)
    assert ops.dn_chunk_plan(cu, dk, dv, qkv.device, mode) is not None
    o = ops.gated_delta_varlen(qkv, ab, a_log, dtb, rs, torch.tensor(ln, **i32), torch.tensor(cu, **i32), nk, nv, dk,
                               dv, ln, cu)
    torch.cuda.synchronize()
    oe = ops.gated_delta_varlen(qkv.cpu(), ab.cpu(), a_log.cpu(), dtb.cpu(), rs2, torch.tensor(ln), torch.tensor(cu),
                                nk, nv, dk, dv, ln, cu)
    if mode == "tc":
        close(o.cpu(), oe, atol=6e-2, rtol=3e-2)
        close(rs.cpu(), rs2, rtol=3e-2, atol=1e-2)
    else:
        close(o.cpu(), oe, atol=2e-2)
        close(rs.cpu(), rs2, rtol=1e-2, atol=1e-3)
    # commit=False leaves the state alone
    before = rs.clone()
    ops.gated_delta_varlen(qkv, ab, a_log, dtb, rs, torch.tensor(ln, **i32), torch.tensor(cu, **i32), nk, nv, dk,
                           dv, ln, cu, commit=False)
    torch.cuda.synchronize()
    assert torch.equal(rs, before)
    status_ok()


@pytest.mark.parametrize("nk,nv,lanes", [(16, 64, 32), (4, 8, 3), (2, 8, 5)])
def test_deltanet_decode_fused(nk, nv, lanes):
    """The fused one-token-per-lane DeltaNet mixer equals the separate conv, delta-rule and
    gated-norm kernels: output, fp32 state and conv window (lanes in shuffled order)."""
    dk = dv = 128
    C = 2 * nk * dk + nv * dv
    g = torch.Generator(device=DEV).manual_seed(nv + lanes)
    proj = (torch.randn(lanes, C + nv * dv + 2 * nv, device=DEV, generator=g)).to(BF)
    conv_w = (0.3 * torch.randn(C, 4, device=DEV, generator=g)).to(BF)
    a_log = torch.log(torch.rand(nv, device=DEV, generator=g) * 15 + 1)
    dt_bias = torch.randn(nv, device=DEV, generator=g)
    norm_w = (1 + 0.1 * torch.randn(dv, device=DEV, generator=g)).to(BF)
    n_lanes = lanes + 2
    cs0 = torch.randn(n_lanes, C, 3, device=DEV, generator=g).to(BF)
    st0 = 0.1 * torch.randn(n_lanes, nv, dk, dv, device=DEV, generator=g)
    seg_lane = torch.randperm(n_lanes, generator=torch.Generator().manual_seed(1))[:lanes].int().to(DEV)
    cs1, st1 = cs0.clone(), st0.clone()
    out = ops.deltanet_decode(proj, cs1, conv_w, a_log, dt_bias, st1, norm_w, seg_lane, nk, nv, dk, dv, 1e-6)
    # the separate kernels on copies
    cs2, st2 = cs0.clone(), st0.clone()
    cu = torch.arange(lanes + 1, dtype=torch.int32, device=DEV)
    lanes_h, cu_h = seg_lane.tolist(), list(range(lanes + 1))
    qkv = ops.causal_conv_varlen(proj[:, :C], cs2, conv_w, seg_lane, cu, lanes_h, cu_h)
    core = ops.gated_delta_varlen(qkv, proj[:, C + nv * dv:], a_log, dt_bias, st2, seg_lane, cu, nk, nv, dk, dv,
                                  lanes_h, cu_h)
    exp = ops.gated_rmsnorm(core, proj[:, C:C + nv * dv].reshape(lanes, nv, dv), norm_w, 1e-6).reshape(lanes, -1)
    torch.cuda.synchronize()
    assert torch.equal(cs1, cs2)
    assert (st1 - st2).abs().max().item() < 1e-4 * st2.abs().max().item() + 1e-6
    close(out, exp, rtol=2e-2, atol=2e-2)
    status_ok()


def test_router_topk_nan_rows_select_no_expert():
    """A row of NaN router logits (padding rows of a fixed-width captured prefill are not
    initialised) gets expert id -1 and weight 0 instead of an index past the expert array;
    the other rows are unaffected and the routed-expert op writes zeros for such rows."""
    E, k = 64, 4
    lg = rnd(6, E, seed=9)
    lg[2] = float("nan")
    lg[4, :] = float("nan")
    w, i = ops.router_topk(lg, k)
    torch.cuda.synchronize()
    assert (i[2] == -1).all() and (i[4] == -1).all() and (w[2] == 0).all() and (w[4] == 0).all()
    ok = [0, 1, 3, 5]
    rw, ri = ref.router_topk(lg[ok], k)
    assert torch.equal(i[ok].long().sort(-1).values, ri.long().sort(-1).values)
    H, I = 256, 128
    w13, s13 = mxfp4.quantize(torch.randn(E, 2 * I, H, device=DEV) * 0.02)
    w2, s2 = mxfp4.quantize(torch.randn(E, H, I, device=DEV) * 0.02)
    h = rnd(6, H, seed=10)
    y = ops.moe_routed(h, w, i, {"w13": w13, "s13": s13, "w2": w2, "s2": s2}, 0, E)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all() and y[2].abs().sum() == 0 and y[4].abs().sum() == 0
    status_ok()
