"""The checkpoint loader's sharding (no GPU): loading the tiny checkpoint as rank r of 2 or 4 gives
exactly rank r's slice of what one rank loads, for the tensors split by rows (vocabulary rows of
the LM head, experts), by columns (the row-parallel output projections: attention o_proj,
DeltaNet out_proj, shared-expert down), and replicated ones (embedding, norms, router)."""

import pytest
import torch

from qwen35_b200.models.config import load_config
from qwen35_b200.models.weights import load_weights
from qwen35_b200.parallel.plan import plan


@pytest.fixture(scope="module")
def full(tiny_dir):
    cfg = load_config(tiny_dir)
    return cfg, load_weights(tiny_dir, cfg, plan(cfg, 0, 1), "cpu", torch.float32, with_mtp=False)


@pytest.mark.parametrize("world", [2, 4])
def test_rank_slices_equal_the_single_rank_load(tiny_dir, full, world):
    cfg, w1 = full
    for r in range(world):
        p = plan(cfg, r, world)
        w = load_weights(tiny_dir, cfg, p, "cpu", torch.float32, with_mtp=False)
        assert torch.equal(w["embed"], w1["embed"]) and torch.equal(w["final_norm"], w1["final_norm"])
        assert torch.equal(w["lm_head"], w1["lm_head"][p.vocab.start:p.vocab.stop])
        hd = cfg.head_dim
        assert any("w_o" in L for L in w["layers"]) and any("w_out" in L for L in w["layers"])
        for i, (L, L1) in enumerate(zip(w["layers"], w1["layers"])):
            assert L["kind"] == L1["kind"]
            for k in ("in_norm", "post_norm"):
                assert torch.equal(L[k], L1[k]), (i, k)
            if "w_o" in L:  # attention: o_proj columns of this rank's query heads
                assert torch.equal(L["w_o"], L1["w_o"][:, p.q.start * hd:p.q.stop * hd]), i
            if "w_out" in L:  # DeltaNet: out_proj columns of this rank's value heads
                dv = cfg.dn_v_dim
                assert torch.equal(L["w_out"], L1["w_out"][:, p.dn_v.start * dv:p.dn_v.stop * dv]), i
            sh = (p.shared.start, p.shared.stop)
            assert torch.equal(L["w_sh2"], L1["w_sh2"][:, sh[0]:sh[1]]), i
            e = (p.experts.start, p.experts.stop)
            for k in L["experts"]:
                assert torch.equal(L["experts"][k], L1["experts"][k][e[0]:e[1]]), (i, k)
