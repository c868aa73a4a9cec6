"""Host-side planning of the varlen kernels (no GPU): the flash-attention tile list and key-range
splits, the chunk table of the chunked DeltaNet prefill and the choice of its path, the widths of
the captured prefill steps. The kernels trust these tables, so every row must be covered exactly
once and the tables must depend only on the segment lengths (the captured graphs reuse them)."""

import pytest
import torch

from qwen35_b200.ops import core as ops
from qwen35_b200.serving.engine import prefill_graph_widths


@pytest.mark.parametrize("g", [1, 4, 8, 16])
def test_fa_tiles_cover_every_row_once(g):
    cu = [0, 1, 130, 130, 131, 700, 829]  # a one-row segment, an empty one, long and ragged ones
    tiles = ops.fa_tiles(cu, g)
    qt = 128 // g
    seen = []
    for seg, first, rows in tiles:
        assert 1 <= rows <= qt
        assert cu[seg] <= first and first + rows <= cu[seg + 1]  # a tile never crosses its segment
        seen.extend(range(first, first + rows))
    assert seen == list(range(cu[-1]))
    assert all(r == qt for s, f, r in tiles if f + qt <= cu[s + 1])  # only a segment's last tile is short


def test_fa_plan_splits_fill_one_wave_only_when_short():
    q = torch.zeros(40, 32, 256, dtype=torch.bfloat16)
    kc = torch.zeros(64, 2, 256, dtype=torch.bfloat16)
    tiles, splits = ops.fa_plan(q, kc, list(range(41)), 16, 6000)  # 40 decode rows: 40 x 2 CTAs
    assert tiles.shape == (40, 3) and splits == 148 // 80
    q = torch.zeros(2048, 32, 256, dtype=torch.bfloat16)
    tiles, splits = ops.fa_plan(q, kc, [0, 2048], 16, 6000)  # 256 tiles x 2 heads fill the SMs
    assert tiles.shape == (256, 3) and splits == 1
    t2, _ = ops.fa_plan(q, kc, [0, 2048], 16, 9000)
    assert t2 is tiles  # cached per segment lengths: one device table per shape
    assert ops.fa_plan(q, kc, [0, 2048], 32, 6000) is None  # other page sizes take the split-K kernel


def test_dn_chunk_plan_covers_segments_in_order():
    cu = [0, 200, 264, 265, 395, 651]
    chunks, seg0 = ops.dn_chunk_plan(cu, 128, 128, torch.device("cpu"), "tc")
    rows = chunks.tolist()
    first = seg0.tolist()
    assert first[0] == 0 and first[-1] == len(rows) and first == sorted(first)
    for s in range(len(cu) - 1):
        covered = []
        for seg, r0, n in rows[first[s]:first[s + 1]]:
            assert seg == s and 1 <= n <= ops.DN_CHUNK
            covered.extend(range(r0, r0 + n))
        assert covered == list(range(cu[s], cu[s + 1]))
    assert ops.dn_chunk_plan(cu, 64, 128, torch.device("cpu"), "tc") is None  # head size 128 only
    assert ops.dn_chunk_plan([0, 10, 20], 128, 128, torch.device("cpu"), "tc") is None  # all shorter than a chunk
    assert ops.dn_chunk_plan(cu, 128, 128, torch.device("cpu"), "recurrence") is None


def test_dn_prefill_mode_rule(monkeypatch):
    monkeypatch.setenv("QB_DN_PREFILL", "auto")
    assert ops.dn_prefill_mode(8, [0, 50]) == "tc"  # few heads per rank: always the chunked form
    assert ops.dn_prefill_mode(64, [0, ops.DN_TC_MIN_TOKENS - 1]) == "recurrence"
    assert ops.dn_prefill_mode(64, [0, 10, 10 + ops.DN_TC_MIN_TOKENS]) == "tc"
    monkeypatch.setenv("QB_DN_PREFILL", "recurrence")
    assert ops.dn_prefill_mode(8, [0, 4096]) == "recurrence"


def test_prefill_graph_widths_parse():
    assert prefill_graph_widths("512,2048") == [512, 2048]
    assert prefill_graph_widths("") == [] and prefill_graph_widths(None) == []
    assert prefill_graph_widths(" 64, x, 0,128") == [64, 128]
