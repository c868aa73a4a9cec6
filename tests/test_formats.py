"""Checkpoint formats on the host: the safetensors reader and writer against the standard
`safetensors` package (files written by either side read back bit for bit, row ranges read
only their rows, shards of one directory merged), and the MXFP4 codec (low nibble = even K,
e8m0 scale = floor(log2(block max)) - 2 + 127, round to nearest with ties to the even code,
saturation at 6 x scale, exact on representable values)."""

import os

import pytest
import torch
from safetensors.torch import load_file, save_file as st_save

from qwen35_b200.utils import mxfp4
from qwen35_b200.utils.safetensors_io import Checkpoint, save_file


def _tensors():
    g = torch.Generator().manual_seed(5)
    return {
        "a.bf16": torch.randn(7, 5, generator=g).bfloat16(),
        "b.f32": torch.randn(3, 4, 2, generator=g),
        "c.u8": torch.randint(0, 256, (9, 16), generator=g, dtype=torch.uint8),
        "d.i64": torch.arange(6, dtype=torch.int64),
        "e.scalar": torch.tensor(2.5),
        "f.empty": torch.zeros(0, 4),
    }


def test_writer_output_reads_in_the_standard_library(tmp_path):
    ts = _tensors()
    path = str(tmp_path / "x.safetensors")
    save_file(ts, path, metadata={"format": "pt"})
    back = load_file(path)
    assert set(back) == set(ts)
    for k, t in ts.items():
        assert back[k].dtype == t.dtype and torch.equal(back[k], t), k


def test_reader_reads_standard_files_and_row_ranges(tmp_path):
    ts = _tensors()
    st_save({k: v for k, v in ts.items() if k < "c"}, str(tmp_path / "model-00001.safetensors"))
    st_save({k: v for k, v in ts.items() if k >= "c"}, str(tmp_path / "model-00002.safetensors"))
    ck = Checkpoint(str(tmp_path))
    try:
        assert sorted(ck.names()) == sorted(ts) and ck.names("b.") == ["b.f32"]
        assert ck.has("c.u8") and not ck.has("zz") and ck.shape("b.f32") == (3, 4, 2)
        for k, t in ts.items():
            assert torch.equal(ck.load(k), t), k
        assert torch.equal(ck.load("a.bf16", rows=(2, 5)), ts["a.bf16"][2:5])
        assert torch.equal(ck.load("c.u8", rows=(8, 9)), ts["c.u8"][8:9])
        assert ck.load("b.f32", rows=(1, 1)).shape == (0, 4, 2)
    finally:
        ck.close()


def test_reader_rejects_a_directory_without_shards(tmp_path):
    os.makedirs(tmp_path / "empty")
    with pytest.raises(FileNotFoundError):
        Checkpoint(str(tmp_path / "empty"))


def test_mxfp4_nibble_order_and_scale_byte():
    # one row, one block of 32: values on the e2m1 grid with block max 6 -> shared exponent 0
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0] * 4)
    vals[1::2] *= -1  # odd K negative: their codes carry the sign bit in the HIGH nibble
    packed, scales = mxfp4.quantize(vals[None])
    assert scales.tolist() == [[127]]  # e8m0 of 2^0
    codes = [0, 1, 2, 3, 4, 5, 6, 7] * 4
    codes = [c | (8 if (i % 2 and c) else 0) for i, c in enumerate(codes)]
    expect = [codes[2 * j] | (codes[2 * j + 1] << 4) for j in range(16)]
    assert packed[0].tolist() == expect
    assert torch.equal(mxfp4.dequantize(packed, scales, torch.float32)[0], vals)


def test_mxfp4_rounding_ties_saturation_and_scale():
    blk = torch.zeros(32)
    blk[0] = 6.0  # block max: exponent floor(log2 6) - 2 = 0
    blk[1:8] = torch.tensor([0.75, 1.25, 2.5, 5.0, 0.2, 1.6, -2.9])
    packed, scales = mxfp4.quantize(blk[None])
    got = mxfp4.dequantize(packed, scales, torch.float32)[0]
    # ties go to the even code: 0.75 -> 1.0, 1.25 -> 1.0, 2.5 -> 2.0, 5.0 -> 4.0; nearest otherwise
    assert got[:8].tolist() == [6.0, 1.0, 1.0, 2.0, 4.0, 0.0, 1.5, -3.0]
    big = torch.full((1, 32), 3.0)
    big[0, 0] = 15.0  # max 15 -> exponent 1 (scale 2): 15 / 2 = 7.5 saturates to 6 -> 12
    p2, s2 = mxfp4.quantize(big)
    assert s2.tolist() == [[128]]
    d2 = mxfp4.dequantize(p2, s2, torch.float32)[0]
    assert d2[0].item() == 12.0 and d2[1].item() == 3.0


def test_mxfp4_round_trip_error_bound():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(16, 256, generator=g) * 0.02
    packed, scales = mxfp4.quantize(w)
    assert packed.shape == (16, 128) and scales.shape == (16, 8)
    d = mxfp4.dequantize(packed, scales, torch.float32)
    blocks = w.view(16, 8, 32)
    err = (d.view(16, 8, 32) - blocks).abs()
    unit = torch.exp2(scales.float() - 127).unsqueeze(-1)  # 2^E of each block
    # rounding moves a value by at most half the widest grid gap (4 -> 6: one unit); the block
    # maximum, in [4, 8) units, saturates at 6: under two units
    assert bool((err <= 2 * unit + 1e-12).all())
    inside = blocks.abs() <= 6 * unit
    assert bool((err[inside] <= unit.expand_as(err)[inside] + 1e-12).all())
    # representable values quantise exactly
    assert torch.equal(mxfp4.dequantize(*mxfp4.quantize(d), torch.float32), d)
    with pytest.raises(ValueError):
        mxfp4.quantize(torch.zeros(2, 30))
