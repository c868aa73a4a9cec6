"""Flag registry, GPU-local CPU affinity, the boot memory report and clock stamps (CPU parts)."""

import re
from pathlib import Path

import pytest
import torch

from qwen35_b200.utils import affinity, flags, memreport
from qwen35_b200.utils.telemetry import Stamps

PKG = Path(__file__).resolve().parent.parent / "qwen3.5-397b-mi300a-bespoke-vibesys-20260920_b200"


def _sources(*suffixes):
    return [p for p in PKG.rglob("*") if p.suffix in suffixes and "_build" not in p.parts]


def test_every_python_flag_read_is_declared():
    reg = flags.registry()
    for p in _sources(".py"):
        text = p.read_text()
        for name in re.findall(r'flags\.get\("(QB_[A-Z0-9_]+)"', text):
            assert name in reg, (p.name, name)
        if p.name != "flags.py":
            # QB_* variables are read through the registry only
            assert not re.search(r'environ(?:\.get|\.setdefault|\.pop)?[\[(]\s*"QB_', text), p.name
            assert not re.search(r'getenv\(\s*"QB_', text), p.name


def test_every_native_flag_read_is_declared():
    reg = flags.registry()
    seen = set()
    for p in _sources(".cu", ".cpp", ".h", ".cuh"):
        for name in re.findall(r'getenv\("(QB_[A-Z0-9_]+)"\)', p.read_text()):
            seen.add(name)
            assert name in reg and reg[name].native, (p.name, name)
    assert seen == {n for n, f in reg.items() if f.native}


def test_flag_put_checks_name_and_value(monkeypatch):
    monkeypatch.setenv("QB_PDL", "")
    flags.put("QB_PDL", 0, only_if_unset=True)
    assert flags.get("QB_PDL") == 0
    flags.put("QB_PDL", 1, only_if_unset=True)  # already set: the explicit value wins
    assert flags.get("QB_PDL") == 0
    flags.put("QB_PDL", 1)
    assert flags.get("QB_PDL") == 1
    import pytest

    with pytest.raises(KeyError):
        flags.put("QB_NOT_A_FLAG", 1)
    with pytest.raises(ValueError):
        flags.put("QB_PDL", "many")


def test_flag_parsing_and_signature():
    assert flags.get("QB_GRAPHS", {}) is True
    assert flags.get("QB_GRAPHS", {"QB_GRAPHS": "0"}) is False
    assert flags.get("QB_SP_MAX_ROWS", {"QB_SP_MAX_ROWS": "128"}) == 128
    assert flags.get("QB_SP_MAX_ROWS", {"QB_SP_MAX_ROWS": ""}) == 4096
    with pytest.raises(ValueError):
        flags.get("QB_SP_MAX_ROWS", {"QB_SP_MAX_ROWS": "many"})
    with pytest.raises(KeyError):
        flags.get("QB_NOT_A_FLAG", {})
    base = flags.signature({})
    assert flags.signature({"QB_STEP_TIMING": "5"}) == base  # diagnostics do not enter it
    assert flags.signature({"QB_COMM": "nccl"}) != base
    assert flags.signature({"QB_MOE_IMPL": "f16"}) != base
    assert "QB_MOE_IMPL" in flags.describe()


def test_parse_cpulist():
    assert affinity.parse_cpulist("") == set()
    assert affinity.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    with pytest.raises(ValueError):
        affinity.parse_cpulist("5-2")


def test_gpu_local_cpus_from_sysfs(tmp_path):
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text("24-26,120\n")
    # CUDA's bus id form (8-digit domain, upper case) maps to the sysfs name
    assert affinity.gpu_local_cpus("00000000:1B:00.0", root=str(tmp_path)) == {24, 25, 26, 120}
    assert affinity.gpu_local_cpus("00000000:99:00.0", root=str(tmp_path)) == set()


def test_pin_to_gpu_with_fakes(tmp_path):
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text("4-7")
    calls = []
    allowed = {0, 1, 2, 3, 4, 5}
    kw = dict(root=str(tmp_path), setter=calls.append, getter=lambda: allowed)
    assert affinity.pin_to_gpu("00000000:1B:00.0", {}, **kw) == "" and not calls  # off by default
    note = affinity.pin_to_gpu("00000000:1B:00.0", {"QB_CPU_AFFINITY": "1"}, **kw)
    assert calls == [{4, 5}] and "2 CPUs" in note  # only CPUs the process may use
    calls.clear()
    assert affinity.pin_to_gpu("00000000:99:00.0", {"QB_CPU_AFFINITY": "1"}, **kw) == "" and not calls


def test_mem_report_off_by_default_and_pool_plan_on_cpu():
    from qwen35_b200.serving.engine import PoolSpec, build_model

    assert memreport.BootMemory(0, torch.device("cpu")).phase("x") is None
    m, _ = build_model("tiny", 0, 1, torch.device("cpu"), PoolSpec(lanes=2, max_seq=64, kv_tokens=128),
                       dtype=torch.float32, graphs=False)
    assert memreport.pool_plan(m) is None  # off unless QB_MEM_REPORT
    lines = []
    rec = memreport.pool_plan(m, sink=lines.append, force=True)
    assert lines and lines[0].startswith("[pool-plan]")
    b = memreport.pool_bytes_of(m)
    kv = sum(t.numel() * t.element_size() for t in m.k_cache + m.v_cache)
    assert b["kv_cache"] == kv and b["experts"] > 0 and b["deltanet"] > 0 and b["attention"] > 0
    assert rec["kv_tokens"] == m.num_blocks * m.block_size and rec["lanes"] == m.max_batch


def test_stamps_on_cpu():
    st = Stamps(torch.device("cpu"), capacity=8)
    for tag in ("start", "a", "b", "a"):
        st.mark(tag)
    seg = st.segments_ms()
    assert [t for t, _ in seg] == ["a", "b", "a"] and all(ms >= 0 for _, ms in seg)
    agg = st.by_tag_ms()
    assert set(agg) == {"a", "b", "total"}
    assert abs(agg["total"] - sum(ms for _, ms in seg)) < 1e-9
    for _ in range(4):
        st.mark("x")
    with pytest.raises(RuntimeError):
        st.mark("overflow")


def test_model_stamps_on_cpu():
    """A tiny CPU model step with stamps installed tags every layer part once per layer."""
    from qwen35_b200.serving.engine import PoolSpec, build_model

    m, _ = build_model("tiny", 0, 1, torch.device("cpu"), PoolSpec(lanes=2, max_seq=64, kv_tokens=128),
                       dtype=torch.float32, graphs=False)
    m.begin(0)
    m.attach_blocks(0, [1, 2])
    m.stamps = Stamps(torch.device("cpu"))
    m.forward([(0, [1, 2, 3], 0)])
    tags = m.stamps.tags
    n = m.cfg.layers
    assert tags[0] == "start" and tags[-1] == "lm_head"
    assert tags.count("moe") == n and tags.count("allreduce") == 2 * n
    assert tags.count("attention") + tags.count("deltanet") == n


def test_mx_tile_codes_layout():
    """Tile-contiguous expert codes: block (expert, tile, stage) holds rows of that tile (gate rows
    then the matching up rows for gate_up) and bytes of that K stage, in order."""
    from qwen35_b200.ops.core import mx_tile_codes

    E, rows, kb2 = 2, 256, 128  # 2 tiles, 2 stages
    w = torch.randint(0, 256, (E, rows, kb2), dtype=torch.uint8)
    for gate_up in (False, True):
        t = mx_tile_codes(w, gate_up).view(E, rows // 128, kb2 // 64, 128, 64)
        for e in range(E):
            for nt in range(rows // 128):
                for ks in range(kb2 // 64):
                    for r in (0, 5, 63, 64, 100, 127):
                        if gate_up:
                            src = nt * 64 + r if r < 64 else rows // 2 + nt * 64 + (r - 64)
                        else:
                            src = nt * 128 + r
                        assert torch.equal(t[e, nt, ks, r], w[e, src, ks * 64:(ks + 1) * 64])

