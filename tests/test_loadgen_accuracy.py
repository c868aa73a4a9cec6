"""The HTTP load generator and the accuracy gates against the tiny model's server (CPU)."""

import asyncio
import json

import pytest

from qwen35_b200.serving import accuracy, loadgen
from test_server import start, stop


@pytest.fixture(scope="module")
def server():
    proc, url = start()
    yield url
    stop(proc)


@pytest.fixture(scope="module")
def pins():
    return accuracy.make_pins("tiny", n_pins=8, n_tokens=12, seed=0, prompt_len=(16, 80))


def test_pins_match_the_served_model(server, pins):
    res = accuracy.check_pins(server, pins)
    assert res["pass"] and res["exact_fraction"] == 1.0, res


def test_a_wrong_pin_fails_with_early_divergence(server, pins):
    bad = json.loads(json.dumps(pins))
    bad["pins"][3]["expected_token_ids"][2] += 1
    res = accuracy.check_pins(server, bad)
    assert not res["pass"] and res["early_divergence"] == [bad["pins"][3]["id"]]


def test_sessions_gate(server):
    res = accuracy.check_sessions(server, sessions=2, turns=3, max_tokens=6)
    assert res["pass"], res


def test_pins_file_validation(tmp_path, pins, server):
    p = tmp_path / "pins.json"
    small = dict(pins, pins=pins["pins"][:3])
    p.write_text(json.dumps(small))
    with pytest.raises(accuracy.PinsError):
        accuracy.load_pins(str(p))
    p.write_text(json.dumps(pins))
    assert len(accuracy.load_pins(str(p))["pins"]) == 8
    # a missing pins file fails the check (exit 1); --skip-pins runs the other gates only
    assert accuracy.main(["check", "--url", server, "--pins", str(tmp_path / "missing.json")]) == 1
    assert accuracy.main(["check", "--url", server, "--pins", str(p)]) == 0


@pytest.mark.parametrize("mode", ["chat", "ids"])
def test_loadgen_level(server, mode):
    spec = loadgen.LoadSpec(levels=(2,), warmup_s=0.0, window_s=4.0, turns=(2, 3), words=(5, 20), ids=(5, 20),
                            first_ids=(20, 60), max_tokens=(3, 6), vocab=3000, c_ref=2, mode=mode)
    res = asyncio.run(loadgen.ramp(server, spec))
    lv = res["levels"][0]
    assert lv["failed"] == 0 and lv["turns"] > 0, lv
    assert lv["goodput_tok_s"] > 0 and lv["p95_ttft_all_ms"] is not None
    if lv["turns_ge2"]:
        assert res["p95_ttft_turn2plus_ms_at_ref"] is not None
        assert lv["cached_token_share"] > 0  # later turns resume from the session cache


def test_session_stream_is_deterministic():
    a = loadgen.SessionStream(loadgen.LoadSpec(mode="ids", vocab=100))
    b = loadgen.SessionStream(loadgen.LoadSpec(mode="ids", vocab=100))
    assert [a.take() for _ in range(3)] == [b.take() for _ in range(3)]
