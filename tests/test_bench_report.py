"""bench.py's TTFT bookkeeping: device TTFT sums the step intervals from admission to first
token; a turn >= 2 still waiting when the loop hit its time limit counts at its wait so far (a
lower bound) and the line says so; the reference arm needs fewer samples than ours."""

import argparse
import os
import sys
import time
from dataclasses import dataclass

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@dataclass
class Rec:
    turn: int
    submit_step: int
    first_step: int = -1
    end_step: int = -1
    t_submit: float = 0.0
    t_first: float = 0.0
    generated: int = 0
    error: object = None


def _args(**kw):
    a = argparse.Namespace(sessions=4, turns=2, steps=10, warmup=3, concurrency=2, max_seq=1024,
                           first_len=(1, 2), user_len=(1, 2), gen_len=(1, 2), seed=0,
                           max_seconds=780.0, budget_seconds=840.0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_ttft_sums_steps_and_censors_waiting_turns():
    steps = [10.0, 20.0, 30.0, 40.0]
    recs = [Rec(turn=0, submit_step=0, first_step=0),            # turn 1: not a sample
            Rec(turn=1, submit_step=1, first_step=2, t_submit=1.0, t_first=1.5),
            Rec(turn=1, submit_step=3)]                           # still waiting at the end
    dev, host, censored = bench.ttft_lists(recs, steps, t_end=3.0)
    assert dev == [50.0, 40.0]
    assert censored == 1
    assert host == [500.0, 3000.0]


def _report(recs, steps, impl):
    return bench.report(_args(), impl=impl, world=1, window_ms=sum(steps), host_s=1.0, records=recs,
                        step_ms=steps, kinds_summary=None, clocks={}, h2d=0, d2h=0, launches=0, sched_steps=len(steps),
                        boot_s=0.0, warm_s=0.0, cfg_desc="x", expert_storage="x", t_end=10.0)


def test_reference_needs_fewer_samples_and_lower_bound_is_marked():
    steps = [5.0] * 40
    recs = [Rec(turn=1, submit_step=i, first_step=i) for i in range(25)] + [Rec(turn=1, submit_step=30)]
    ours = _report(recs, steps, "ours")
    assert ours["value"] is None and "invalid" in ours
    ref = _report(recs, steps, "reference")
    assert ref["value"] is not None and ref["ttft_samples"] == 26
    assert ref["ttft_censored"] == 1 and ref["value_kind"].startswith("lower bound")
    # the censored turn waited 10 steps: p95 over 25 x 5 ms and one 50 ms lower bound
    assert 5.0 <= ref["value"] <= 50.0


def test_loop_seconds_fits_the_budget():
    a = _args(budget_seconds=(time.monotonic() - bench.T_PROCESS0) + 130.0, max_seconds=780.0)
    assert 90.0 <= bench.loop_seconds(a) <= 100.0
    a = _args(budget_seconds=1e6, max_seconds=780.0)
    assert bench.loop_seconds(a) == 780.0


def test_line_carries_the_driver_contract():
    """The JSON line has every key the benchmark contract names, with the right types: the
    metric, value and unit, the GPU count, steps and warm-up as given, ms per step x steps = the
    timed window, the direction and scaling kind, dtype and data, the config's model / batch /
    sequence / parallelism, clocks, the end-to-end block with its per-step copy bytes, and the
    launch count."""
    import json

    steps = [4.0] * 300
    recs = [Rec(turn=1, submit_step=i, first_step=i, t_submit=0.0, t_first=0.004, generated=3) for i in range(250)]
    line = bench.report(_args(steps=20, warmup=5), impl="ours", world=2, window_ms=sum(steps), host_s=1.3,
                        records=recs, step_ms=steps, kinds_summary={}, clocks={"sm_mhz": 1900.0, "sm_max_mhz": 1965.0,
                        "reasons": []}, h2d=20 * 1000, d2h=20 * 80, launches=12345, sched_steps=300, boot_s=1.0,
                        warm_s=1.0, cfg_desc="full", expert_storage="all layers distinct", t_end=2.0)
    parsed = json.loads(json.dumps(line))  # one plain JSON object
    for k, t in (("metric", str), ("unit", str), ("n_gpus", int), ("steps", int), ("warmup", int),
                 ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str), ("dtype", str),
                 ("data", str), ("config", dict), ("clocks", dict), ("e2e", dict), ("gpu_launches", int)):
        assert isinstance(parsed[k], t), k
    assert parsed["metric"] == bench.METRIC and parsed["n_gpus"] == 2
    assert parsed["steps"] == 20 and parsed["warmup"] == 5
    assert abs(parsed["ms_per_step"] * parsed["steps"] - sum(steps)) < 1e-6
    assert parsed["higher_is_better"] is False and parsed["scaling"] == "strong" and parsed["dtype"] == "bf16"
    assert isinstance(parsed["value"], float) and parsed["ttft_samples"] == 250
    for k in ("model", "global_batch", "seq_len", "parallelism"):
        assert k in parsed["config"], k
    assert parsed["config"]["parallelism"] == "tp2+ep2"
    e2e = parsed["e2e"]
    assert e2e["h2d_bytes_per_step"] == 1000 and e2e["d2h_bytes_per_step"] == 80 and "value" in e2e
    assert parsed["gpu_launches"] == 12345 and "vs_baseline" in parsed
