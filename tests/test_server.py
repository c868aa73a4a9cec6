"""The HTTP server end to end on the tiny random-init model (CPU): SSE contract, token-id
completions, exact max_tokens, cache reuse across turns, reset, score, health, faults, TP=2."""

import json
import os
import random
import socket
import subprocess
import sys
import time

import pytest
import requests

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def start(tp=1, env_extra=None, model="tiny", extra_args=()):
    port = free_port()
    env = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="2", **(env_extra or {}))
    cmd = [sys.executable, "-m", "qwen35_b200.serving.server", "--model-path", model, "--port", str(port),
           "--tp", str(tp), "--device", "cpu", "--max-batch", "4", "--max-seq-len", "2048", "--kv-tokens", "16384",
           "--master-port", str(free_port()), *extra_args]
    proc = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
                            start_new_session=True)
    url = f"http://127.0.0.1:{port}"
    for _ in range(300):
        try:
            if requests.get(url + "/health", timeout=2).status_code == 200:
                return proc, url
        except Exception:
            pass
        if proc.poll() is not None:
            raise RuntimeError("server exited")
        time.sleep(0.5)
    proc.kill()
    raise RuntimeError("server did not become healthy")


def stop(proc):
    try:
        os.killpg(proc.pid, 15)
    except Exception:
        pass
    proc.wait(timeout=30)


@pytest.fixture(scope="module")
def server():
    proc, url = start()
    yield url
    stop(proc)


def sse(resp):
    out = []
    for line in resp.iter_lines():
        if not line:
            continue
        assert line.startswith(b"data: "), line
        payload = line[6:]
        if payload == b"[DONE]":
            out.append("[DONE]")
            break
        out.append(json.loads(payload))
    return out


def test_completions_token_ids_exact_length(server):
    ids = [random.Random(1).randrange(3000) for _ in range(50)]
    r = requests.post(server + "/v1/completions", json={"prompt": ids, "max_tokens": 12, "ignore_eos": True}).json()
    ch = r["choices"][0]
    assert len(ch["token_ids"]) == 12 and r["usage"]["completion_tokens"] == 12
    assert r["usage"]["prompt_tokens"] == 50
    r2 = requests.post(server + "/v1/completions", json={"prompt": ids, "max_tokens": 12, "ignore_eos": True}).json()
    assert r2["choices"][0]["token_ids"] == ch["token_ids"]  # greedy + exact-duplicate cache


def test_chat_stream_contract_and_usage(server):
    body = {"messages": [{"role": "user", "content": "hello there, how are you?"}], "max_tokens": 10,
            "stream": True, "ignore_eos": True, "stream_options": {"include_usage": True},
            "chat_template_kwargs": {"enable_thinking": False}}
    with requests.post(server + "/v1/chat/completions", json=body, stream=True) as resp:
        chunks = sse(resp)
    assert chunks[-1] == "[DONE]"
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    finals = [c for c in chunks[:-1] if c["choices"] and c["choices"][0]["finish_reason"]]
    assert finals and finals[-1]["choices"][0]["finish_reason"] == "length"
    usage = [c for c in chunks[:-1] if c.get("usage")]
    assert usage and usage[-1]["usage"]["completion_tokens"] == 10


def test_second_turn_reuses_cache(server):
    msgs = [{"role": "user", "content": "tell me about the sea " * 5}]
    r1 = requests.post(server + "/v1/chat/completions", json={"messages": msgs, "max_tokens": 8, "ignore_eos": True}).json()
    msgs += [{"role": "assistant", "content": r1["choices"][0]["message"]["content"]},
             {"role": "user", "content": "and the mountains?"}]
    r2 = requests.post(server + "/v1/chat/completions", json={"messages": msgs, "max_tokens": 8, "ignore_eos": True}).json()
    cached = r2["usage"]["prompt_tokens_details"]["cached_tokens"]
    # the reply comes back as text; the server splices in the ids it generated, so the cached
    # sequence covers the first prompt and the reply, not just the history before the reply
    assert cached >= r1["usage"]["prompt_tokens"] + r1["usage"]["completion_tokens"] - 1, (cached, r1["usage"])


def test_reset_score_health(server):
    assert requests.get(server + "/health").status_code == 200
    assert requests.get(server + "/v1/models").json()["data"]
    ev = requests.post(server + "/reset_prefix_cache").json()
    assert "evicted" in ev and ev["status"] == "ok" and "cleared_slots" in ev
    s = requests.post(server + "/v1/score", json={"prompt": [5, 6, 7, 8], "continuation": [9, 10, 11]}).json()
    assert len(s["logprobs"]) == 3 and all(x <= 0 for x in s["logprobs"])
    # the reference's request form: the same positions, with top-k alternatives
    r = requests.post(server + "/v1/score", json={"prompt": [5, 6, 7, 8, 9, 10, 11], "continuation_start": 4,
                                                   "top_k": 3}).json()
    assert r["object"] == "token_scores" and r["continuation_start"] == 4 and r["prompt_tokens"] == 7
    assert [x["token_id"] for x in r["scores"]] == [9, 10, 11]
    for x, lp in zip(r["scores"], s["logprobs"]):
        assert abs(x["logprob"] - lp) < 1e-4 and len(x["top_logprobs"]) == 3
        assert x["top_logprobs"][0]["logprob"] >= x["logprob"] - 1e-6
    bad = requests.post(server + "/v1/score", json={"prompt": [5, 6], "continuation_start": 2})
    assert bad.status_code == 400
    for bad in ({}, {"messages": []}, {"messages": ["hi"]}, {"messages": [{"role": "user", "content": "x" * 100000}]}):
        assert requests.post(server + "/v1/chat/completions", json=bad).status_code == 400, bad
    for bad_prompt in ([], [1.5, 2], [[1, 2], [3]], [7] * 100000):
        r = requests.post(server + "/v1/completions", json={"prompt": bad_prompt, "max_tokens": 2})
        assert r.status_code == 400, (bad_prompt[:3], r.status_code)
    assert requests.post(server + "/debug/fault", json={"name": "rope_base", "value": 10}).status_code == 404


@pytest.mark.slow
def test_fault_endpoint_changes_output_and_tp2_matches_tp1(tiny_dir):
    ids = list(range(100, 180))
    p1, u1 = start(env_extra={"QB_FAULT_ENDPOINT": "1"}, model=tiny_dir)
    try:
        base = requests.post(u1 + "/v1/completions", json={"prompt": ids, "max_tokens": 10, "ignore_eos": True}).json()
        r = requests.post(u1 + "/debug/fault", json={"name": "drop_expert", "value": 3})
        assert r.status_code == 200 and r.json()["faults"]["drop_expert"] == 3
        assert r.json()["faults"]["flip_causal_mask"] is None
        requests.post(u1 + "/reset_prefix_cache")
        assert requests.post(u1 + "/debug/fault", json={"name": "rope_base", "value": 10.0}).status_code == 200
        hurt = requests.post(u1 + "/v1/completions", json={"prompt": ids, "max_tokens": 10, "ignore_eos": True}).json()
        assert hurt["choices"][0]["token_ids"] != base["choices"][0]["token_ids"]
    finally:
        stop(p1)
    p2, u2 = start(tp=2, model=tiny_dir)
    try:
        tp2 = requests.post(u2 + "/v1/completions", json={"prompt": ids, "max_tokens": 10, "ignore_eos": True}).json()
        assert tp2["choices"][0]["token_ids"] == base["choices"][0]["token_ids"]
    finally:
        stop(p2)


def test_mtp_speculative_server_matches_plain(server):
    """``--mtp-k 2``: decode steps are speculative rounds (draft, wide verify, accept, commit);
    greedy acceptance keeps the emitted tokens identical to plain decoding."""
    ids = [random.Random(7).randrange(3000) for _ in range(40)]
    body = {"prompt": ids, "max_tokens": 16, "ignore_eos": True}
    plain = requests.post(server + "/v1/completions", json=body).json()["choices"][0]["token_ids"]
    proc, url = start(extra_args=("--mtp-k", "2"))
    try:
        spec = requests.post(url + "/v1/completions", json=body).json()["choices"][0]["token_ids"]
    finally:
        stop(proc)
    assert len(spec) == 16 and spec == plain


def test_prefill_graphs_option_sets_the_flag(monkeypatch):
    from qwen35_b200.serving import server
    from qwen35_b200.utils import flags

    monkeypatch.setenv("QB_PREFILL_GRAPHS", "")  # restored after the test (parse writes os.environ)
    server.parse(["--model-path", "tiny"])
    assert flags.get("QB_PREFILL_GRAPHS") == ""
    server.parse(["--model-path", "tiny", "--prefill-graphs", "512,2048"])
    assert flags.get("QB_PREFILL_GRAPHS") == "512,2048"
    monkeypatch.setenv("QB_MIXED_GRAPHS", "")
    server.parse(["--model-path", "tiny", "--mixed", "--mixed-graphs", "32:256"])
    assert flags.get("QB_MIXED_GRAPHS") == "32:256"
