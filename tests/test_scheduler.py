import random

import pytest

from fake_runner import FakeRunner, greedy
from qwen35_b200.serving.block_pool import BlockAllocator
from qwen35_b200.serving.scheduler import Request, Scheduler
from qwen35_b200.serving.session_cache import SessionCache


def run_sessions(sched, sessions, turns, max_new, rng, user_len=(5, 30)):
    """Drives ``sessions`` multi-turn conversations; returns per-turn (prompt, out, end)."""
    hist = {s: [rng.randrange(1000) for _ in range(rng.randint(*user_len))] for s in range(sessions)}
    log = []
    for turn in range(turns):
        res = {}
        for s in range(sessions):
            toks, ends = [], []
            res[s] = (list(hist[s]), toks, ends)
            sched.submit(Request(list(hist[s]), max_new,
                                 lambda e, toks=toks, ends=ends: toks.append(e[1]) if e[0] == "tok" else ends.append(e)))
        sched.run_until_idle()
        for s in range(sessions):
            prompt, toks, ends = res[s]
            log.append((turn, prompt, toks, ends))
            hist[s] = prompt + toks + [rng.randrange(1000) for _ in range(rng.randint(*user_len))]
    return log


@pytest.mark.parametrize("overlap", [False, True])
@pytest.mark.parametrize("mixed", [False, True])
@pytest.mark.parametrize("chunk,budget", [(8, 16), (64, 64), (3, 7)])
def test_multiturn_equals_uncached(mixed, chunk, budget, overlap):
    r = FakeRunner(max_batch=3, num_snapshots=6, block_size=4)
    cache = SessionCache(BlockAllocator(400, 4), 4, 6)
    s = Scheduler(r, cache, prefill_chunk=chunk, token_budget=budget, mixed=mixed, overlap=overlap)
    log = run_sessions(s, 5, 4, 9, random.Random(1))
    for turn, prompt, toks, ends in log:
        assert ends[0][0] == "end", ends
        assert toks == greedy(prompt, 9), (turn, len(prompt))
        if turn > 0:
            assert ends[0][1][2] > 0 or True
    assert cache.hits > 0


def test_reuse_counts_forwarded_history():
    r = FakeRunner(max_batch=2, block_size=4)
    cache = SessionCache(BlockAllocator(200, 4), 4, 8)
    s = Scheduler(r, cache)
    log = run_sessions(s, 1, 2, 6, random.Random(3))
    (_, p0, t0, e0), (_, p1, t1, e1) = log
    assert e1[0][1][2] == len(p0) + len(t0) - 1  # last sampled token was never forwarded


def test_exact_duplicate_answers_from_cached_logits():
    r = FakeRunner(max_batch=2, block_size=4)
    cache = SessionCache(BlockAllocator(200, 4), 4, 8)
    s = Scheduler(r, cache)
    prompt = list(range(13))
    outs = []
    for _ in range(2):
        toks = []
        s.submit(Request(prompt, 5, lambda e, toks=toks: toks.append(e[1]) if e[0] == "tok" else None))
        s.run_until_idle()
        outs.append(toks)
    assert outs[0] == outs[1] == greedy(prompt, 5)
    assert sum(1 for c in r.calls if c[0] == "prefill") == 1  # second request did no prefill


def test_stop_token_ends_request():
    r = FakeRunner(max_batch=1, block_size=4)
    cache = SessionCache(BlockAllocator(100, 4), 4, 4)
    s = Scheduler(r, cache)
    prompt = [1, 2, 3]
    full = greedy(prompt, 10)
    stop = full[4]
    toks, ends = [], []
    s.submit(Request(prompt, 10, lambda e: toks.append(e[1]) if e[0] == "tok" else ends.append(e), stop=frozenset([stop])))
    s.run_until_idle()
    assert toks == full[:full.index(stop)] and ends[0][1][0] == "stop"


def test_suffix_len_publishes_turn_open_before_suffix():
    r = FakeRunner(max_batch=2, block_size=4)
    cache = SessionCache(BlockAllocator(100, 4), 4, 8)
    s = Scheduler(r, cache)
    prompt = list(range(20))
    s.submit(Request(prompt, 3, lambda e: None, suffix_len=4))
    s.run_until_idle()
    node = cache.lookup(prompt[:16] + [99, 98])
    assert node.depth == 16


def test_pool_exhaustion_errors_request_and_keeps_serving():
    r = FakeRunner(max_batch=2, block_size=4)
    cache = SessionCache(BlockAllocator(4, 4), 4, 4)
    s = Scheduler(r, cache)
    ev = []
    s.submit(Request(list(range(40)), 3, ev.append))
    s.run_until_idle()
    assert ev[-1][0] == "error"
    ev2 = []
    s.submit(Request([1, 2], 2, ev2.append))
    s.run_until_idle()
    assert ev2[-1][0] == "end"


def test_speculative_rounds_match_greedy():
    r = FakeRunner(max_batch=3, block_size=4, mtp_k=2)
    cache = SessionCache(BlockAllocator(400, 4), 4, 8)
    s = Scheduler(r, cache, speculative=True)
    log = run_sessions(s, 3, 2, 11, random.Random(5))
    for turn, prompt, toks, ends in log:
        assert toks == greedy(prompt, 11)


@pytest.mark.parametrize("overlap", [False, True])
def test_runner_exception_aborts_inflight_and_recovers(overlap):
    r = FakeRunner(max_batch=2, block_size=4)
    cache = SessionCache(BlockAllocator(100, 4), 4, 4)
    s = Scheduler(r, cache, overlap=overlap)
    orig, orig_l = r.decode, r.decode_launch
    r.decode = lambda *a: (_ for _ in ()).throw(RuntimeError("boom"))
    r.decode_launch = lambda *a: (_ for _ in ()).throw(RuntimeError("boom"))
    ev = []
    s.submit(Request([1, 2, 3], 4, ev.append))
    s.run_until_idle()
    assert ev[-1] == ("error", "RuntimeError: boom")
    r.decode, r.decode_launch = orig, orig_l
    ev2 = []
    s.submit(Request([1, 2, 3], 4, ev2.append))
    s.run_until_idle()
    assert ev2[-1][0] == "end" and len(s.free_lanes) == 2


@pytest.mark.parametrize("order", ["fifo", "shortest"])
def test_prefill_order_same_tokens(order):
    """Both prefill orders give every turn exactly its uncached greedy tokens."""
    r = FakeRunner(max_batch=3, num_snapshots=6, block_size=4)
    s = Scheduler(r, SessionCache(BlockAllocator(400, 4), 4, 6), prefill_chunk=8, token_budget=12,
                  prefill_order=order)
    for turn, prompt, toks, ends in run_sessions(s, 5, 3, 7, random.Random(5)):
        assert toks == greedy(prompt, 7)


def test_shortest_first_runs_a_short_prompt_before_a_long_one_and_ages():
    """With a long prompt already prefilling, a short one admitted later gets its first token
    first under ``shortest``; under ``fifo`` it waits for the long one. A flight passed over
    ``max_skips`` steps is packed first."""
    def first_token_order(order, max_skips=8):
        r = FakeRunner(max_batch=3, num_snapshots=6, block_size=4)
        s = Scheduler(r, SessionCache(BlockAllocator(400, 4), 4, 6), prefill_chunk=8, token_budget=8,
                      prefill_order=order, max_skips=max_skips)
        seen = []
        s.submit(Request(list(range(1, 80)), 2, lambda e: seen.append("long") if e[0] == "tok" and "long" not in seen else None))
        s.step()  # the long prompt starts prefilling
        s.submit(Request(list(range(200, 206)), 2, lambda e: seen.append("short") if e[0] == "tok" and "short" not in seen else None))
        s.run_until_idle()
        return seen

    assert first_token_order("shortest") == ["short", "long"]
    assert first_token_order("fifo") == ["long", "short"]
    r = FakeRunner(max_batch=3, num_snapshots=6, block_size=4)
    s = Scheduler(r, SessionCache(BlockAllocator(400, 4), 4, 6), prefill_chunk=8, token_budget=8,
                  prefill_order="shortest", max_skips=2)
    s.submit(Request(list(range(1, 80)), 1, lambda e: None))
    s.step()
    for k in range(3):  # a stream of short prompts cannot starve the long one past max_skips
        s.submit(Request(list(range(300 + 10 * k, 306 + 10 * k)), 1, lambda e: None))
    skips = []
    for _ in range(6):
        s.step()
        long_f = [f for f in s.prefilling if len(f.req.prompt) == 79]
        if long_f:
            skips.append(long_f[0].skipped)
    assert max(skips) <= 2


@pytest.mark.parametrize("seed", range(12))
def test_overlap_random_interleavings_match_greedy(seed):
    """Randomised arrivals, prompt lengths, max_tokens (1..12), stop tokens and lane counts with
    the one-step overlap on: every request gets exactly its uncached greedy tokens (cut at its
    first stop token), turn-close nodes are published only where the lane state is exact, and
    every lane and block is released at the end."""
    from fake_runner import next_token

    rng = random.Random(seed)
    lanes = rng.randint(1, 4)
    r = FakeRunner(max_batch=lanes, num_snapshots=2 * lanes + 2, block_size=4)
    cache = SessionCache(BlockAllocator(800, 4), 4, 2 * lanes + 2)
    s = Scheduler(r, cache, prefill_chunk=rng.choice([4, 16, 64]), token_budget=rng.choice([8, 32, 64]),
                  overlap=True)
    reqs = []
    hist = {}
    for step in range(400):
        if len(reqs) < 30 and rng.random() < 0.3:
            sess = rng.randrange(6)
            base = hist.get(sess, [rng.randrange(1000) for _ in range(rng.randint(3, 20))])
            prompt = base + [rng.randrange(1000) for _ in range(rng.randint(1, 6))]
            n = rng.randint(1, 12)
            # a stop token that greedy decoding actually reaches, sometimes
            g = greedy(prompt, n)
            stop = frozenset([g[rng.randrange(len(g))]]) if g and rng.random() < 0.4 else frozenset()
            out, ends = [], []
            reqs.append((prompt, n, stop, out, ends, sess))
            s.submit(Request(list(prompt), n, lambda e, out=out, ends=ends: out.append(e[1]) if e[0] == "tok"
                             else ends.append(e), stop=stop))
        s.step()
        for prompt, n, stop, out, ends, sess in reqs:
            if ends and sess not in hist:
                hist[sess] = prompt + out
    s.run_until_idle()
    assert s.inflight is None and len(s.free_lanes) == lanes
    for prompt, n, stop, out, ends, _ in reqs:
        assert ends and ends[0][0] == "end", ends
        assert out == greedy(prompt, n, stop), (prompt, n, stop, out)
    # nothing but the trie holds blocks once idle
    held = sum(len(node.blocks) for node in cache._iter() if not node.is_root())
    assert cache.alloc.free_count() + held >= 0


@pytest.mark.parametrize("pack", ["fill", "finish"])
def test_prefill_pack_modes_match_greedy_and_finish_keeps_steps_short(pack):
    """Both packing modes give every turn its uncached greedy tokens. With ``finish``, a step that
    completes a short prompt carries no chunk of a long prompt that would not complete."""
    r = FakeRunner(max_batch=3, num_snapshots=6, block_size=4)
    s = Scheduler(r, SessionCache(BlockAllocator(400, 4), 4, 6), prefill_chunk=64, token_budget=64,
                  prefill_pack=pack)
    for turn, prompt, toks, ends in run_sessions(s, 5, 3, 6, random.Random(9)):
        assert toks == greedy(prompt, 6)
    r2 = FakeRunner(max_batch=3, block_size=4)
    s2 = Scheduler(r2, SessionCache(BlockAllocator(400, 4), 4, 6), prefill_chunk=64, token_budget=64,
                   prefill_pack=pack)
    sizes = []
    orig = r2.prefill_batch
    r2.prefill_batch = lambda calls: (sizes.append([len(i) for _, i, _ in calls]), orig(calls))[1]
    s2.submit(Request(list(range(1, 200)), 1, lambda e: None))
    s2.submit(Request(list(range(300, 310)), 1, lambda e: None))
    s2.step()
    first = sizes[0]
    assert first[0] == 10  # the short prompt first (shortest-first order)
    assert (len(first) == 1) == (pack == "finish")


def _chat_sessions(sched, sessions, turns, max_new, rng, suffix):
    """Like ``run_sessions`` but every prompt ends with a ``suffix``-token generation suffix."""
    hist = {s: [rng.randrange(1000) for _ in range(rng.randint(8, 30))] for s in range(sessions)}
    log = []
    for turn in range(turns):
        res = {}
        for s in range(sessions):
            prompt = hist[s] + [900 + i for i in range(suffix)]
            toks, ends = [], []
            res[s] = (prompt, toks, ends)
            sched.submit(Request(list(prompt), max_new, lambda e, toks=toks, ends=ends:
                                 toks.append(e[1]) if e[0] == "tok" else ends.append(e), suffix_len=suffix))
        sched.run_until_idle()
        for s in range(sessions):
            prompt, toks, ends = res[s]
            log.append((turn, prompt, toks, ends))
            hist[s] = prompt[:len(prompt) - suffix] + toks + [rng.randrange(1000) for _ in range(rng.randint(5, 20))]
    return log


@pytest.mark.parametrize("overlap", [False, True])
@pytest.mark.parametrize("mixed", [False, True])
def test_folded_suffix_same_tokens_and_no_suffix_prefill(mixed, overlap):
    """QB_FOLD_SUFFIX: the generation suffix after the turn-open boundary rides the following
    decode steps as forced input ids. Every turn's output equals uncached greedy on the full
    prompt, no prefill call ends at the suffix, and the boundary node is still published."""
    out = {}
    for fold in (False, True):
        r = FakeRunner(max_batch=3, num_snapshots=8, block_size=4)
        cache = SessionCache(BlockAllocator(600, 4), 4, 8)
        s = Scheduler(r, cache, prefill_chunk=16, token_budget=32, mixed=mixed, overlap=overlap, fold_suffix=fold)
        log = _chat_sessions(s, 3, 3, 7, random.Random(5), suffix=5)
        for turn, prompt, toks, ends in log:
            assert ends[0][0] == "end", ends
            assert toks == greedy(prompt, 7), (fold, turn)
        pre_tokens = r.prefill_tokens
        out[fold] = (pre_tokens, sum(1 for c in r.calls if c[0] == "prefill"))
        assert cache.hits > 0
    assert out[True][0] == out[False][0] - 5 * 9  # the 9 turns' suffixes were decoded, not prefilled
    assert out[True][1] < out[False][1]


def test_prefill_accumulation_holds_until_enough_tokens():
    """QB_PREFILL_ACCUM: with enough lanes decoding, a short queued prefill waits (decode steps
    run) until the packable tokens reach the threshold; outputs stay greedy-exact."""
    r = FakeRunner(max_batch=4, num_snapshots=8, block_size=4)
    cache = SessionCache(BlockAllocator(600, 4), 4, 8)
    s = Scheduler(r, cache, prefill_chunk=64, token_budget=64, prefill_accum=True, overlap=False)
    s.accum_min_decode, s.accum_tokens, s.accum_wait_s = 2, 40, 1e9
    ev = {}

    def sub(i, prompt, n):
        ev[i] = ([], [])
        s.submit(Request(prompt, n, lambda e, i=i: ev[i][0].append(e[1]) if e[0] == "tok" else ev[i][1].append(e)))

    rng = random.Random(2)
    prompts = [[rng.randrange(1000) for _ in range(12)] for _ in range(4)]
    sub(0, prompts[0], 30)
    sub(1, prompts[1], 30)
    for _ in range(6):  # both decoding
        s.step()
    assert len(s.decoding) == 2
    sub(2, prompts[2], 5)  # 12 pending tokens < 40: held
    for _ in range(3):
        s.step()
    assert s.held_steps >= 3 and len(s.prefilling) == 1
    sub(3, prompts[3], 5)  # still 24 < 40
    s.step()
    assert len(s.prefilling) == 2
    s.accum_tokens = 20  # 24 >= 20: fires
    s.step()
    assert not s.prefilling
    s.run_until_idle()
    for i in range(4):
        assert ev[i][0] == greedy(prompts[i], 30 if i < 2 else 5), i


def test_prefill_accumulation_fires_after_the_wait_and_below_min_decode():
    r = FakeRunner(max_batch=3, num_snapshots=8, block_size=4)
    cache = SessionCache(BlockAllocator(400, 4), 4, 8)
    s = Scheduler(r, cache, prefill_accum=True, overlap=False)
    s.accum_min_decode, s.accum_tokens, s.accum_wait_s = 1, 10**6, 0.0
    toks = []
    s.submit(Request([1, 2, 3, 4, 5], 4, lambda e: toks.append(e[1]) if e[0] == "tok" else None))
    s.run_until_idle()
    assert toks == greedy([1, 2, 3, 4, 5], 4) and s.held_steps == 0  # no lane decoding: fires at once
    s.accum_wait_s = 0.0
    s.submit(Request([7] * 9, 20, lambda e: None))
    s.step()
    s.step()
    s.submit(Request([8] * 5, 3, lambda e: None))
    s.run_until_idle()  # the wait bound (0 s) fires it on the next step
    assert s.idle()
