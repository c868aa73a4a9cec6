"""A deterministic ``Runner`` whose model is a pure function of the token history.

Any mistake in the scheduler's cache bookkeeping (wrong snapshot, wrong start position, a
missing block) changes the history a lane sees and therefore the tokens it emits, so the
scheduler can be checked against plain uncached generation without any tensors."""

from __future__ import annotations

import hashlib

V = 1000


def next_token(history) -> int:
    h = hashlib.blake2b(repr(tuple(history)).encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") % V


class Logits:
    def __init__(self, rows):
        self.rows = rows  # list of histories

    def __getitem__(self, i):
        return Logits([self.rows[i]])


def greedy(prompt, n, stop=()):
    hist, out = list(prompt), []
    for _ in range(n):
        t = next_token(hist)
        if t in stop:
            break
        out.append(t)
        hist.append(t)
    return out


class FakeRunner:
    def __init__(self, max_batch=4, num_snapshots=8, block_size=4, max_seq=10**6, mtp_k=0):
        self.max_batch, self.block_size, self.max_seq = max_batch, block_size, max_seq
        self.hist = [[] for _ in range(max_batch)]
        self.tables = [[] for _ in range(max_batch)]
        self.snaps = {}
        self.node_logits = {}
        self.calls = []
        self.prefill_tokens = 0
        self.mtp_k = mtp_k

    def begin(self, lane):
        self.hist[lane] = []
        self.tables[lane] = []

    def lane_blocks(self, lane):
        return tuple(self.tables[lane])

    def lane_block_count(self, lane):
        return len(self.tables[lane])

    def attach_blocks(self, lane, blocks):
        self.tables[lane] = list(blocks)

    def extend_blocks(self, grants):
        for lane, b in grants:
            self.tables[lane].append(b)

    def copy_block(self, dst, src, filled):
        self.calls.append(("cow", dst, src, filled))

    def save_snapshot(self, lane, snap):
        self.snaps[snap] = list(self.hist[lane])

    def load_snapshot(self, lane, snap):
        self.hist[lane] = list(self.snaps[snap])

    def cache_node_logits(self, snap, logits):
        self.node_logits[snap] = logits

    def cached_node_logits(self, snap):
        return self.node_logits[snap]

    def _fwd(self, lane, ids, start):
        assert len(self.hist[lane]) == start, (lane, len(self.hist[lane]), start)
        assert len(self.tables[lane]) * self.block_size >= start + len(ids), "forward past the lane's blocks"
        self.hist[lane].extend(ids)
        return list(self.hist[lane])

    def prefill_batch(self, calls):
        self.calls.append(("prefill", len(calls)))
        self.prefill_tokens += sum(len(ids) for _, ids, _ in calls)
        return [Logits([self._fwd(l, ids, s)]) for l, ids, s in calls]

    def prefill(self, lane, ids, start):
        return self.prefill_batch([(lane, ids, start)])[0]

    def decode(self, lanes, tokens, positions):
        self.calls.append(("decode", len(lanes)))
        return Logits([self._fwd(l, [t], p) for l, t, p in zip(lanes, tokens, positions)])

    def decode_launch(self, lanes, tokens, positions, src_rows, keep_rows=()):
        """One-step overlap form of ``decode``: a token of -1 means "the previous launch's
        sampled id at row ``src_rows[i]``" (the device feedback of the real runner)."""
        self.calls.append(("launch", len(lanes)))
        prev = getattr(self, "_launched_ids", None)
        toks = [prev[s] if t < 0 else t for t, s in zip(tokens, src_rows)]
        rows = [self._fwd(l, [t], p) for l, t, p in zip(lanes, toks, positions)]
        ids = [next_token(h) for h in rows]
        self._launched_ids = ids
        return (ids, {i: Logits([rows[i]]) for i in keep_rows})

    def decode_collect(self, handle):
        return list(handle[0])

    def decode_kept(self, handle):
        return handle[1]

    def decode_mixed(self, lanes, tokens, positions, calls):
        d = self.decode(lanes, tokens, positions)
        return d, self.prefill_batch(calls)

    def decode_row(self, logits, i):
        return logits[i]

    def sample_batch(self, logits, temps):
        return [next_token(h) for h in logits.rows]

    def decode_tokens_per_step(self):
        return self.mtp_k + 1

    def speculative_decode(self, lanes, tokens, positions, budgets, stops):
        out = []
        for l, t, p, b, st in zip(lanes, tokens, positions, budgets, stops):
            hist = self._fwd(l, [t], p)
            got = []
            for _ in range(self.mtp_k + 1):
                nt = next_token(hist)
                got.append(nt)
                if nt in st or len(got) >= b:
                    break
                hist = hist + [nt]
            # state holds t plus every committed token except the last
            self.hist[l].extend(got[:-1])
            out.append(got)
        return out

    def score(self, lane, ids, cs):
        return [next_token(ids[:i]) for i in range(max(cs, 1), len(ids) + 1)]
