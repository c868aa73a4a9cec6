"""SPMD command protocol: rank 0 drives, every other rank mirrors.

Rank 0 runs the scheduler (and the HTTP server). ``Broadcaster`` implements the scheduler's
``Runner`` by sending every state-changing call to the other ranks before running it locally;
``serve_worker`` is the loop the other ranks run, applying each received call to their own
``Model`` shard. Because every rank applies the same calls in the same order, their block
tables, lane states and snapshot pools stay identical, and the collectives inside each forward
line up. Only rank 0 samples; its results are never sent back.

Wire format: a command is ``(op, args)`` pickled into a uint8 tensor, sent as an int64 length
followed by the payload over a gloo (host) group, so rank 0 can enqueue the next command while
the workers are still computing the previous one. Reference behaviour: ``tp_driver.py:54-607``
(``Op``, ``Command``, ``Channel``, ``Broadcaster``, ``apply``, ``serve_worker``,
``pool_handshake``).
"""

from __future__ import annotations

import enum
import hashlib
import pickle

import torch
import torch.distributed as dist


class Op(enum.IntEnum):
    BEGIN = 1
    ATTACH_BLOCKS = 2
    EXTEND_BLOCKS = 3
    COPY_BLOCK = 4
    SAVE_SNAPSHOT = 5
    LOAD_SNAPSHOT = 6
    PREFILL_BATCH = 7
    DECODE = 8
    DECODE_MIXED = 9
    SPECULATIVE_DECODE = 10
    SCORE = 11
    WARMUP = 12
    SET_FAULT = 13
    CALL = 14  # generic named method (rarely used control calls)
    SHUTDOWN = 15
    DECODE_LAUNCH = 16


class PoolMismatchError(RuntimeError):
    """Ranks booted with different pool geometry or config; serving would desynchronise."""


class Channel:
    """Host-side broadcast of pickled commands from rank 0 over a gloo group."""

    def __init__(self, group=None, src: int = 0):
        self.group = group
        self.src = src

    def send(self, op: Op, args: tuple) -> None:
        raw = pickle.dumps((int(op), args), protocol=pickle.HIGHEST_PROTOCOL)
        n = torch.tensor([len(raw)], dtype=torch.int64)
        dist.broadcast(n, self.src, group=self.group)
        dist.broadcast(torch.frombuffer(bytearray(raw), dtype=torch.uint8), self.src, group=self.group)

    def recv(self) -> tuple[Op, tuple]:
        n = torch.zeros(1, dtype=torch.int64)
        dist.broadcast(n, self.src, group=self.group)
        buf = torch.empty(int(n.item()), dtype=torch.uint8)
        dist.broadcast(buf, self.src, group=self.group)
        op, args = pickle.loads(buf.numpy().tobytes())
        return Op(op), args


def open_channel(world: int, rank: int, group, device_type: str = "cuda"):
    """The command channel for this node: the shared-memory ring (``QB_CMD_CHANNEL=shm``, the
    default) or the gloo broadcast channel (``gloo``). Every rank must call this."""
    from ..utils import flags

    if world <= 1:
        return None
    if flags.get("QB_CMD_CHANNEL") == "shm":
        from .shm_channel import make_channel

        ch = make_channel(world, rank, group)
        if device_type != "cuda":
            ch.poll_s = 5e-5  # CPU ranks share cores with the compute: do not spin hard
        return ch
    return Channel(group)


def command_group(world: int):
    """A gloo group over all ranks for the command channel (every rank must call this)."""
    if world <= 1:
        return None
    return dist.new_group(list(range(world)), backend="gloo")


def apply(model, op: Op, args: tuple):
    if op == Op.BEGIN:
        return model.begin(*args)
    if op == Op.ATTACH_BLOCKS:
        return model.attach_blocks(*args)
    if op == Op.EXTEND_BLOCKS:
        return model.extend_blocks(*args)
    if op == Op.COPY_BLOCK:
        return model.copy_block(*args)
    if op == Op.SAVE_SNAPSHOT:
        return model.save_snapshot(*args)
    if op == Op.LOAD_SNAPSHOT:
        return model.load_snapshot(*args)
    if op == Op.PREFILL_BATCH:
        return model.prefill_batch(*args)
    if op == Op.DECODE:
        return model.decode(*args)
    if op == Op.DECODE_MIXED:
        return model.decode_mixed(*args)
    if op == Op.DECODE_LAUNCH:
        return model.decode_launch(*args)
    if op == Op.SPECULATIVE_DECODE:
        return model.speculative_decode(*args)
    if op == Op.SCORE:
        return model.score(*args)
    if op == Op.WARMUP:
        return model.warmup(*args)
    if op == Op.SET_FAULT:
        name, value = args
        if value is None:
            model.fault.pop(name, None)
        else:
            model.fault[name] = value
        return None
    if op == Op.CALL:
        name, a, kw = args
        return getattr(model, name)(*a, **kw)
    raise ValueError(f"unknown op {op}")


STEP_OPS = (Op.PREFILL_BATCH, Op.DECODE, Op.DECODE_MIXED, Op.SPECULATIVE_DECODE, Op.SCORE, Op.DECODE_LAUNCH)


def serve_worker(model, channel: Channel) -> int:
    """Apply rank 0's commands until SHUTDOWN; returns the number of commands applied. A nonzero
    device status word (``utils.devstatus``) ends the worker with ``DeviceStatusError``."""
    n = 0
    watch = getattr(model, "status_watch", None)
    while True:
        op, args = channel.recv()
        if op == Op.SHUTDOWN:
            return n
        apply(model, op, args)
        if watch is not None and op in STEP_OPS:
            watch.step()
        n += 1


class Broadcaster:
    """``Runner`` on rank 0 that mirrors every call to the other ranks first."""

    def __init__(self, model, channel: Channel | None):
        self.model = model
        self.channel = channel
        self.max_batch = model.max_batch
        self.max_seq = model.max_seq
        self.block_size = model.block_size

    @property
    def status_watch(self):
        return getattr(self.model, "status_watch", None)

    def _send(self, op: Op, *args):
        if self.channel is not None:
            self.channel.send(op, args)

    # -- state-changing calls (mirrored)
    def begin(self, lane):
        self._send(Op.BEGIN, lane)
        return self.model.begin(lane)

    def attach_blocks(self, lane, blocks):
        blocks = list(blocks)
        self._send(Op.ATTACH_BLOCKS, lane, blocks)
        return self.model.attach_blocks(lane, blocks)

    def extend_blocks(self, grants):
        grants = [tuple(g) for g in grants]
        self._send(Op.EXTEND_BLOCKS, grants)
        return self.model.extend_blocks(grants)

    def copy_block(self, dst, src, filled):
        self._send(Op.COPY_BLOCK, dst, src, filled)
        return self.model.copy_block(dst, src, filled)

    def save_snapshot(self, lane, snap):
        self._send(Op.SAVE_SNAPSHOT, lane, snap)
        return self.model.save_snapshot(lane, snap)

    def load_snapshot(self, lane, snap):
        self._send(Op.LOAD_SNAPSHOT, lane, snap)
        return self.model.load_snapshot(lane, snap)

    def prefill_batch(self, calls):
        calls = [(l, list(ids), s) for l, ids, s in calls]
        self._send(Op.PREFILL_BATCH, calls)
        return self.model.prefill_batch(calls)

    def prefill(self, lane, ids, start):
        return self.prefill_batch([(lane, ids, start)])[0]

    def decode(self, lanes, tokens, positions):
        lanes, tokens, positions = list(lanes), [int(t) for t in tokens], list(positions)
        self._send(Op.DECODE, lanes, tokens, positions)
        return self.model.decode(lanes, tokens, positions)

    def decode_launch(self, lanes, tokens, positions, src_rows, keep_rows=()):
        args = (list(lanes), [int(t) for t in tokens], list(positions), list(src_rows), list(keep_rows))
        self._send(Op.DECODE_LAUNCH, *args)
        return self.model.decode_launch(*args)

    def decode_collect(self, handle):
        return self.model.decode_collect(handle)

    def decode_kept(self, handle):
        return self.model.decode_kept(handle)

    def decode_mixed(self, lanes, tokens, positions, calls):
        lanes, tokens, positions = list(lanes), [int(t) for t in tokens], list(positions)
        calls = [(l, list(ids), s) for l, ids, s in calls]
        self._send(Op.DECODE_MIXED, lanes, tokens, positions, calls)
        return self.model.decode_mixed(lanes, tokens, positions, calls)

    def speculative_decode(self, lanes, tokens, positions, budgets, stops):
        args = (list(lanes), [int(t) for t in tokens], list(positions), list(budgets), [list(s) for s in stops])
        self._send(Op.SPECULATIVE_DECODE, *args)
        return self.model.speculative_decode(*args)

    def score(self, lane, ids, cs):
        self._send(Op.SCORE, lane, list(ids), cs)
        return self.model.score(lane, list(ids), cs)

    def warmup(self):
        self._send(Op.WARMUP)
        return self.model.warmup()

    def set_fault(self, name, value):
        self._send(Op.SET_FAULT, name, value)
        apply(self.model, Op.SET_FAULT, (name, value))

    def shutdown(self):
        self._send(Op.SHUTDOWN)

    # -- local-only calls (no device state change on other ranks)
    def lane_blocks(self, lane):
        return self.model.lane_blocks(lane)

    def lane_block_count(self, lane):
        return self.model.lane_block_count(lane)

    def cache_node_logits(self, snap, logits):
        return self.model.cache_node_logits(snap, logits)

    def cached_node_logits(self, snap):
        return self.model.cached_node_logits(snap)

    def decode_row(self, logits, row):
        return self.model.decode_row(logits, row)

    def sample_batch(self, logits, temps):
        return self.model.sample_batch(logits, temps)

    def decode_tokens_per_step(self):
        return self.model.decode_tokens_per_step()


def pool_signature(model) -> str:
    """Hash of everything that must agree across ranks for the protocol to stay in lockstep."""
    from ..utils import flags

    d = (model.cfg.to_json(), model.max_batch, model.max_seq, model.block_size, model.num_blocks,
         model.num_snapshots, model.plan.world, flags.signature())
    return hashlib.sha1(repr(d).encode()).hexdigest()


def pool_handshake(model, group=None) -> None:
    """All ranks compare ``pool_signature``; any difference raises ``PoolMismatchError``."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    sig = pool_signature(model)
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, sig, group=group)
    if len(set(out)) != 1:
        raise PoolMismatchError(f"pool configuration differs across ranks: {out}")
