"""Sharding independent utterances across the GPUs of one box.

Every utterance is an independent unit of the path (tokens + style ->
PCM), so multi-GPU runs need no collective in the data path: each GPU gets
whole utterances, runs them through its own rk_ctx, and the host gathers the
PCM back in the original order.

* Bucketing: utterances are grouped by (token count, decoder-frame bucket
  L_b = ceil(L / 32) * 32), the keys the reference caches its CUDA graphs on
  (src/rokoko_f16.cpp:790-802, 672-682), so each GPU replays a small set of
  graphs.
* Assignment: greedy longest-processing-time: buckets in decreasing cost
  order, each to the rank with the least load so far.  Cost is linear in the
  frame count (decoder FLOPs are linear in L) plus a per-token term for the
  front half; a bucket larger than a fair share is split so that one bucket
  cannot leave the other ranks idle.
* Gather: with one process per GPU (torchrun) the ranks exchange only
  (utterance, sample count) over the host process group; rank 0 sizes one
  node-local file of the total (in $RK_GATHER_DIR, else /dev/shm) and writes a
  random token beside it; when every rank reads the token back (they share the
  file system, whatever their host names say), the other ranks write their PCM
  at their utterances' offsets (original order) and rank 0 keeps its own
  arrays, so no sample crosses a socket.  Otherwise every rank falls back to a
  pickled gather over the process group.  With one process and one host thread per
  GPU the threads write into a shared list.  Nothing here is a device
  collective.
"""
from __future__ import annotations

import os
import tempfile
import threading
import uuid
from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np

L_BUCKET = 32
FRAME_COST = 1.0    # decoder + generator, per frame
TOKEN_COST = 0.15   # ALBERT + text encoder + duration encoder, per token (relative)


@dataclass
class Unit:
    index: int   # position in the caller's list
    T: int       # token count (with BOS/EOS)
    L: int       # decoder frames (sum of durations)

    @property
    def L_b(self) -> int:
        return (self.L + L_BUCKET - 1) // L_BUCKET * L_BUCKET

    @property
    def cost(self) -> float:
        return FRAME_COST * self.L_b + TOKEN_COST * self.T


def units(utterances: Sequence) -> list[Unit]:
    """Units from objects with .tokens and .durations (rokoko_b200.configs.Utterance)."""
    return [Unit(i, int(u.tokens.shape[0]), int(np.asarray(u.durations).sum())) for i, u in enumerate(utterances)]


def plan(items: Sequence[Unit], world: int) -> list[list[int]]:
    """Indices per rank.  Deterministic: every rank computes the same plan."""
    if world < 1:
        raise ValueError("world must be >= 1")
    buckets: dict[tuple[int, int], list[Unit]] = {}
    for u in items:
        buckets.setdefault((u.T, u.L_b), []).append(u)
    total = sum(u.cost for u in items)
    share = total / world if world else total
    pieces: list[list[Unit]] = []
    for key in sorted(buckets):
        b = sorted(buckets[key], key=lambda u: u.index)
        cur: list[Unit] = []
        for u in b:  # split buckets larger than half a fair share
            if cur and sum(x.cost for x in cur) + u.cost > 0.5 * share:
                pieces.append(cur)
                cur = []
            cur.append(u)
        if cur:
            pieces.append(cur)
    pieces.sort(key=lambda p: (-sum(u.cost for u in p), p[0].index))
    load = [0.0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for p in pieces:
        r = min(range(world), key=lambda k: (load[k], k))
        load[r] += sum(u.cost for u in p)
        out[r].extend(u.index for u in p)
    for r in range(world):  # run each rank's utterances bucket by bucket
        out[r].sort(key=lambda i: (items[i].T, items[i].L_b, i))
    return out


def imbalance(items: Sequence[Unit], assignment: list[list[int]]) -> float:
    """max rank load / mean rank load (1.0 = perfect balance)."""
    loads = [sum(items[i].cost for i in idx) for idx in assignment]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0


def run_rank(synth: Callable[[int], np.ndarray], indices: Sequence[int]) -> list[tuple[int, np.ndarray]]:
    """Run this rank's utterances in order; synth(i) -> PCM of utterance i."""
    return [(i, synth(i)) for i in indices]


def _shm_dir() -> str:
    d = os.environ.get("RK_GATHER_DIR")
    if d:
        return d
    return "/dev/shm" if os.path.isdir("/dev/shm") and os.access("/dev/shm", os.W_OK) else tempfile.gettempdir()


def gather_pcm(local: list[tuple[int, np.ndarray]], n_total: int, group=None) -> list[np.ndarray] | None:
    """Gather of (index, PCM) pairs to rank 0 over the host process group.
    Returns the PCM list in original order on rank 0, None elsewhere.  Ranks
    on one host write into a shared node-local file (no sample crosses a
    socket); otherwise the PCM is pickled through the group.  Without an
    initialised process group, returns `local` in order."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        out: list = [None] * n_total
        for i, pcm in local:
            out[i] = pcm
        return out
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    meta = [None] * world
    dist.all_gather_object(meta, [(int(i), int(p.shape[0])) for i, p in local], group=group)
    lengths = [-1] * n_total
    for part in meta:
        for i, n in part:
            lengths[i] = n
    missing = [i for i, n in enumerate(lengths) if n < 0]
    if missing:
        raise RuntimeError(f"gather_pcm: no PCM for utterances {missing[:8]}")
    done, out = _gather_shared_file(local, lengths, rank, world, group)
    if done:
        return out
    bucket = [None] * world if rank == 0 else None
    dist.gather_object(local, bucket, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_total
    for part in bucket:
        for i, pcm in part:
            out[i] = pcm
    return out


def _gather_shared_file(local, lengths: list[int], rank: int, world: int, group):
    """Node-local gather: rank 0 sizes a file for every sample (float32, original
    order) and writes a random token beside it; if every rank reads the token
    back they share the file, the other ranks write their utterances at their
    offsets with pwrite, and rank 0 maps the file copy-on-write (its name removed
    once mapped) and keeps its own arrays.  Returns (True, PCM list on rank 0 /
    None elsewhere), or (False, None) on every rank when some rank cannot see
    the file (the caller then gathers over the process group)."""
    import torch.distributed as dist
    offsets = np.zeros(len(lengths) + 1, np.int64)
    np.cumsum(np.asarray(lengths, np.int64), out=offsets[1:])
    total = int(offsets[-1])
    info = [None, None]
    if rank == 0:
        info[0] = f"rk_pcm_{os.getpid()}_{uuid.uuid4().hex}"
        info[1] = uuid.uuid4().hex
    dist.broadcast_object_list(info, src=0, group=group)
    name, token = info
    path = os.path.join(_shm_dir(), name)  # every rank looks in its own node-local directory
    if rank == 0:
        with open(path, "wb") as f:
            f.truncate(max(total, 1) * 4)
        with open(path + ".id", "w") as f:
            f.write(token)
    dist.barrier(group=group)
    try:
        with open(path + ".id") as f:
            sees = f.read() == token
    except OSError:
        sees = False
    seen = [None] * world
    dist.all_gather_object(seen, sees, group=group)
    try:
        if not all(seen):
            return False, None
        if rank != 0 and local and total:
            fd = os.open(path, os.O_WRONLY)
            try:
                for i, pcm in local:
                    view = memoryview(np.ascontiguousarray(pcm, dtype=np.float32).reshape(-1)).cast("B")
                    off = int(offsets[i]) * 4
                    while len(view):
                        n = os.pwrite(fd, view, off)
                        view, off = view[n:], off + n
            finally:
                os.close(fd)
        dist.barrier(group=group)
        if rank != 0:
            return True, None
        mine = {int(i): np.asarray(p, np.float32).reshape(-1) for i, p in local}
        if total == 0:
            return True, [np.zeros(0, np.float32) for _ in lengths]
        flat = np.memmap(path, dtype=np.float32, mode="c", shape=(total,))
        return True, [mine[i] if i in mine else flat[offsets[i]:offsets[i + 1]] for i in range(len(lengths))]
    finally:
        if rank == 0:
            for f in (path, path + ".id"):
                try:
                    os.remove(f)
                except FileNotFoundError:
                    pass


def run_threads(synths: Sequence[Callable[[int], np.ndarray]], items: Sequence[Unit]) -> list[np.ndarray]:
    """One process, one host thread per GPU: synths[r](i) runs utterance i on
    GPU r (its own rk_ctx).  Returns PCM in original order."""
    assignment = plan(items, len(synths))
    out: list = [None] * len(items)
    errors: list[BaseException] = []

    def worker(r: int) -> None:
        try:
            for i, pcm in run_rank(synths[r], assignment[r]):
                out[i] = pcm
        except BaseException as e:  # surfaced after join
            errors.append(e)

    th = [threading.Thread(target=worker, args=(r,)) for r in range(len(synths))]
    for t in th:
        t.start()
    for t in th:
        t.join()
    if errors:
        raise errors[0]
    return out
