"""Box throughput over many utterances, one process per GPU.

    python -m rokoko_b200.boxbench [--count 1024] [--batch 32] [--fp32]
    python -m torch.distributed.run --nproc-per-node N -m rokoko_b200.boxbench ...

Workload: `count` utterances with token counts from a seeded truncated normal
(mean 120, sd 60, clipped to [16, 510]), durations U[2, 8], a seeded style
vector each (configs.config4), FP16 weights (the KOKO v2 file) unless --fp32.
The utterances are sharded over the ranks by rokoko_b200.shard (length
buckets, greedy longest-processing-time; no collective in the data path);
each rank runs its share through rk_encode + rk_decode in batches of `batch`
utterances in the plan's bucket order, taken from a shared queue by `contexts`
rk_ctx on the same GPU, each driven by its own host thread, so that one context's
latency-bound front half (ALBERT, BiLSTM recurrences) overlaps another's
SM-saturating decode; rank 0 gathers the PCM on the host (ranks on one host
write it into one shared node-local file, rokoko_b200.shard.gather_pcm).

Reported (rank 0, one JSON line): total audio seconds / wall time from the
first dispatch to the last PCM gathered, the per-rank maximum wall time, the
load imbalance of the shard plan and the front-half / decode split of rank 0.
Before the timed pass every rank runs one utterance of each decode-length
bucket of its share, so the timed pass replays cached decode graphs.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

import numpy as np


def _args(argv=None):
    p = argparse.ArgumentParser(prog="rokoko_b200.boxbench")
    p.add_argument("--count", type=int, default=1024)
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--fp32", action="store_true")
    p.add_argument("--contexts", type=int, default=2,
                   help="rk_ctx per GPU, each driven by its own host thread on alternating batches")
    return p.parse_args(argv)


def run_share(ctxs, utts, indices, batch: int, timings=None):
    """This rank's share `indices` of `utts` through rk_encode + rk_decode in
    batches of `batch` (in the given order), taken from a shared queue by the
    contexts `ctxs` (all on this rank's GPU), each context driven by its own
    host thread.  Returns [(index, PCM)] (context by context); `timings`, if given,
    receives [encode_s, decode_s] per context."""
    batches = [indices[k:k + batch] for k in range(0, len(indices), batch)]
    return run_batches(ctxs, utts, batches, timings)


def run_batches(ctxs, utts, batches, timings=None, nvtx: str | None = None, failures: list | None = None,
                max_tries: int = 2):
    """run_share over explicit batches (lists of indices into `utts`): every
    context's host thread takes the next batch not yet taken, so a context that
    drew short utterances takes more batches (the outputs do not depend on
    which context runs a batch).  nvtx: name of an NVTX range each host thread
    holds while it runs batches (NVTX ranges are per thread).

    Failure handling: a context whose encode or decode raises is taken out of
    service (its thread stops) and the batch goes back to the front of the
    queue for another context, up to `max_tries` attempts per batch; `failures`
    (if given) receives (context, batch, error text) for each failed attempt.
    The call raises when a batch has failed `max_tries` times or when no
    context is left in service."""
    import threading
    results = [[] for _ in ctxs]
    tim = [[0.0, 0.0] for _ in ctxs]
    fatal = []
    cond = threading.Condition()
    queue = list(range(len(batches)))[::-1]  # pop() from the end = next batch
    tries = [0] * len(batches)
    alive = [True] * len(ctxs)
    inflight = [0]

    def take():
        # the next batch; with the queue empty, wait while batches are in flight (one may come back)
        with cond:
            while True:
                if fatal:
                    return None
                if queue:
                    inflight[0] += 1
                    return queue.pop()
                if inflight[0] == 0:
                    return None
                cond.wait()

    def finished(c: int, bi: int, err) -> None:
        with cond:
            inflight[0] -= 1
            if err is not None:
                alive[c] = False
                tries[bi] += 1
                if failures is not None:
                    failures.append((c, bi, repr(err)))
                if tries[bi] >= max_tries or not any(alive):
                    fatal.append(err)
                else:
                    queue.append(bi)
            cond.notify_all()

    def worker(c: int) -> None:
        if nvtx:
            import torch
            torch.cuda.nvtx.range_push(nvtx)
        try:
            while True:
                bi = take()
                if bi is None:
                    return
                idx = batches[bi]
                try:
                    te = time.perf_counter()
                    _, Ls = ctxs[c].encode([utts[i] for i in idx])
                    td = time.perf_counter()
                    pcms = ctxs[c].decode(Ls)
                except BaseException as e:  # this context leaves service; the batch is retried
                    finished(c, bi, e)
                    return
                tim[c][0] += td - te
                tim[c][1] += time.perf_counter() - td
                results[c].extend(zip(idx, pcms))
                finished(c, bi, None)
        finally:
            if nvtx:
                torch.cuda.nvtx.range_pop()

    threads = [threading.Thread(target=worker, args=(c,)) for c in range(len(ctxs))]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    if fatal:
        raise fatal[0]
    if queue:  # every context left service with batches still queued
        raise RuntimeError(f"{len(queue)} batches not run: no context left in service")
    if timings is not None:
        timings[:] = tim
    return [x for r in results for x in r]


def main(argv=None) -> int:
    a = _args(argv)
    import torch
    import torch.distributed as dist

    from . import configs, convert_v2, koko, shard
    from .context import FP16, FP32, Context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        # host-side process group: barriers and the PCM gather move bytes on the host
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))

    utts = configs.config4(seed=a.seed, count=a.count)
    items = shard.units(utts)
    assignment = shard.plan(items, world)
    mine = assignment[rank]

    blob = koko.random_v1_blob(0)
    prec = FP32 if a.fp32 else FP16
    if prec == FP16:
        blob = convert_v2.convert_blob(blob)
    ctxs = [Context(local, prec) for _ in range(max(1, a.contexts))]
    for ctx in ctxs:
        ctx.load_weights(blob)

    # warm-up outside the timed pass: one utterance of every decode-length bucket
    # of this rank's share on every context (the predictor and decode graphs are
    # cached per bucket), largest first so that the decode workspace is sized once
    first = {}
    for i in mine:
        first.setdefault(items[i].L_b, i)
    warm = [first[k] for k in sorted(first, reverse=True)]
    for ctx in ctxs:
        for k in range(0, len(warm), a.batch):
            _, Ls = ctx.encode([utts[i] for i in warm[k:k + a.batch]])
            ctx.decode(Ls)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # one host thread per context: while one context runs the latency-bound front
    # half (encode) of a batch, another's decoders fill the SMs
    timings = []
    t0 = time.perf_counter()
    local_pcm = run_share(ctxs, utts, mine, a.batch, timings)
    t_enc = sum(t[0] for t in timings)
    t_dec = sum(t[1] for t in timings)
    t_rank = time.perf_counter() - t0
    out = shard.gather_pcm(local_pcm, len(utts))
    t_all = time.perf_counter() - t0
    t_max = t_rank
    if world > 1:
        tt = torch.tensor([t_rank], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max = float(tt.item())

    if rank == 0:
        samples = sum(p.shape[0] for p in out)
        expected = sum(600 * int(np.asarray(u.durations).sum()) for u in utts)
        audio_s = samples / 24000.0
        line = {
            "metric": "box throughput, audio-sec/sec", "value": round(audio_s / t_all, 2), "unit": "audio-s/s",
            "n_gpus": world, "utterances": len(utts), "audio_s": round(audio_s, 1),
            "samples_match_durations": samples == expected,
            "wall_s": round(t_all, 3), "max_rank_s": round(t_max, 3),
            "plan_imbalance": round(shard.imbalance(items, assignment), 4),
            "rank0": {"utterances": len(mine), "contexts": len(ctxs), "encode_s_summed": round(t_enc, 3),
                      "decode_s_summed": round(t_dec, 3)},
            "precision": "FP32 semantics (split bf16)" if a.fp32 else "FP16 weights (KOKO v2), FP32 accumulate",
            "config": "config4: T ~ truncated N(120, 60) in [16, 510] + BOS/EOS, durations U[2,8], seeded styles",
            "batch": a.batch, "data": "synthetic; random-init weights",
        }
        print(json.dumps(line), flush=True)
    for ctx in ctxs:
        ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
