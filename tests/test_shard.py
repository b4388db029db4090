"""Host-side sharding of independent utterances (no GPU): the length-bucketed
LPT plan and the PCM gather, the latter over a world-size-2 gloo group."""
import os
import socket

import numpy as np
import pytest

from rokoko_b200 import configs, shard


def test_plan_covers_every_utterance_once_and_balances():
    items = shard.units(configs.config4(seed=0, count=1024))
    for world in (1, 2, 4, 8):
        a = shard.plan(items, world)
        flat = sorted(i for r in a for i in r)
        assert flat == list(range(len(items)))
        assert shard.imbalance(items, a) <= 1.02, (world, shard.imbalance(items, a))
        assert shard.plan(items, world) == a  # deterministic: every rank computes the same plan


def test_plan_groups_buckets_and_orders_by_bucket():
    items = shard.units(configs.config2(seed=1))
    a = shard.plan(items, 3)
    for idx in a:
        keys = [(items[i].T, items[i].L_b) for i in idx]
        assert keys == sorted(keys)


def test_plan_edge_cases():
    assert shard.plan([], 4) == [[], [], [], []]
    one = [shard.Unit(0, 66, 330)]
    assert shard.plan(one, 8)[0] == [0] and sum(map(len, shard.plan(one, 8))) == 1
    with pytest.raises(ValueError):
        shard.plan(one, 0)


def test_run_threads_returns_original_order():
    items = shard.units(configs.config2(seed=4))
    synths = [lambda i, r=r: np.full(600 * items[i].L, i, np.float32) for r in range(3)]
    out = shard.run_threads(synths, items)
    for i, pcm in enumerate(out):
        assert pcm.shape == (600 * items[i].L,) and pcm[0] == i


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_worker(rank, world, port, q, other_host=False, n_utts=None):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if other_host and rank == 1:
        # this rank's node-local directory is not rank 0's (as on another host, even
        # under the same host name): it cannot read the token, so the gather must
        # take the pickled path
        import tempfile
        os.environ["RK_GATHER_DIR"] = tempfile.mkdtemp()
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    used_file = []
    orig = shard._gather_shared_file

    def spy(*a, **k):
        r = orig(*a, **k)
        used_file.append(r[0])
        return r

    shard._gather_shared_file = spy
    try:
        utts = configs.config2(seed=7)[:n_utts]
        items = shard.units(utts)
        mine = shard.plan(items, world)[rank]
        local = shard.run_rank(lambda i: np.full(600 * items[i].L, i, np.float32), mine)
        out = shard.gather_pcm(local, len(items))
        if rank == 0:
            q.put(([(p.shape[0], float(p[0])) for p in out], used_file[0]))
        else:
            q.put((out, used_file[0]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("other_host,n_utts", [(False, None), (True, None), (False, 1)],
                         ids=["shared-file", "separate-dirs-pickled", "one-utterance-idle-rank"])
def test_gather_pcm_over_gloo_world2(other_host, n_utts):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q, other_host, n_utts)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = [r for r, _ in res if r is not None]
    assert len(got) == 1
    # the shared file is used exactly when both ranks can read rank 0's token
    assert [f for _, f in res] == [not other_host] * 2
    items = shard.units(configs.config2(seed=7)[:n_utts])
    assert got[0] == [(600 * u.L, float(u.index)) for u in items]
