"""Multi-rank host logic on CPU with gloo process groups (world size 2 and 3): the exchange
of the token-range sharded cold search and the ragged-batch partition agreed by all ranks.
The per-range search and the merge are the oracle's exact inner-product top-k here (the
CUDA kernels behind them are checked on the GPU); what runs under test is the range split,
the all-gather layout and the id bookkeeping of shard.ShardedColdSearch."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exact_topk(X, q, k):
    sc = X.astype(np.float64) @ q.astype(np.float64)
    order = np.lexsort((np.arange(len(sc)), -sc))[:k]
    return order, sc[order]


def _host_local(rows, lo, q, k):
    """Stand-in of hc_cold_topk: the k best rows as (score, lo + row), -1 / -inf padded."""
    X = rows.numpy()
    ids, sc = _exact_topk(X, q.numpy(), k) if len(X) else (np.zeros(0, np.int64), np.zeros(0))
    out_s = np.full(k, -np.inf, np.float32)
    out_i = np.full(k, -1, np.int32)
    out_s[: len(ids)] = sc
    out_i[: len(ids)] = ids + lo
    return torch.from_numpy(out_s), torch.from_numpy(out_i)


def _host_merge(cs, ci, n_shards, k):
    """Stand-in of hc_shard_merge: best k live candidates, ties to the lower id."""
    s, i = cs.numpy().astype(np.float64), ci.numpy()
    live = i >= 0
    s, i = s[live], i[live]
    order = np.lexsort((i, -s))[:k]
    out = np.full(k, -1, np.int32)
    out[: len(order)] = i[order]
    return torch.from_numpy(s[order].astype(np.float32)), torch.from_numpy(out)


def _problem():
    rng = np.random.default_rng(11)
    ns = [1000, 37, 2, 0]
    F, k = 64, 16
    q = rng.standard_normal((len(ns), F)).astype(np.float32)
    index = [rng.standard_normal((n, F)).astype(np.float32) for n in ns]
    index[0][10] = q[0] * 4.0  # equal best rows in different ranges: the lower id first
    index[0][990] = q[0] * 4.0
    return ns, F, k, q, index


def _sharded_worker(rank, world, port, out_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from hotcold_kv_cache_b200.shard import ShardedColdSearch, age_runs, token_range
        from hotcold_kv_cache_b200 import synth
        ns, F, k, q, index = _problem()
        s = ShardedColdSearch(local=_host_local, merge=_host_merge)
        assert (s.rank, s.world) == (rank, world)
        runs = [[(torch.from_numpy(index[b][lo:hi]), lo)] if hi > lo else []
                for b in range(len(ns)) for lo, hi in [token_range(ns[b], rank, world)]]
        ids = s.search(runs, ns, torch.from_numpy(q), k).numpy()
        # the same index in a wrapped ring: age a sits at slot (head + a) % n, so a rank's ages can
        # cross the end of the ring and come as two runs of slots
        wids = []
        for b, n in enumerate(ns):
            head = (7 * n) // 10
            ring = np.roll(index[b], head, axis=0) if n else index[b]
            lo, hi = token_range(n, rank, world)
            rr = [(torch.from_numpy(ring[s0:s0 + c]), a0) for s0, c, a0 in age_runs(head, max(n, 1), lo, hi)]
            wids.append(s.search([rr], [n], torch.from_numpy(q[b:b + 1]), k).numpy()[0])
        # the ragged partition: every rank derives the same one and the parts cover the batch
        items = synth.ragged_batch(3, 64)
        parts = synth.balanced_partition(items, world)
        mine = parts[rank]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        out_q.put((rank, ids, gathered, parts, np.stack(wids, 0)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_search_and_partition_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, ids, gathered, parts, wids = q.get(timeout=120)
            res[r] = (ids, gathered, parts, wids)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    ns, F, k, qv, index = _problem()
    for b, n in enumerate(ns):
        want = np.full(k, -1, np.int64)
        if n:
            o, _ = _exact_topk(index[b], qv[b], k)
            want[: len(o)] = o
        for r in range(world):
            assert np.array_equal(res[r][0][b], want), (r, b)
            assert np.array_equal(res[r][3][b], want), ("wrapped ring", r, b)
    assert list(res[0][0][0][:2]) == [10, 990]
    for r in range(world):
        ids, gathered, parts, _ = res[r]
        assert gathered == parts
        assert sorted(i for p in parts for i in p) == list(range(64))
