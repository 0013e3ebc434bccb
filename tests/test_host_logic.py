"""Host-side logic on CPU: the compression plan the host mirrors agrees with the
oracle's (hence with cache.py:44-53 and scoring.py:117-120), seeded inputs are
reproducible, and the ragged-batch partition is balanced."""

import numpy as np
import pytest

from hotcold_kv_cache_b200 import synth
from hotcold_kv_cache_b200.arena import plan_keep
from oracle.hotcold_oracle import Policy, plan_keep as oracle_plan


@pytest.mark.parametrize("policy", ["hotcold", "snapkv"])
def test_plan_matches_oracle(policy):
    for budget in (1, 2, 31, 32, 64, 128, 512, 1000, 2048):
        for recent in (0, 1, 16, 32, 128):
            for ratio in (0.0, 0.15, 0.5, 0.99):
                for S in (0, 1, 5, budget, budget + 1, budget + 7, 4096, 131072):
                    p = oracle_plan(Policy(policy=policy, cap=budget, recent=recent, topk_ratio=ratio), S)
                    q = plan_keep(policy, budget, recent, ratio, S)
                    assert (p is None and q is None) or (p[:2] == q), (policy, budget, recent, ratio, S, p, q)


def test_benchmark_topk_ratio():
    # run_baselines.py:86-87: budget 512, recent 128 -> 0.5 -> keep 256 + 128
    ratio = max(0.05, 0.75 - 128 / 512)
    assert plan_keep("hotcold", 512, 128, ratio, 8192) == (8064, 256)
    assert plan_keep("snapkv", 512, 32, 0.0, 8192) == (8160, 480)
    assert plan_keep("snapkv", 512, 32, 0.0, 513) == (481, 480)


def test_inputs_are_reproducible():
    a = synth.layer_inputs(3, 1, 4, 2, 64, 10, 2, "float16")
    b = synth.layer_inputs(3, 1, 4, 2, 64, 10, 2, "float16")
    for k in a:
        assert np.array_equal(a[k], b[k])
    assert a["q_pre"].dtype == np.float16


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3.0e38], np.float32)
    r = synth.round_bf16(x)
    bits = r.view(np.uint32)
    assert np.all(bits & 0xFFFF == 0)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0078125)


def test_balanced_partition():
    items = synth.ragged_batch(7, 64)
    assert len(items) == 64 and all(2048 <= L <= 32768 for L, _ in items)
    assert [b for _, b in items[:6]] == [512, 1024, 2048, 512, 1024, 2048]
    for n in (1, 2, 4, 8):
        parts = synth.balanced_partition(items, n)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(items[i][0] + items[i][1] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(L + b for L, b in items)


def test_oracle_chunked_prefill_one_chunk_is_prefill():
    """The oracle's chunked prefill with one chunk equals its plain prefill."""
    from oracle import hotcold_oracle as O
    from golden_cases import oracle_kwargs
    c = dict(B=1, Hq=4, Hk=2, D=64, T=200, dtype="float32", policy="snapkv", cap=48, recent=8, topk_ratio=0.0,
             pool_kernel=7, ccap=400, faiss_dim=64, window_size=1 << 20, pool=4, R=8, hold=True, rap=True,
             theta=500000.0)
    inp = synth.layer_inputs(3, 1, 4, 2, 64, 200, 3, "float32")
    a, oa, ha = O.run_layer(inp, 3, **oracle_kwargs(c))
    b, ob, hb = O.run_layer(inp, 3, chunks=[0, 200], **oracle_kwargs(c))
    assert np.array_equal(oa, ob) and all(np.array_equal(x, y) for x, y in zip(ha, hb))
    assert a.dbg == b.dbg
    d, od, hd = O.run_layer(inp, 3, chunks=[0, 50, 120, 200], **oracle_kwargs(c))
    assert d.P.shape[1] == a.P.shape[1]  # the same budget is kept either way


def test_token_ranges_partition_the_index():
    """The ranks' token ranges of a cold index of n entries are contiguous, disjoint and cover
    [0, n) in rank order, for every world size the benchmark runs."""
    from hotcold_kv_cache_b200.shard import token_range
    for n in (0, 1, 7, 256, 129033):
        for world in range(1, 9):
            spans = [token_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(lo <= hi for lo, hi in spans)


def test_age_runs_map_ages_to_ring_slots():
    """A range of ages on a ring (age 0 at slot `head`) split into runs of contiguous slots:
    every age lands on slot (head + age) % ccap, in age order, in one run or two (the second
    from slot 0 when the range crosses the ring's end)."""
    from hotcold_kv_cache_b200.shard import age_runs
    rng = np.random.default_rng(3)
    for _ in range(500):
        ccap = int(rng.integers(1, 64))
        head = int(rng.integers(0, ccap))
        lo = int(rng.integers(0, ccap + 1))
        hi = int(rng.integers(lo, ccap + 1))
        runs = age_runs(head, ccap, lo, hi)
        ages = [a0 + i for _, c, a0 in runs for i in range(c)]
        slots = [s0 + i for s0, c, _ in runs for i in range(c)]
        assert ages == list(range(lo, hi))
        assert slots == [(head + a) % ccap for a in ages]
        assert len(runs) <= 2 and all(c > 0 for _, c, _ in runs)
        if len(runs) == 2:
            assert runs[1][0] == 0


def test_sharded_search_refuses_lookahead_beyond_kernel_limits():
    """hc_cold_topk keeps at most 256 per rank and hc_shard_merge at most 4096 candidates: the
    sharded search refuses such a lookahead when it is attached, not at the first search."""
    from hotcold_kv_cache_b200.shard import ShardedColdSearch
    ShardedColdSearch(rank=0, world=8).check_k(256)
    ShardedColdSearch(rank=0, world=16).check_k(256)
    for world, k in ((1, 0), (1, 257), (17, 256), (32, 200)):
        with pytest.raises(ValueError):
            ShardedColdSearch(rank=0, world=world).check_k(k)
    from hotcold_kv_cache_b200 import KVController
    ctrl = KVController(lookahead_k=300)
    with pytest.raises(ValueError):
        ctrl.cold_search = ShardedColdSearch(rank=0, world=1)
    ctrl = KVController(lookahead_k=256)
    ctrl.cold_search = ShardedColdSearch(rank=0, world=16)
    assert ctrl.cold_search is not None


def test_oracle_retrieval_lag_attends_one_step_later():
    """The oracle's schedule for async_retrieval (retrieval_lag=1): every decode-step search is
    attended one step later than in the deterministic schedule (a search at the last step is
    never attended), the same number of searches runs, and the steps before the first attended
    search are identical in both."""
    from golden_cases import oracle_kwargs
    from oracle import hotcold_oracle as O
    n = 30
    c = dict(B=2, Hq=8, Hk=2, D=64, T=300, steps=n, dtype="float32", policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=1024, faiss_dim=64, window_size=8, pool=4, R=16, hold=True,
             rap=False, theta=500000.0, seed=11)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 64, 300, n, "float32")
    l0, o0, _ = O.run_layer(inp, n, **oracle_kwargs(c))
    l1, o1, _ = O.run_layer(inp, n, **oracle_kwargs(dict(c, **{"async": True})))
    s0 = [e["step"] for e in l0.events]
    s1 = [e["step"] for e in l1.events]
    assert len(s0) >= 3
    assert s1 == [s + 1 for s in s0 if s + 1 <= n]
    assert l0.dbg["retrieval_launched"] == l1.dbg["retrieval_launched"]
    np.testing.assert_array_equal(o0[:s0[0] - 1], o1[:s0[0] - 1])
    assert not np.array_equal(o0[s0[0] - 1], o1[s0[0] - 1])
