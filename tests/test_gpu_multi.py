"""The multi-GPU paths on one GPU: the token-range sharded cold search (per-range top-k,
merge) against the whole-index search and the oracle, the sharded retrieval against the
single-device one, and a ragged batch (own prompt lengths, budgets and cold capacities per
sequence) against the oracle run sequence by sequence."""

import numpy as np
import pytest
import torch

from golden_cases import assert_close, oracle_kwargs
from oracle_follow import assert_same_run, run_following

pytestmark = pytest.mark.gpu

from oracle import hotcold_oracle as O  # noqa: E402


def _oracle_topk(X, q, k):
    """Exact top k by float64 inner product, ties to the lower row; the gap at the cut."""
    sc = X.astype(np.float64) @ q.astype(np.float64)
    order = np.lexsort((np.arange(len(sc)), -sc))
    return order[:k], O.boundary_gap(sc, k)


@pytest.mark.parametrize("n,F,k", [(5000, 128, 64), (70000, 128, 256), (3001, 200, 17), (40, 64, 64), (0, 128, 8)])
def test_cold_topk_vs_oracle_and_shards(n, F, k):
    from hotcold_kv_cache_b200.shard import local_topk, merge_candidates, token_range
    g = torch.Generator().manual_seed(n + F + k)
    X = torch.randn((n, F), generator=g)
    q = torch.randn(F, generator=g)
    if n > 100:
        X[n - 7] = X[3]  # an exact tie across ranges: the lower id goes first
        X[3] = q * 3.0
        X[n - 7] = q * 3.0
    dev = torch.device("cuda", 0)
    Xd, qd = X.to(dev), q.to(dev)
    sc, ids = local_topk(Xd, 0, qd, k)
    ids = ids.cpu().numpy()
    m = min(n, k)
    assert (ids[m:] == -1).all()
    if n:
        want, gap = _oracle_topk(X.numpy(), q.numpy(), m)
        if not np.array_equal(ids[:m], want):
            assert gap <= 1e-5, f"top-k differs with gap {gap}"
        if n > 100:
            assert list(ids[:2]) == [3, n - 7]
    for world in (2, 3, 8):
        cs, ci = [], []
        for r in range(world):
            lo, hi = token_range(n, r, world)
            s_r, i_r = local_topk(Xd[lo:hi], lo, qd, k)
            cs.append(s_r)
            ci.append(i_r)
        ms, mi = merge_candidates(torch.cat(cs), torch.cat(ci), world, k)
        assert np.array_equal(mi.cpu().numpy(), ids), f"{world} ranges"
        assert torch.equal(ms[:m].cpu(), sc[:m].cpu())


class _EmulatedRanks:
    """The ranks of a sharded search emulated in one process: search() runs every rank's
    search of its token range (the age runs of the arena's cold ring that rank r would get)
    and merges them as the all-gather would."""

    def __init__(self, world, arena_of):
        self.rank, self.world, self.ws, self.arena_of = 0, world, None, arena_of

    def check_k(self, k):
        from hotcold_kv_cache_b200.shard import ShardedColdSearch
        ShardedColdSearch(rank=0, world=self.world).check_k(k)

    def search(self, runs, n, qvecs, k):
        from hotcold_kv_cache_b200.shard import ShardedColdSearch, age_runs, merge_candidates, token_range
        a = self.arena_of()
        heads = a.cold_head()
        out = torch.empty((len(n), k), dtype=torch.int32, device=qvecs.device)
        for b in range(len(n)):
            cs = torch.empty((self.world, k), dtype=torch.float32, device=qvecs.device)
            ci = torch.empty((self.world, k), dtype=torch.int32, device=qvecs.device)
            for r in range(self.world):
                lo, hi = token_range(int(n[b]), r, self.world)
                rr = [(a.cold_vec[b, s0:s0 + c], age0) for s0, c, age0 in age_runs(int(heads[b]), a.ccaps[b], lo, hi)]
                one = ShardedColdSearch(rank=r, world=self.world)
                one._local_runs(rr, qvecs[b], k, (cs[r], ci[r]))
            merge_candidates(cs.view(-1), ci.view(-1), self.world, k, out_id=out[b])
        return out


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_sharded_retrieval_matches_single_device(dtype):
    """Prompt-end retrieval of a batch of 2 through the sharded search (4 emulated ranks)
    splices exactly the held segment of the single-device retrieval."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(B=2, Hq=8, Hk=2, D=128, T=900, steps=1, dtype=dtype, policy="snapkv", cap=128, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=2000, faiss_dim=128, window_size=1 << 20, pool=4, R=32,
             hold=True, rap=True, theta=500000.0, seed=321)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], 1, dtype)
    res = run_cuda_layer(c, inp, 1)
    a = res["ctrl"].arenas[0]
    dev = a.device
    q_tail = torch.from_numpy(np.ascontiguousarray(inp["q_pre"][:, :, -4:, :]).astype(np.float32)).to(dev, a.dtype)
    a.retrieve(q_dense=q_tail)
    ref = [t.clone() for t in (a.held_k, a.held_v, a.held_pos, a.held_valid, a.held_src)]
    a.held_k.zero_()
    a.held_src.fill_(-1)
    em = _EmulatedRanks(4, lambda: a)
    a.retrieve_sharded(em, q_dense=q_tail)
    got = (a.held_k, a.held_v, a.held_pos, a.held_valid, a.held_src)
    for r, g2, name in zip(ref, got, ("held_k", "held_v", "held_pos", "held_valid", "held_src")):
        assert torch.equal(r, g2), name
    assert int(a.held_valid.sum()) == 2 * 32
    assert res["ctrl"].device_status() == 0


@pytest.mark.parametrize("dtype,policy", [("float16", "snapkv"), ("float32", "hotcold"), ("bfloat16", "snapkv")])
def test_ragged_batch_vs_oracle(dtype, policy):
    """Three sequences of different prompt lengths, budgets and cold capacities in one batch:
    each matches the oracle run of that sequence alone, step by step."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_ragged
    lens, budgets, ccaps = [700, 1301, 260], [128, 256, 64], [1000, 1200, 300]
    steps = 6
    c = dict(Hq=8, Hk=2, D=128, dtype=dtype, policy=policy, cap=max(budgets), recent=16 if policy == "snapkv" else 32,
             topk_ratio=0.0 if policy == "snapkv" else 0.5, pool_kernel=7, ccap=max(ccaps), faiss_dim=128,
             window_size=1 << 20, pool=8, R=16, hold=True, rap=True, theta=500000.0)
    ins = [synth.layer_inputs(900 + b, 1, 8, 2, 128, lens[b], steps, dtype) for b in range(3)]
    res = run_cuda_ragged(c, ins, budgets, ccaps, steps)
    from cuda_runner import ragged_seq
    for b in range(3):
        cb = dict(c, B=1, T=lens[b], cap=budgets[b], ccap=ccaps[b])
        rb = ragged_seq(res, b)
        layer, o_outs, o_hot, _ = run_following(O, ins[b], steps, rb, **oracle_kwargs(cb))
        assert assert_same_run(rb, layer, o_outs, o_hot, dtype, steps, f"seq {b}") == steps
    assert res["ctrl"].device_status() == 0


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_sharded_retrieval_on_wrapped_ring(dtype):
    """A decode that keeps evicting into a cold ring past its capacity (the ring wraps), with
    a search every 3 steps through the sharded path (3 emulated ranks, so some ranks' token
    ranges cross the end of the ring): held segments, hot sets and outputs equal those of the
    same run with the single-device search (both on the split ops, which a sharded search
    uses)."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(B=2, Hq=8, Hk=2, D=128, T=300, steps=40, dtype=dtype, policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=250, faiss_dim=128, window_size=3, pool=4, R=16,
             hold=True, rap=True, theta=500000.0, seed=4711)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], c["steps"], dtype)
    single = run_cuda_layer(c, inp, c["steps"], fused=False)
    sharded = run_cuda_layer(c, inp, c["steps"], fused=False,
                             searcher=lambda ctrl: _EmulatedRanks(3, lambda: ctrl.arenas[0]))
    a = sharded["ctrl"].arenas[0]
    assert (a.cold_pushed > a.ccaps[0]).all(), "the ring did not wrap"
    assert sorted(single["held"]) == sorted(sharded["held"])
    for st in single["held"]:
        for x, y in zip(single["held"][st], sharded["held"][st]):
            assert np.array_equal(x, y), st
    for i in range(c["steps"]):
        assert np.array_equal(single["hot"][i], sharded["hot"][i]), i
        assert np.array_equal(single["outs"][i], sharded["outs"][i]), i
    assert np.array_equal(a.cold_head(), a.device_state()[:, 2])
    assert sharded["ctrl"].device_status() == 0


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_async_sharded_retrieval_vs_oracle(dtype):
    """async_retrieval with the sharded search (3 emulated ranks) on a ring that wraps, a search
    every 3 steps on a side stream attended from the next step: the same held segments, hot
    sets and outputs as the async run with the single-device search, and that run step by step
    against the oracle with the one-step lag."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(B=2, Hq=8, Hk=2, D=128, T=300, steps=40, dtype=dtype, policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=250, faiss_dim=128, window_size=3, pool=4, R=16,
             hold=True, rap=True, theta=500000.0, seed=4712, **{"async": True})
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], c["steps"], dtype)
    single = run_cuda_layer(c, inp, c["steps"], fused=False)
    sharded = run_cuda_layer(c, inp, c["steps"], fused=False,
                             searcher=lambda ctrl: _EmulatedRanks(3, lambda: ctrl.arenas[0]))
    a = sharded["ctrl"].arenas[0]
    assert (a.cold_pushed > a.ccaps[0]).all(), "the ring did not wrap"
    assert sorted(single["held"]) == sorted(sharded["held"])
    for st in single["held"]:
        for x, y in zip(single["held"][st], sharded["held"][st]):
            assert np.array_equal(x, y), st
    for i in range(c["steps"]):
        assert np.array_equal(single["hot"][i], sharded["hot"][i]), i
        assert np.array_equal(single["outs"][i], sharded["outs"][i]), i
    layer, o_outs, o_hot, _ = run_following(O, inp, c["steps"], single, **oracle_kwargs(c))
    assert assert_same_run(single, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
    assert [e["step"] for e in layer.events][:3] == [1, 3, 6]
    assert sharded["ctrl"].device_status() == 0 and single["ctrl"].device_status() == 0
