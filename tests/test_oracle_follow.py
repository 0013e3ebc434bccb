"""The near-tie resynchronisation of tests/oracle_follow.py, checked on the CPU with the
oracle standing in for the CUDA run: following its own run adopts nothing and compares every
step; a kept set or a hit list that differs far from the selection boundary fails; one that
differs only at a near-tie is adopted."""

import numpy as np
import pytest

from golden_cases import oracle_kwargs
from oracle import hotcold_oracle as O
from oracle_follow import FollowCuda, assert_same_run, run_following


def _case():
    return dict(B=2, Hq=8, Hk=2, D=64, T=200, steps=10, dtype="float32", policy="snapkv", cap=48, recent=8,
                topk_ratio=0.0, pool_kernel=7, ccap=300, faiss_dim=64, window_size=4, pool=2, R=8, hold=True,
                rap=True, theta=500000.0, seed=5)


def _as_cuda(layer, outs, hot, B, T):
    """An oracle run in the layout of cuda_runner.run_cuda_layer."""
    c0 = [e for e in layer.compress_log if e["step"] == 0]
    hot0 = np.stack([c0[b]["keep_pos"] for b in range(B)], 0) if c0 else np.tile(np.arange(T), (B, 1))
    held = {e["step"]: (e["pos"], e["valid"], e["kmem"]) for e in layer.events}
    launched = {e["launched"] for e in layer.events if e["launched"] > 0}
    return dict(outs=outs, hot=hot, hot0=[hot0], held=held, launched=launched)


def test_following_its_own_run_adopts_nothing():
    from hotcold_kv_cache_b200 import synth
    c = _case()
    inp = synth.layer_inputs(c["seed"], c["B"], c["Hq"], c["Hk"], c["D"], c["T"], c["steps"], c["dtype"])
    layer, outs, hot = O.run_layer(inp, c["steps"], **oracle_kwargs(c))
    res = _as_cuda(layer, outs, hot, c["B"], c["T"])
    l2, o2, h2, fc = run_following(O, inp, c["steps"], res, **oracle_kwargs(c))
    assert fc.adopted == []
    assert assert_same_run(res, l2, o2, h2, c["dtype"], c["steps"]) == c["steps"]
    assert len(layer.events) >= 3 and len(layer.compress_log) == 2 * (1 + c["steps"])


def _keep_case(cuda_keeps):
    """Ten prefix tokens at positions 100..109 with distinct scores; the 5th and 6th best
    (tokens 4 and 5) are a near-tie (1e-6 apart). The oracle keeps the best five."""
    sc = np.array([9.0, 8.0, 7.0, 6.0, 5.0, 5.0 * (1 - 1e-6), 3.0, 2.0, 1.0, 0.5])
    P = np.arange(100, 110)
    top = np.arange(5)
    res = dict(hot=[np.array([np.sort(P[cuda_keeps])])], hot0=[], held={})
    return FollowCuda(res), sc, P, top


def test_keep_near_tie_is_adopted():
    fc, sc, P, top = _keep_case([0, 1, 2, 3, 5])
    got = fc.keep(1, 0, sc, 10, 5, top, P)
    assert list(got) == [0, 1, 2, 3, 5]
    assert fc.adopted[0][0] == "keep" and fc.adopted[0][3] <= 1e-5


def test_keep_far_difference_fails():
    fc, sc, P, top = _keep_case([1, 2, 3, 4, 6])
    with pytest.raises(AssertionError, match="kept set differs"):
        fc.keep(1, 0, sc, 10, 5, top, P)
    fc, sc, P, top = _keep_case([0, 1, 2, 3])
    with pytest.raises(AssertionError, match="CUDA kept 4"):
        fc.keep(1, 0, sc, 10, 5, top, P)


def test_hits_near_tie_adopted_and_far_difference_fails():
    sc = np.array([0.9, 0.5, 0.7, 0.7 * (1 - 5e-5), 0.1])
    ring_pos = np.array([10, 11, 12, 13, 14])
    ids = np.array([0, 2, 3])  # the oracle's best three
    for cuda_ids, ok in (([0, 3, 2], True), ([0, 2, 1], False), ([0, 2, 3], True)):
        pos = np.zeros((1, 4), np.int64)
        valid = np.zeros((1, 4), bool)
        pos[0, :3] = ring_pos[cuda_ids]
        valid[0, :3] = True
        fc = FollowCuda(dict(hot=[], hot0=[], held={1: (pos, valid, None)}))
        if ok:
            assert list(fc.hits(0, 0, sc, ids, ring_pos)) == cuda_ids
        else:
            with pytest.raises(AssertionError, match="hit 2 differs"):
                fc.hits(0, 0, sc, ids, ring_pos)
