"""The HBM cold store with the known-answer checks of the reference's
tests/test_cold_store.py: searching with a token's own key returns that token
with its exact pre-RoPE key and value; the ring and its index stay aligned when
the ring wraps; a batch larger than the ring keeps its newest tokens."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from hotcold_kv_cache_b200 import EvictedKV  # noqa: E402

HK, D = 2, 16 * 8  # head_dim must be 64 or 128 on the CUDA path


def _controller(cap, lookahead=4):
    from hotcold_kv_cache_b200 import KVController
    ctrl = KVController(cpu_buffer_size=cap, faiss_dim=D, lookahead_k=lookahead, enable_asserts=True,
                        profile_overlap=False)
    ctrl.set_rotary(torch.ones(D // 2), 1.0)
    ctrl._lazy_init(torch.zeros(1, HK, 1, D, device="cuda"), n_layers=1)
    ctrl.arena(0, HK, torch.float32, torch.device("cuda"))
    return ctrl


def _tokens(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, HK, D, generator=g)


def _evict(ctrl, keys, positions):
    te = keys.shape[0]
    ctrl.add_evicted_to_cold_store(0, EvictedKV(
        k_pre_cpu=keys.permute(1, 0, 2).unsqueeze(0).contiguous(),
        v_cpu=(-keys).permute(1, 0, 2).unsqueeze(0).contiguous(),
        pos_cpu=torch.tensor(positions, dtype=torch.long).unsqueeze(0),
        evicted_idx=torch.arange(te, dtype=torch.long).unsqueeze(0),
    ))


def _top1(ctrl, key):
    q = ctrl._k_token_to_vec_np(key)[None, :]
    ctrl._retrieval_worker(0, q)
    kpre, v, pos, valid = ctrl._retrieval_ready_cpu[0]
    assert bool(valid[0, 0]), "top hit is not valid"
    return (int(pos[0, 0]), kpre[0, :, 0, :].cpu(), v[0, :, 0, :].cpu(),
            pos[0][valid[0]].cpu().tolist())


def test_no_wrap_returns_queried_token():
    ctrl = _controller(cap=64)
    keys = _tokens(20)
    _evict(ctrl, keys, list(range(100, 120)))
    for t in (0, 7, 19):
        pos, kpre, v, _ = _top1(ctrl, keys[t])
        assert pos == 100 + t, (t, pos)
        assert torch.equal(kpre, keys[t]) and torch.equal(v, -keys[t])


def test_wrap_keeps_ids_aligned():
    cap = 8
    ctrl = _controller(cap)
    keys = _tokens(15, seed=1)
    for lo in (0, 5, 10):
        _evict(ctrl, keys[lo:lo + 5], list(range(lo, lo + 5)))
    ring = ctrl.cpu_kpre_ring[0][0]
    assert len(ring) == cap and ctrl.index[0][0].ntotal == cap
    live = range(15 - cap, 15)
    for t in live:
        pos, kpre, v, _ = _top1(ctrl, keys[t])
        assert pos == t, (t, pos)
        assert torch.equal(kpre, keys[t]) and torch.equal(v, -keys[t])
    for t in range(15 - cap):
        _, _, _, hits = _top1(ctrl, keys[t])
        assert all(h in live for h in hits), (t, hits)


def test_batch_larger_than_ring():
    cap = 8
    ctrl = _controller(cap)
    keys = _tokens(20, seed=2)
    _evict(ctrl, keys, list(range(20)))
    assert len(ctrl.cpu_kpre_ring[0][0]) == cap and ctrl.index[0][0].ntotal == cap
    for t in range(20 - cap, 20):
        pos, kpre, _, _ = _top1(ctrl, keys[t])
        assert pos == t and torch.equal(kpre, keys[t]), (t, pos)


def test_padding_entries_are_skipped_and_order_is_by_score():
    ctrl = _controller(cap=32, lookahead=6)
    keys = _tokens(10, seed=3)
    kp = keys.permute(1, 0, 2).unsqueeze(0).contiguous()
    idx = torch.arange(10).unsqueeze(0)
    idx[0, 3] = -1
    ctrl.add_evicted_to_cold_store(0, EvictedKV(kp, -kp, torch.arange(10).unsqueeze(0), idx))
    assert ctrl.cold_size(0) == 9
    q = ctrl._k_token_to_vec_np(keys[5])[None, :]
    ctrl._retrieval_worker(0, q)
    kpre, v, pos, valid = ctrl._retrieval_ready_cpu[0]
    got = pos[0][valid[0]].cpu().tolist()
    assert 3 not in got and got[0] == 5 and len(got) == 6
    vecs = np.stack([ctrl._k_token_to_vec_np(keys[i]) for i in range(10)])
    sc = vecs @ q[0]
    sc[3] = -np.inf
    assert got == list(np.argsort(-sc, kind="stable")[:6])


@pytest.mark.parametrize("dtype,fused", [("float16", True), ("float16", False), ("float32", False)])
def test_cold_payload_in_host_memory(dtype, fused):
    """The cold ring's payload in page-locked host memory (cold_payload="host", the reference's
    CPU cold tier for stores larger than HBM): kernels write evicted tokens there and gather
    retrieved hits from it. Same outputs, hot sets, held segments and cold ring as the payload
    in HBM, bit for bit, through a wrapping ring and a search every 3 steps; and the oracle."""
    import numpy as np
    import torch
    from golden_cases import oracle_kwargs
    from hotcold_kv_cache_b200 import synth
    from oracle import hotcold_oracle as O
    from oracle_follow import assert_same_run, run_following
    import cuda_runner
    c = dict(B=2, Hq=8, Hk=2, D=128, T=400, steps=24, dtype=dtype, policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=350, faiss_dim=128, window_size=3, pool=2, R=16, hold=True,
             rap=True, theta=500000.0, seed=606)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], c["steps"], dtype)
    dev_run = cuda_runner.run_cuda_layer(c, inp, c["steps"], fused=fused)
    kw = cuda_runner.controller_kwargs
    try:
        cuda_runner.controller_kwargs = lambda case: dict(kw(case), cold_payload="host")
        host_run = cuda_runner.run_cuda_layer(c, inp, c["steps"], fused=fused)
    finally:
        cuda_runner.controller_kwargs = kw
    a_h, a_d = host_run["ctrl"].arenas[0], dev_run["ctrl"].arenas[0]
    assert not a_h.cold_kpre.is_cuda and a_h.cold_kpre.is_pinned() and a_d.cold_kpre.is_cuda
    assert (a_h.cold_pushed > a_h.ccaps[0]).all(), "the ring did not wrap"
    assert np.array_equal(host_run["outs"], dev_run["outs"])
    for i in range(c["steps"]):
        assert np.array_equal(host_run["hot"][i], dev_run["hot"][i])
    assert sorted(host_run["held"]) == sorted(dev_run["held"])
    for st in host_run["held"]:
        for x, y in zip(host_run["held"][st], dev_run["held"][st]):
            assert np.array_equal(x, y)
    assert torch.equal(a_h.cold_kpre.cuda(), a_d.cold_kpre) and torch.equal(a_h.cold_v.cuda(), a_d.cold_v)
    assert torch.equal(a_h.cold_pos, a_d.cold_pos) and torch.equal(a_h.cold_vec, a_d.cold_vec)
    layer, o_outs, o_hot, _ = run_following(O, inp, c["steps"], host_run, **oracle_kwargs(c))
    assert assert_same_run(host_run, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
    assert host_run["ctrl"].device_status() == 0
