"""CUDA hot path of one layer against the CPU oracle and against the golden
vectors of the reference itself: attention outputs, hot sets after every step,
cold ring contents, retrieved sets, re-rotated held keys and debug counters."""

import math

import numpy as np
import pytest
import torch

from golden_cases import LAYER_CASES, assert_close, inputs, load, oracle_kwargs, split_hot

pytestmark = pytest.mark.gpu

from oracle import hotcold_oracle as O  # noqa: E402


def _run(case, model_cos=True):
    from cuda_runner import run_cuda_layer
    return run_cuda_layer(case, inputs(case), case["steps"], model_cos=model_cos)


def _compare_layer(res, case, layer, o_outs, o_hot, near_tie=1e-4):
    """Step-by-step comparison. A hot-set difference is accepted only where the oracle's
    selection boundary has a relative score gap within `near_tie`; the states differ from
    there on, so the comparison stops. Returns the number of steps compared."""
    dt = case["dtype"]
    n = len(o_hot)
    for i in range(n):
        if not np.array_equal(res["hot"][i], o_hot[i]):
            gaps = [e["gap"] for e in layer.compress_log if e["step"] == i + 1]
            assert gaps and min(gaps) <= near_tie, f"hot set differs at step {i + 1} (gap {gaps})"
            return i
        assert_close(res["outs"][i], o_outs[i], dt, f"attention step {i + 1}")
    return n


@pytest.mark.parametrize("name", LAYER_CASES)
@pytest.mark.parametrize("model_cos", [True, False])
def test_layer_vs_oracle_and_golden(name, model_cos):
    g = load(name)
    c = g["case"]
    layer, o_outs, o_hot = O.run_layer(inputs(c), c["steps"], **oracle_kwargs(c))
    res = _run(c, model_cos)
    steps = _compare_layer(res, c, layer, o_outs, o_hot)
    assert steps == c["steps"], "golden cases are chosen free of near-ties"
    # against the reference's own outputs
    assert_close(res["outs"], g["outs"], c["dtype"], "attention vs reference")
    for i, (a, b) in enumerate(zip(res["hot"], split_hot(g))):
        assert np.array_equal(a, b), f"hot set vs reference, step {i + 1}"
    from cuda_runner import cold_positions
    cold = cold_positions(res["ctrl"])
    if g["cold_pos"].size:
        assert np.array_equal(np.stack(cold), g["cold_pos"])
    for b, cp in enumerate(layer.cold_positions()):
        assert np.array_equal(cold[b], cp)
    # retrieved sets: same steps, same positions and validity, held keys re-rotated alike
    assert sorted(res["held"]) == [e["step"] for e in layer.events]
    for e in layer.events:
        pos, valid, k = res["held"][e["step"]]
        assert np.array_equal(valid, e["valid"]), e["step"]
        assert np.array_equal(pos[valid], e["pos"][e["valid"]]), e["step"]
        assert_close(k, e["kmem"], c["dtype"], f"held keys step {e['step']}")
    if "ret_pos" in g:
        for e, p, v in zip(sorted(res["held"]), g["ret_pos"], g["ret_valid"]):
            pos, valid, _ = res["held"][e]
            assert np.array_equal(valid, v) and np.array_equal(pos[valid], p[v])
    # counters
    ctrl = res["ctrl"]
    for k, v in layer.dbg.items():
        assert ctrl.dbg[k] == v, (k, ctrl.dbg[k], v)
    assert ctrl.dbg["triton_decode_calls"] == c["steps"]
    assert ctrl.device_status() == 0


@pytest.mark.parametrize("name", LAYER_CASES)
def test_fused_step_matches_split_ops(name):
    """hc_step (one cluster launch) against hc_append + hc_compress + hc_attend."""
    from cuda_runner import run_cuda_layer
    c = load(name)["case"]
    fused = run_cuda_layer(c, inputs(c), c["steps"], fused=True)
    split = run_cuda_layer(c, inputs(c), c["steps"], fused=False)
    for i in range(c["steps"]):
        assert np.array_equal(fused["hot"][i], split["hot"][i]), f"hot set differs at step {i + 1}"
        assert_close(fused["outs"][i], split["outs"][i], c["dtype"], f"attention step {i + 1}")
    assert sorted(fused["held"]) == sorted(split["held"])
    assert fused["ctrl"].dbg == split["ctrl"].dbg
    a_f, a_s = fused["ctrl"].arenas[0], split["ctrl"].arenas[0]
    assert a_f.launches < a_s.launches, "the fused step did not run"
    assert fused["ctrl"].device_status() == 0


@pytest.mark.parametrize("policy", ["snapkv", "hotcold"])
def test_fused_step_bench_geometry(policy):
    """The benchmark's layer geometry (fp16, 32/8 heads, budget 512, 64 held): 289 tokens per
    CTA, more than its 256 threads. Fused against the oracle and against the split ops."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    recent = 32 if policy == "snapkv" else 128
    c = dict(B=1, Hq=32, Hk=8, D=128, T=1024, steps=8, dtype="float16", policy=policy, cap=512, recent=recent,
             topk_ratio=0.0 if policy == "snapkv" else 0.5, pool_kernel=7, ccap=4096, faiss_dim=128,
             window_size=1 << 20, pool=4, R=64, hold=True, rap=True, theta=500000.0, seed=77)
    inp = synth.layer_inputs(c["seed"], 1, 32, 8, 128, c["T"], c["steps"], "float16")
    layer, o_outs, o_hot = O.run_layer(inp, c["steps"], **oracle_kwargs(c))
    fused = run_cuda_layer(c, inp, c["steps"], fused=True)
    split = run_cuda_layer(c, inp, c["steps"], fused=False)
    # one launch per fused step, plus the one-launch prompt-end retrieval
    assert fused["ctrl"].arenas[0].launches == c["steps"] + 1, "the fused step did not run"
    for i in range(c["steps"]):
        assert np.array_equal(fused["hot"][i], split["hot"][i]), f"fused vs split hot set, step {i + 1}"
        assert_close(fused["outs"][i], split["outs"][i], "float16", f"fused vs split, step {i + 1}")
    assert _compare_layer(fused, c, layer, o_outs, o_hot, near_tie=2e-3) >= 1
    assert fused["ctrl"].device_status() == 0


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("policy", ["hotcold", "snapkv"])
def test_random_configs_vs_oracle(dtype, policy):
    """Seeded random geometry: batch 2, GQA 4, small budgets so that compression fires at
    prefill and during decode, ring wrap, retrieval every 3 steps with hold."""
    from hotcold_kv_cache_b200 import synth
    c = dict(B=2, Hq=8, Hk=2, D=128, T=300, steps=25, dtype=dtype, policy=policy, cap=64, recent=16,
             topk_ratio=0.5, pool_kernel=7, ccap=200, faiss_dim=128, window_size=3, pool=4, R=12, hold=True,
             rap=True, theta=500000.0, seed=4242)
    inp = synth.layer_inputs(c["seed"], c["B"], c["Hq"], c["Hk"], c["D"], c["T"], c["steps"], dtype)
    layer, o_outs, o_hot = O.run_layer(inp, c["steps"], **oracle_kwargs(c))
    from cuda_runner import run_cuda_layer
    res = run_cuda_layer(c, inp, c["steps"])
    near = 1e-4 if dtype == "float32" else 2e-3 if dtype == "float16" else 2e-2
    steps = _compare_layer(res, c, layer, o_outs, o_hot, near_tie=near)
    assert steps >= 1
    assert res["ctrl"].device_status() == 0


def test_cfg0_full_size():
    """The CPU-runnable configuration at full size: one layer, fp32, 4096-token prompt,
    SnapKV (window 32, max-pool 7, budget 512), prompt-end retrieval of 64 from the last 8
    queries, held, 63 decode steps — compared step by step with the oracle."""
    from hotcold_kv_cache_b200 import synth
    c = dict(B=1, Hq=32, Hk=8, D=128, T=4096, steps=63, dtype="float32", policy="snapkv", cap=512, recent=32,
             topk_ratio=0.0, pool_kernel=7, ccap=4096, faiss_dim=128, window_size=1 << 20, pool=8, R=64,
             hold=True, rap=True, theta=500000.0, seed=0)
    inp = synth.layer_inputs(c["seed"], 1, 32, 8, 128, 4096, 63, "float32")
    layer, o_outs, o_hot = O.run_layer(inp, 63, **oracle_kwargs(c))
    from cuda_runner import run_cuda_layer
    res = run_cuda_layer(c, inp, 63)
    steps = _compare_layer(res, c, layer, o_outs, o_hot)
    assert steps >= 1
    if steps == 63:
        for k, v in layer.dbg.items():
            assert res["ctrl"].dbg[k] == v, k


@pytest.mark.parametrize("dtype,D,recent,T", [("float16", 128, 32, 2048), ("bfloat16", 128, 20, 1537),
                                              ("float16", 64, 8, 2177), ("bfloat16", 64, 32, 1000)])
def test_snapkv_prompt_scoring_tensor_cores(dtype, D, recent, T):
    """Prompt compression of 16-bit layers whose scores exceed one selection CTA: the
    observation x prefix logits run on the tensor cores (M = 128 tokens, N = 16 or 32 rows)
    with ragged tails (T not a multiple of 32 or 128). Hot sets after the prompt and three
    decode steps against the oracle."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(B=2, Hq=32, Hk=8, D=D, T=T, steps=3, dtype=dtype, policy="snapkv", cap=256, recent=recent,
             topk_ratio=0.0, pool_kernel=7, ccap=4096, faiss_dim=D, window_size=1 << 20, pool=4, R=16,
             hold=True, rap=True, theta=500000.0, seed=91 + D + recent)
    inp = synth.layer_inputs(c["seed"], c["B"], c["Hq"], c["Hk"], D, T, c["steps"], dtype)
    layer, o_outs, o_hot = O.run_layer(inp, c["steps"], **oracle_kwargs(c))
    res = run_cuda_layer(c, inp, c["steps"])
    near = 2e-3 if dtype == "float16" else 2e-2
    assert _compare_layer(res, c, layer, o_outs, o_hot, near_tie=near) >= 1
    assert res["ctrl"].device_status() == 0


def _continue(ctrl, c, inp, i0, n):
    """Decode steps i0..i0+n-1 of `inp` on an existing controller (as run_cuda_layer does)."""
    from cuda_runner import TORCH_DT, rotary
    dev = torch.device("cuda", 0)
    dt = TORCH_DT[c["dtype"]]
    rot = rotary(c["Hq"], c["D"], c["theta"], dev)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x).astype(np.float32)).to(device=dev, dtype=dt)
    dq, dk, dv = t(inp["dq"]), t(inp["dk"]), t(inp["dv"])
    outs, hot = [], []
    for i in range(i0, i0 + n):
        pd = torch.full((c["B"],), c["T"] + i, device=dev, dtype=torch.long)
        c1, s1 = rot(torch.empty(1, dtype=dt, device=dev), pd[:, None])
        o = ctrl.decode_layer(0, dq[i], dk[i], dv[i], c1.reshape(c["B"], c["D"]), s1.reshape(c["B"], c["D"]), pd)
        outs.append(o.double().cpu().numpy())
        hot.append(ctrl.arenas[0].hot_positions().cpu().numpy())
    return outs, hot


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_state_dict_resume(dtype, tmp_path):
    """Save the arena and the schedule mid-decode (through torch.save), restore them into a
    new controller, and continue: outputs, hot sets and counters match the run that never
    stopped, bit for bit (retrievals every 3 steps and held segments included)."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import controller_kwargs, rotary, run_cuda_layer
    from hotcold_kv_cache_b200.controller import KVController
    c = dict(B=2, Hq=8, Hk=2, D=128, T=400, steps=12, dtype=dtype, policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=500, faiss_dim=128, window_size=3, pool=4, R=12, hold=True,
             rap=True, theta=500000.0, seed=77)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], c["steps"], dtype)
    res = run_cuda_layer(c, inp, 5)
    ctrl = res["ctrl"]
    sd = ctrl.state_dict()
    path = tmp_path / "arena.pt"
    torch.save(sd, path)
    outs_a, hot_a = _continue(ctrl, c, inp, 5, 7)
    dev = torch.device("cuda", 0)
    ctrl2 = KVController(**controller_kwargs(c))
    rot = rotary(c["Hq"], c["D"], c["theta"], dev)
    ctrl2.set_rotary(rot.inv_freq, rot.attention_scaling)
    ctrl2.load_state_dict(torch.load(path, weights_only=False), dev)
    outs_b, hot_b = _continue(ctrl2, c, inp, 5, 7)
    for i in range(7):
        assert np.array_equal(outs_a[i], outs_b[i]), f"output, step {6 + i}"
        assert np.array_equal(hot_a[i], hot_b[i]), f"hot set, step {6 + i}"
    assert ctrl.dbg == ctrl2.dbg
    assert ctrl2.device_status() == 0


@pytest.mark.parametrize("dtype,policy,chunks", [
    ("float16", "snapkv", [0, 300, 301, 700, 1200]),
    ("float32", "hotcold", [0, 64, 500, 1200]),
    ("bfloat16", "snapkv", [0, 1200]),
])
def test_chunked_prefill_vs_oracle(dtype, policy, chunks):
    """A prompt forwarded in chunks (ragged sizes, a one-token chunk, a chunk within the
    budget): hot sets, cold rings and the decode steps after it against the oracle's chunked
    prefill; one chunk is the plain prefill."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import cold_positions, run_cuda_layer
    c = dict(B=2, Hq=8, Hk=2, D=128, T=1200, steps=6, dtype=dtype, policy=policy, cap=128,
             recent=16 if policy == "snapkv" else 32, topk_ratio=0.0 if policy == "snapkv" else 0.5, pool_kernel=7,
             ccap=2000, faiss_dim=128, window_size=1 << 20, pool=8, R=16, hold=True, rap=True, theta=500000.0,
             seed=515)
    inp = synth.layer_inputs(c["seed"], 2, 8, 2, 128, c["T"], c["steps"], dtype)
    layer, o_outs, o_hot = O.run_layer(inp, c["steps"], chunks=chunks, **oracle_kwargs(c))
    res = run_cuda_layer(c, inp, c["steps"], chunks=chunks)
    near = 1e-4 if dtype == "float32" else 2e-3 if dtype == "float16" else 2e-2
    steps = _compare_layer(res, c, layer, o_outs, o_hot, near_tie=near)
    assert steps >= 1
    if steps == c["steps"]:
        got = cold_positions(res["ctrl"])
        want = layer.cold_positions()
        for b in range(2):
            assert np.array_equal(np.sort(got[b]), np.sort(want[b])), f"cold ring of sequence {b}"
        for k, v in layer.dbg.items():
            assert res["ctrl"].dbg[k] == v, k
    assert res["ctrl"].device_status() == 0


@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_split_attention_large_batch_vs_oracle(dtype):
    """The split-path attention for batches that fill the GPU (16 sequences x 8 KV heads x
    3 blocks of 256 rows): four double-buffered chunks per CTA with an online softmax. Against
    the oracle, with retrieval and a held segment."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(B=16, Hq=32, Hk=8, D=128, T=700, steps=3, dtype=dtype, policy="snapkv", cap=512, recent=32,
             topk_ratio=0.0, pool_kernel=7, ccap=1000, faiss_dim=128, window_size=2, pool=1, R=16, hold=True,
             rap=True, theta=500000.0, seed=2024)
    inp = synth.layer_inputs(c["seed"], 16, 32, 8, 128, c["T"], c["steps"], dtype)
    layer, o_outs, o_hot = O.run_layer(inp, c["steps"], **oracle_kwargs(c))
    res = run_cuda_layer(c, inp, c["steps"], fused=False)
    near = 1e-4 if dtype == "float32" else 2e-3
    assert _compare_layer(res, c, layer, o_outs, o_hot, near_tie=near) >= 1
    assert res["ctrl"].device_status() == 0
