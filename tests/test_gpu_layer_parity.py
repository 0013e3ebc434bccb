"""CUDA hot path of one layer against the CPU oracle and against the golden
vectors of the reference itself: attention outputs, hot sets after every step,
cold ring contents, retrieved sets, re-rotated held keys and debug counters.

Every test compares every step. Where the oracle's selection (float64 scores) and the CUDA
path's (float32) differ only at a near-tie of the top-k boundary (relative gap <= 1e-4), the
oracle adopts the CUDA selection and the comparison goes on (tests/oracle_follow.py)."""

import math

import numpy as np
import pytest
import torch

from golden_cases import LAYER_CASES, assert_close, inputs, load, oracle_kwargs, split_hot
from oracle_follow import NEAR, assert_same_run, run_following

pytestmark = pytest.mark.gpu

from oracle import hotcold_oracle as O  # noqa: E402


def _run(case, model_cos=True):
    from cuda_runner import run_cuda_layer
    return run_cuda_layer(case, inputs(case), case["steps"], model_cos=model_cos)


def _oracle(c, inp, res, chunks=None, near=NEAR):
    """The oracle over the same inputs, following the CUDA run at near-ties (gap <= near)."""
    return run_following(O, inp, c["steps"], res, near=near, chunks=chunks, **oracle_kwargs(c))


@pytest.mark.parametrize("name", LAYER_CASES)
@pytest.mark.parametrize("model_cos", [True, False])
def test_layer_vs_oracle_and_golden(name, model_cos):
    g = load(name)
    c = g["case"]
    res = _run(c, model_cos)
    layer, o_outs, o_hot, fc = _oracle(c, inputs(c), res)
    assert fc.adopted == [], "golden cases are chosen free of near-ties"
    assert assert_same_run(res, layer, o_outs, o_hot, c["dtype"], c["steps"]) == c["steps"]
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


def bench_case(policy="snapkv", steps=63, T=8192):
    """The benchmark's layer configuration (bench.py config()): fp16, 32/8 heads, D 128, an
    8192-token prompt compressed to budget 512, top-64 retrieval every 16 steps from a pool of
    4 queries, held until replaced, no prompt-end retrieval."""
    recent = 32 if policy == "snapkv" else 128
    return dict(B=1, Hq=32, Hk=8, D=128, T=T, steps=steps, dtype="float16", policy=policy, cap=512,
                recent=recent, topk_ratio=0.0 if policy == "snapkv" else max(0.05, 0.75 - recent / 512),
                pool_kernel=7, ccap=32768, faiss_dim=128, window_size=16, pool=4, R=64, hold=True, rap=False,
                theta=500000.0, seed=1234)


def test_bench_configuration_all_steps():
    """The exact layer configuration bench.py times, two layers chained as in a model (each
    layer's step launched right after the previous layer's), 63 decode steps through the fused
    step with the decode-step retrievals (steps 15, 31, 47, 63) through hc_retrieve_decode;
    every step of both layers against the oracle: hot sets, attention outputs, retrieved sets
    and re-rotated held keys, counters."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layers
    c = bench_case()
    ins = [synth.layer_inputs(c["seed"] + li, 1, 32, 8, 128, c["T"], c["steps"], "float16") for li in range(2)]
    res = run_cuda_layers(c, ins, c["steps"], fused=True)
    ctrl = res[0]["ctrl"]
    # one step_kernel per layer-step, one retr_kernel per search, nothing else
    n_search = (c["steps"] + 1) // c["window_size"]  # the prompt counts as a forward: steps 15, 31, 47, 63
    for li in range(2):
        assert ctrl.arenas[li].launches == c["steps"] + n_search, "the fused kernels did not run"
    for li in range(2):
        layer, o_outs, o_hot, fc = _oracle(c, ins[li], res[li])
        assert assert_same_run(res[li], layer, o_outs, o_hot, "float16", c["steps"], f"layer {li}") == 63
        assert [e["step"] for e in layer.events] == [15, 31, 47, 63]
        assert len(layer.compress_log) == 1 + c["steps"]
        for k, v in layer.dbg.items():
            assert ctrl.dbg[k] == 2 * v, (k, ctrl.dbg[k], v)
    assert ctrl.device_status() == 0


def test_bench_configuration_async_retrieval():
    """bench.py's layer configuration with async_retrieval: each decode-step search runs on a
    side stream after the step's compression and is attended from the next step. Two layers,
    63 steps, every step against the oracle run with the same one-step lag (searches at steps
    15, 31, 47, 63 attended at 16, 32, 48; the last falls after the run)."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layers
    c = dict(bench_case(), **{"async": True})
    ins = [synth.layer_inputs(c["seed"] + li, 1, 32, 8, 128, c["T"], c["steps"], "float16") for li in range(2)]
    res = run_cuda_layers(c, ins, c["steps"], fused=True)
    ctrl = res[0]["ctrl"]
    n_search = (c["steps"] + 1) // c["window_size"]
    for li in range(2):
        a = ctrl.arenas[li]
        per_search = 1 if a._retr_fused() else 4
        assert a.launches == c["steps"] + n_search * per_search, "the fused step did not run"
        assert sorted(res[li]["launched"]) == [15, 31, 47, 63]
    for li in range(2):
        layer, o_outs, o_hot, fc = _oracle(c, ins[li], res[li])
        assert assert_same_run(res[li], layer, o_outs, o_hot, "float16", c["steps"], f"layer {li}") == 63
        assert [e["step"] for e in layer.events] == [16, 32, 48]
        for k, v in layer.dbg.items():
            assert ctrl.dbg[k] == 2 * v, (k, ctrl.dbg[k], v)
    assert ctrl.device_status() == 0


def test_back_to_back_steps_of_one_layer():
    """One layer's decode steps launched back to back, nothing read in between: each fused step
    may start while the previous one (same layer) still runs, so it must not read that layer's
    state before its dependency wait. Outputs, hot set, cold ring and held segment equal, bit for
    bit, those of the same run synchronised after every step (which the tests above check
    against the oracle)."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import TORCH_DT, cold_positions, rotary, run_cuda_layer
    c = dict(bench_case(steps=40, T=2048), window_size=8)
    inp = synth.layer_inputs(c["seed"], 1, 32, 8, 128, c["T"], c["steps"], "float16")
    ref = run_cuda_layer(c, inp, c["steps"])
    from cuda_runner import controller_kwargs
    from hotcold_kv_cache_b200.controller import KVController
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    dev = torch.device("cuda", 0)
    dt = TORCH_DT["float16"]
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x).astype(np.float32)).to(device=dev, dtype=dt)
    rot = rotary(32, 128, c["theta"], dev)
    ctrl = KVController(**controller_kwargs(c))
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    q_pre, k_pre, v = t(inp["q_pre"]), t(inp["k_pre"]), t(inp["v"])
    ctrl._lazy_init(k_pre, n_layers=1)
    pos = torch.arange(c["T"], device=dev)[None]
    cos, sin = rot(torch.empty(1, dtype=dt, device=dev), pos)
    q_post, k_post = apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
    ctrl.prefill_layer(0, q_pre, q_post, k_pre, k_post, v, pos)
    dq, dk, dv = t(inp["dq"]), t(inp["dk"]), t(inp["dv"])
    pd = torch.arange(c["T"], c["T"] + c["steps"], device=dev)
    cs, sn = rot(torch.empty(1, dtype=dt, device=dev), pd[None])
    cs, sn = cs[0].contiguous(), sn[0].contiguous()
    out = torch.empty((c["steps"], 1, 32, 128), dtype=dt, device=dev)
    torch.cuda.synchronize(dev)
    for i in range(c["steps"]):
        ctrl.decode_layer(0, dq[i], dk[i], dv[i], cs[i:i + 1], sn[i:i + 1], pd[i:i + 1], out=out[i])
    got = out.double().cpu().numpy()
    assert np.array_equal(got, ref["outs"])
    a, b = ctrl.arenas[0], ref["ctrl"].arenas[0]
    assert np.array_equal(a.hot_positions().cpu().numpy(), ref["hot"][-1])
    assert np.array_equal(cold_positions(ctrl)[0], cold_positions(ref["ctrl"])[0])
    for name in ("held_k", "held_v", "held_pos", "held_valid"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    assert ctrl.dbg == ref["ctrl"].dbg
    assert a.launches == b.launches == c["steps"] + (c["steps"] + 1) // c["window_size"]
    assert ctrl.device_status() == 0


@pytest.mark.parametrize("policy", ["snapkv", "hotcold"])
def test_fused_step_bench_geometry(policy):
    """The benchmark's layer geometry (fp16, 32/8 heads, budget 512, 64 held): 289 tokens per
    CTA, more than its 256 threads. Fused against the oracle over every step and against the
    split ops, with a 1024-token prompt and a search every 4 steps."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import run_cuda_layer
    c = dict(bench_case(policy, steps=12, T=1024), window_size=4, rap=True, ccap=4096, seed=77)
    inp = synth.layer_inputs(c["seed"], 1, 32, 8, 128, c["T"], c["steps"], "float16")
    fused = run_cuda_layer(c, inp, c["steps"], fused=True)
    split = run_cuda_layer(c, inp, c["steps"], fused=False)
    for i in range(c["steps"]):
        assert np.array_equal(fused["hot"][i], split["hot"][i]), f"fused vs split hot set, step {i + 1}"
        assert_close(fused["outs"][i], split["outs"][i], "float16", f"fused vs split, step {i + 1}")
    layer, o_outs, o_hot, _ = _oracle(c, inp, fused)
    assert assert_same_run(fused, layer, o_outs, o_hot, "float16", c["steps"]) == c["steps"]
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
    from cuda_runner import run_cuda_layer
    res = run_cuda_layer(c, inp, c["steps"])
    layer, o_outs, o_hot, _ = _oracle(c, inp, res)
    assert assert_same_run(res, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
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
    from cuda_runner import run_cuda_layer
    res = run_cuda_layer(c, inp, 63)
    layer, o_outs, o_hot, _ = _oracle(c, inp, res)
    assert assert_same_run(res, layer, o_outs, o_hot, "float32", 63) == 63
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
    res = run_cuda_layer(c, inp, c["steps"])
    layer, o_outs, o_hot, _ = _oracle(c, inp, res)
    assert assert_same_run(res, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
    assert res["ctrl"].device_status() == 0


@pytest.mark.parametrize("T,ccap,ties,pooling", [(9000, 4096, False, "maxpool"), (9000, 9000, False, "avgpool"),
                                                 (20000, 20000, True, "maxpool"), (40000, 40000, False, "maxpool"),
                                                 (70000, 70000, True, "maxpool")])
def test_prompt_selection_cluster_sizes(T, ccap, ties, pooling):
    """Long prompts, whose keep / evict lists come from a cluster of 16 CTAs: 9000 tokens, one
    per thread, the token scores computed by the cluster; 20000, 40000 and 70000 tokens, 2, 3
    and 5 per thread, after token_kernel (shorter prompts, on clusters of 1 to 8 CTAs, are the
    other tests' cases). Hot set, cold ring (9000 tokens into a ring of 4096: only the last 4096
    evicted are stored; once with average pooling) and one decode step against the oracle.
    With `ties`, every prefix key but 64 is zero, so the top-k boundary falls inside one group
    of exactly equal scores that spans every CTA of the cluster, and the lower positions are
    the ones kept."""
    from hotcold_kv_cache_b200 import synth
    from cuda_runner import cold_positions, run_cuda_layer
    c = dict(B=1, Hq=8, Hk=2, D=128, T=T, steps=1, dtype="float16", policy="snapkv", cap=512, recent=32,
             topk_ratio=0.0, pool_kernel=7, ccap=ccap, faiss_dim=128, window_size=1 << 20, pool=4, R=16,
             hold=True, rap=not ties, theta=500000.0, seed=5 + T, pooling=pooling)
    inp = synth.layer_inputs(c["seed"], 1, 8, 2, 128, T, 1, "float16")
    if ties:
        live = np.zeros(T, bool)
        live[np.random.default_rng(T).choice(T - 32, 64, replace=False)] = True
        live[T - 32:] = True
        inp["k_pre"][:, :, ~live] = 0
    res = run_cuda_layer(c, inp, 1)
    layer, o_outs, o_hot, fc = _oracle(c, inp, res)
    if ties:
        assert fc.adopted == []
    assert assert_same_run(res, layer, o_outs, o_hot, "float16", 1) == 1
    for got, want in zip(cold_positions(res["ctrl"]), layer.cold_positions()):
        assert np.array_equal(got, want)
    assert res["ctrl"].device_status() == 0


def test_snapkv_f16_prompt_vs_reference():
    """The tensor-core prompt scoring (fp16, 2048 tokens, window 32, max-pool 7, budget 256)
    against the reference's own SnapKV selection (tests/golden/snapkv_f16_prompt.npz): kept set
    equal up to tokens within the fp16 band of the reference's boundary; then the prompt and one
    decode step against the oracle, every selection within 1e-4."""
    from golden_cases import assert_keep_within_band
    from cuda_runner import run_cuda_layer
    g = load("snapkv_f16_prompt")
    c = g["case"]
    inp = inputs(c)
    res = run_cuda_layer(c, inp, c["steps"])
    T, W = c["T"], c["recent"]
    assert_keep_within_band(res["hot0"][0][0], g["keep_idx"][0], g["token_scores"][0], T - W, c["cap"] - W,
                            what="CUDA vs reference")
    layer, o_outs, o_hot, _ = _oracle(c, inp, res)
    assert assert_same_run(res, layer, o_outs, o_hot, "float16", c["steps"]) == c["steps"]
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
    res = run_cuda_layer(c, inp, c["steps"], chunks=chunks)
    layer, o_outs, o_hot, _ = _oracle(c, inp, res, chunks=chunks)
    assert assert_same_run(res, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
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
    res = run_cuda_layer(c, inp, c["steps"], fused=False)
    layer, o_outs, o_hot, _ = _oracle(c, inp, res)
    assert assert_same_run(res, layer, o_outs, o_hot, dtype, c["steps"]) == c["steps"]
    assert res["ctrl"].device_status() == 0
