"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py). CPU only."""

import math

import numpy as np
import pytest

from golden_cases import LAYER_CASES, assert_close, inputs, load, oracle_kwargs, split_hot
from hotcold_kv_cache_b200 import synth
from oracle import hotcold_oracle as O


@pytest.mark.parametrize("name", LAYER_CASES)
def test_layer_case(name):
    g = load(name)
    c = g["case"]
    layer, outs, hot = O.run_layer(inputs(c), c["steps"], **oracle_kwargs(c))
    # attention outputs of every decode step
    assert_close(outs, g["outs"], c["dtype"], "attention outputs")
    # hot tier contents (positions, logical order) after every step
    for step, (a, b) in enumerate(zip(hot, split_hot(g))):
        assert np.array_equal(a, b), f"hot set differs at step {step + 1}"
    # cold ring contents at the end
    if g["cold_pos"].size:
        cold = layer.cold_positions()
        assert np.array_equal(np.stack(cold), g["cold_pos"])
    # retrieved sets and the re-rotated held keys of the first one
    if "ret_pos" in g:
        assert len(layer.events) == g["ret_pos"].shape[0]
        for e, p, v in zip(layer.events, g["ret_pos"], g["ret_valid"]):
            assert np.array_equal(e["valid"], v)
            assert np.array_equal(e["pos"], p)
        # the reference returns (B,1,Hk,R,D) here (its broadcast adds a dim; patch.py:250 squeezes it)
        km = layer.events[0]["kmem"]
        assert_close(km, g["kmem0"].reshape(km.shape), c["dtype"], "held keys")
    # debug counters (the reference counts Triton calls only on CUDA)
    for k, v in g["dbg"].items():
        if k in O.DBG_KEYS:
            assert layer.dbg[k] == v, (k, layer.dbg[k], v)


def test_scores_function_level():
    g = load("scores")
    Hq, Hk, D, W = 32, 8, 128, 32
    for dt, (q, k) in synth.score_case_inputs(11).items():
        tag = "f32" if dt == "float32" else "f16"
        q = q.astype(np.float64)[0]
        k = k.astype(np.float64)[0]
        snap = O.snapkv_token_scores(q[:, -W:], k, 1.0 / math.sqrt(D), 7, "maxpool", dt)
        hc = O.hotcold_token_scores(q[:, -W:], k, dt)
        rt = 1e-5 if dt == "float32" else 3e-3
        np.testing.assert_allclose(snap, g[f"snap_{tag}"][0], rtol=rt, atol=rt * np.abs(snap).max())
        np.testing.assert_allclose(hc, g[f"hc_{tag}"][0], rtol=rt, atol=rt * np.abs(hc).max())
    # keep_index on float32 scores (no ties): top-(budget - window) prefix + window
    sc = g["ki_scores"].astype(np.float64)
    for b in range(sc.shape[0]):
        for h in range(sc.shape[1]):
            top = O.topk_lower_index(sc[b, h, :92], 22)
            assert np.array_equal(np.concatenate([top, np.arange(92, 100)]), g["ki_full"][b, h])
    x = g["pool_x"].astype(np.float64)
    np.testing.assert_allclose(O.pool1d(x, 7, "maxpool"), g["pool_max"], rtol=1e-6)
    np.testing.assert_allclose(O.pool1d(x, 7, "avgpool"), g["pool_avg"], rtol=1e-5, atol=1e-6)


def test_reference_decode_kernel():
    g = load("triton_kernel")
    q, k, v, m = synth.attention_case_inputs(7)
    out = O.decode_attention(q[:, :, 0], k, v, m, 1.0 / math.sqrt(q.shape[-1]), "float32")
    assert_close(out, g["out"][:, 0], "float32", "attention")
    idx = O.evict_loss_argmin(q[:, :, 0], k, v, m, 1.0 / math.sqrt(q.shape[-1]), "float32")
    assert np.array_equal(idx, g["evict_idx"])


def test_decode_attention_edge_cases():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 4, 16))
    k = rng.standard_normal((1, 1, 5, 16))
    v = rng.standard_normal((1, 1, 5, 16))
    # nothing unmasked: the reference divides 0 by 0
    assert np.isnan(O.decode_attention(q, k, v, np.zeros((1, 5), bool), 0.25, "float32")).all()
    # an fp32 exp overflow of the unstabilised softmax
    big = k.copy()
    big[0, 0, 2] = q[0, 0] * 100
    out = O.decode_attention(q, big, v, np.ones((1, 5), bool), 0.25, "float32")
    assert np.isnan(out[0, 0]).all()


def test_snapkv_f16_prompt_compression():
    """fp16 SnapKV prompt compression (2048 tokens, window 32, max-pool 7, budget 256): the
    oracle's token scores against the reference's own (fp16 logits, scoring.py:50-79 averaged
    over heads), and its keep set against the reference's keep_index (scoring.py:110-132) up to
    tokens within the fp16 band of the reference's boundary."""
    from golden_cases import assert_keep_within_band
    g = load("snapkv_f16_prompt")
    c = g["case"]
    inp = inputs(c)
    T, W = c["T"], c["recent"]
    inv = synth.rope_inv_freq(c["D"], c["theta"])
    cos, sin = O.rope_cos_sin(np.arange(T), inv, 1.0, c["dtype"])
    qp = O.apply_rope(inp["q_pre"][0], cos, sin, c["dtype"])
    kp = O.apply_rope(inp["k_pre"][0], cos, sin, c["dtype"])
    sc = O.snapkv_token_scores(qp[:, -W:], kp, 1.0 / math.sqrt(c["D"]), c["pool_kernel"], "maxpool", c["dtype"])
    ref = g["token_scores"][0].astype(np.float64)
    err = np.abs(sc - ref) / np.abs(ref).max()
    assert err.max() <= 3e-3, err.max()
    prefix, ntop = T - W, c["cap"] - W
    keep = np.concatenate([O.topk_lower_index(sc[:prefix], ntop), np.arange(prefix, T)])
    assert_keep_within_band(keep, g["keep_idx"][0], ref, prefix, ntop, what="oracle vs reference")
