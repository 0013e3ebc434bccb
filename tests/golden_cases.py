"""Loading helpers for the committed golden vectors (tests/golden/*.npz) and the
oracle configuration that matches each single-layer case."""

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYER_CASES = ("hotcold_f32", "snapkv_f32", "hotcold_f16_b2", "hotcold_f16_once")


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)
    d = {k: z[k] for k in z.files}
    for k in ("case", "dbg"):
        if k in d:
            d[k] = json.loads(str(d[k]))
    return d


def oracle_kwargs(case):
    """OracleLayer keyword arguments for a single-layer golden case."""
    from oracle.hotcold_oracle import Policy
    from hotcold_kv_cache_b200 import synth
    c = case
    return dict(Hq=c["Hq"], Hk=c["Hk"], D=c["D"], dtype=c["dtype"],
                inv_freq=synth.rope_inv_freq(c["D"], c["theta"]), attention_scaling=1.0,
                policy=Policy(policy=c["policy"], cap=c["cap"], recent=c["recent"],
                              topk_ratio=c["topk_ratio"], pool_kernel=c["pool_kernel"],
                              pooling=c.get("pooling", "maxpool")),
                cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], normalize_for_ip=True,
                window_size=c["window_size"], query_pool_size=c["pool"], lookahead_k=c["R"],
                hold_retrieved=c["hold"], retrieve_after_prefill=c["rap"],
                retrieval_lag=1 if c.get("async") else 0)


def inputs(case):
    from hotcold_kv_cache_b200 import synth
    c = case
    return synth.layer_inputs(c["seed"], c["B"], c["Hq"], c["Hk"], c["D"], c["T"], c["steps"], c["dtype"])


def split_hot(g):
    """Per-step hot positions (B, len) from the concatenated golden layout."""
    out, off = [], 0
    for n in g["hot_len"]:
        out.append(g["hot_pos"][:, off:off + n])
        off += n
    return out


REL_TOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 1.6e-2}


def assert_close(actual, desired, dtype, what=""):
    """Relative agreement at the tolerance of `dtype` (1e-5 fp32, 2e-3 fp16),
    measured against the magnitude of the desired tensor: every element must
    satisfy |a - d| <= rel * max|d| + rel * |d|. NaNs must match."""
    a = np.asarray(actual, np.float64)
    d = np.asarray(desired, np.float64)
    assert a.shape == d.shape, (what, a.shape, d.shape)
    na, nd = np.isnan(a), np.isnan(d)
    assert np.array_equal(na, nd), f"{what}: NaN pattern differs"
    a, d = np.where(na, 0, a), np.where(nd, 0, d)
    rel = REL_TOL[dtype]
    scale = max(np.abs(d).max(), 1e-30)
    err = np.abs(a - d) - rel * np.abs(d)
    worst = float(err.max() / scale) if err.size else 0.0
    assert worst <= rel, f"{what}: max scaled error {worst:.3e} > {rel:.1e}"


# the fp16 band of a comparison with the reference's own fp16-logit selections: its logits are
# rounded to fp16, so its scores carry relative errors up to about 1e-3
REF_F16_BAND = 2e-3


def assert_keep_within_band(kept_pos, ref_keep, ref_scores, prefix_len, n_top, band=REF_F16_BAND, what=""):
    """A prompt compression's kept positions against the reference's keep set: equal, except
    for tokens of the prefix whose reference score lies within `band` (relative) of both sides
    of the reference's own top-n_top boundary. Returns the number of such swaps."""
    sc = np.asarray(ref_scores, np.float64)[:prefix_len]
    got = set(int(x) for x in np.asarray(kept_pos).ravel())
    want = set(int(x) for x in np.asarray(ref_keep).ravel())
    assert len(got) == len(want), f"{what}: kept {len(got)} tokens, reference {len(want)}"
    order = np.sort(sc)[::-1]
    thr_in, thr_out = order[n_top - 1], order[n_top]
    rel = lambda a, b: abs(a - b) / max(abs(a), abs(b), 1e-300)
    diff = got ^ want
    for t in diff:
        assert t < prefix_len, f"{what}: the recent window differs at {t}"
        g = max(rel(sc[t], thr_in), rel(sc[t], thr_out))
        assert g <= band, f"{what}: token {t} kept/evicted differently, {g:.2e} from the boundary"
    return len(diff) // 2
