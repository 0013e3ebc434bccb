"""Step-exact comparison of a CUDA run with the oracle over every step.

The CUDA path scores in float32 and the oracle in float64, so where two candidates of a
top-k boundary (a compression's keep set, a cold search's hits) are within rounding of each
other the two may choose differently, and from there on their states would differ. Instead
of stopping the comparison there, the oracle adopts the CUDA selection, but only after
checking that every token it swaps in or out scores within `near` (relative) of the token it
replaces at the boundary; any other difference fails at once. The comparison then goes on
with identical states, so every step is compared.

BASELINE's rule: kept and retrieved index sets match exactly except where score gaps are
within 1e-4 relative. That is the default band here.
"""

import numpy as np

from golden_cases import assert_close

NEAR = 1e-4


def _rel(a, b):
    return abs(a - b) / max(abs(a), abs(b), 1e-300)


class FollowCuda:
    """Resolvers for OracleLayer.resolve_keep / resolve_hits built from one CUDA run (the dict
    of cuda_runner.run_cuda_layer for one layer: hot0, hot, held). `adopted` lists every
    adoption as (kind, step, b, worst relative gap)."""

    def __init__(self, res, near=NEAR):
        self.res, self.near = res, near
        self.adopted = []
        self.layer = None

    def attach(self, layer):
        self.layer = layer
        layer.resolve_keep = self.keep
        layer.resolve_hits = self.hits

    def keep(self, step, b, sc, prefix_len, n_top, top, P_b):
        if step == 0:
            after = self.res["hot0"][getattr(self.layer, "chunk_index", 0)][b]
        else:
            after = self.res["hot"][step - 1][b]
        cset = set(np.asarray(after).tolist())
        ctop = np.array([t for t in range(prefix_len) if int(P_b[t]) in cset], np.int64)
        if np.array_equal(ctop, top):
            return top
        assert len(ctop) == n_top, f"step {step} seq {b}: CUDA kept {len(ctop)} of the prefix, oracle {n_top}"
        order = np.lexsort((np.arange(prefix_len), -sc))
        thr_in, thr_out = sc[order[n_top - 1]], sc[order[n_top]] if n_top < prefix_len else -np.inf
        swapped = np.setxor1d(ctop, top)
        worst = 0.0
        for t in swapped:
            # a token on the wrong side of the boundary must score within `near` of both sides
            g = max(_rel(sc[t], thr_in), _rel(sc[t], thr_out))
            worst = max(worst, g)
            assert g <= self.near, (f"step {step} seq {b}: kept set differs at token {t} (pos {int(P_b[t])}), "
                                    f"score {sc[t]:.9g} vs boundary {thr_in:.9g}/{thr_out:.9g}, gap {g:.2e}")
        self.adopted.append(("keep", step, b, worst))
        return ctop

    def hits(self, step, b, sc, ids, ring_pos):
        if step == 0 and 1 in self.res.get("launched", ()):
            # the prompt-end retrieval is replaced by the search of decode step 1 before it is
            # attended: nothing of it is observable in either run
            return ids
        st = max(step, 1)
        if st not in self.res["held"] and st > len(self.res["hot"]):
            return ids  # a search attended only after the last compared step (one-step lag)
        assert st in self.res["held"], f"the CUDA run injected nothing at step {st}"
        pos, valid, _ = self.res["held"][st]
        cpos = pos[b][valid[b]]
        where = {int(p): i for i, p in enumerate(ring_pos)}
        assert all(int(p) in where for p in cpos), f"step {step} seq {b}: CUDA hit outside the ring"
        cids = np.array([where[int(p)] for p in cpos], np.int64)
        if np.array_equal(cids, ids):
            return ids
        assert len(cids) == len(ids), f"step {step} seq {b}: {len(cids)} CUDA hits, oracle {len(ids)}"
        worst = 0.0
        for j in np.nonzero(cids != ids)[0]:
            g = _rel(sc[cids[j]], sc[ids[j]])
            worst = max(worst, g)
            assert g <= self.near, (f"step {step} seq {b}: hit {j} differs (ring {cids[j]} vs {ids[j]}), "
                                    f"scores {sc[cids[j]]:.9g} vs {sc[ids[j]]:.9g}, gap {g:.2e}")
        self.adopted.append(("hits", step, b, worst))
        return cids


def run_following(O, inputs, n_steps, res, near=NEAR, chunks=None, **kw):
    """O.run_layer with the oracle following the CUDA run `res` at near-ties. Returns
    (layer, outs, hot, follow)."""
    fc = FollowCuda(res, near)
    layer, outs, hot = O.run_layer(inputs, n_steps, chunks=chunks, follow=fc, **kw)
    return layer, outs, hot, fc


def assert_same_run(res, layer, o_outs, o_hot, dtype, n_steps, what=""):
    """Every step: hot set equal, attention output within the dtype's tolerance; every
    retrieval: same injection step, positions, validity and re-rotated held keys."""
    assert len(res["hot"]) == n_steps and len(o_hot) == n_steps
    for i in range(n_steps):
        assert np.array_equal(res["hot"][i], o_hot[i]), f"{what} hot set differs at step {i + 1}"
        assert_close(res["outs"][i], o_outs[i], dtype, f"{what} attention step {i + 1}")
    want = [e["step"] for e in layer.events]
    assert sorted(res["held"]) == want, f"{what} injection steps {sorted(res['held'])} vs {want}"
    for e in layer.events:
        pos, valid, k = res["held"][e["step"]]
        assert np.array_equal(valid, e["valid"]), f"{what} held validity, step {e['step']}"
        assert np.array_equal(pos[valid], e["pos"][e["valid"]]), f"{what} held positions, step {e['step']}"
        assert_close(k, e["kmem"], dtype, f"{what} held keys step {e['step']}")
    return n_steps
