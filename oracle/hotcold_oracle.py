"""CPU oracle for the hot/cold per-layer decode path.

TEST INFRASTRUCTURE ONLY. This module is a numpy restatement of the reference
algorithm (tarun931/hotcold-kv-cache, `src/hotcold_kv`). Only `tests/`,
`__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py` may import it,
and only as the checker or the timed CPU baseline. The product path never
calls it.

Parity pinning: this restatement is checked against golden vectors produced by
running the reference's own Python code (with the shims listed in
`tests/golden/make_golden.py`), committed under `tests/golden/`.

Arithmetic model. Values of the model dtype (float32 / float16 / bfloat16) are
carried in float64 arrays that hold dtype-representable numbers. Where the
reference rounds to the model dtype (RoPE, GQA query means, the pooled query
vector, the attention output) the oracle rounds too; everything else
(dot products, softmax, sums) runs in float64. Top-k ties go to the lower
index, the tie rule the CUDA path implements.
"""

from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass, field

import numpy as np

EXP_OVERFLOW_F32 = 88.72283935546875  # logits at or above this overflow fp32 exp


# ---------------------------------------------------------------------------
# dtype rounding
# ---------------------------------------------------------------------------
def rnd(x, dt: str) -> np.ndarray:
    """Round to `dt` and return float64 (`dt` in float32/float16/bfloat16)."""
    x = np.asarray(x, dtype=np.float64)
    if dt == "float32":
        return x.astype(np.float32).astype(np.float64)
    if dt == "float16":
        return x.astype(np.float16).astype(np.float64)
    if dt == "bfloat16":
        f = x.astype(np.float32)
        b = f.view(np.uint32).astype(np.uint64)
        b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
        return b.astype(np.uint32).view(np.float32).astype(np.float64)
    raise ValueError(dt)


# ---------------------------------------------------------------------------
# RoPE  (HF LlamaRotaryEmbedding.forward / apply_rotary_pos_emb / rotate_half,
#        used by patch.py:161-162 and patch.py:76-102)
# ---------------------------------------------------------------------------
def rope_cos_sin(pos, inv_freq, attention_scaling: float, dt: str):
    """cos/sin tables (len(pos), D) in `dt`.

    HF forms the angle as a float32 product inv_freq * float(pos), duplicates it
    over both halves, takes cos/sin in float32, scales by attention_scaling and
    casts to the model dtype (transformers modeling_llama.py
    LlamaRotaryEmbedding.forward). cos/sin are evaluated in float64 and rounded
    to float32, i.e. correctly rounded.
    """
    pos = np.asarray(pos, dtype=np.int64).reshape(-1)
    inv = np.asarray(inv_freq, dtype=np.float32)
    ang = (inv[None, :] * pos.astype(np.float32)[:, None]).astype(np.float32)
    ang = np.concatenate([ang, ang], axis=-1).astype(np.float64)
    c = np.cos(ang).astype(np.float32) * np.float32(attention_scaling)
    s = np.sin(ang).astype(np.float32) * np.float32(attention_scaling)
    return rnd(c.astype(np.float32), dt), rnd(s.astype(np.float32), dt)


def apply_rope(x, cos, sin, dt: str):
    """(x * cos) + (rotate_half(x) * sin), each op rounded to `dt`.
    x (..., D); cos/sin broadcastable to x."""
    x = np.asarray(x, dtype=np.float64)
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return rnd(rnd(x * cos, dt) + rnd(rot * sin, dt), dt)


# ---------------------------------------------------------------------------
# decode attention  (kernels.py:9-74, wrapper kernels.py:77-137)
# ---------------------------------------------------------------------------
def decode_attention(q, K, V, mask, scale: float, dt: str):
    """Single-query attention with GQA.

    q (B,Hq,D), K/V (B,Hk,S,D), mask (B,S) bool -> out (B,Hq,D) in `dt`.
    The reference kernel exponentiates raw scores without subtracting a max
    (kernels.py:144-153): masked scores become -1e35 and contribute 0; a row
    with no unmasked token divides 0 by 0; a score whose fp32 exp overflows
    makes every output of that head NaN. The oracle reproduces those three
    outcomes and otherwise computes the softmax stably in float64.
    """
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    B, Hq, D = q.shape
    Hk = K.shape[1]
    g = Hq // Hk
    sc = float(np.float32(scale))
    out = np.empty((B, Hq, D), dtype=np.float64)
    for b in range(B):
        m = np.asarray(mask[b], dtype=bool)
        for h in range(Hq):
            kh = h // g
            s = (K[b, kh] @ q[b, h]) * sc
            if not m.any():
                out[b, h] = np.nan
                continue
            mx = s[m].max()
            if mx >= EXP_OVERFLOW_F32:
                out[b, h] = np.nan
                continue
            p = np.where(m, np.exp(s - mx), 0.0)
            out[b, h] = (p @ V[b, kh]) / p.sum()
    return rnd(out, dt)


def evict_loss_argmin(q, K, V, mask, scale: float, dt: str):
    """The wrapper's second output (kernels.py:134-137): per token
    mean over q-heads of softmax-prob * sum_d |v_d| / D, cast to the query dtype,
    argmin over the sequence (first index on ties). -> (B,) int64."""
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    B, Hq, D = q.shape
    Hk = K.shape[1]
    g = Hq // Hk
    sc = float(np.float32(scale))
    res = np.zeros(B, dtype=np.int64)
    for b in range(B):
        m = np.asarray(mask[b], dtype=bool)
        acc = np.zeros(K.shape[2])
        for h in range(Hq):
            kh = h // g
            s = (K[b, kh] @ q[b, h]) * sc
            mx = s[m].max() if m.any() else 0.0
            p = np.where(m, np.exp(s - mx), 0.0)
            l = p.sum()
            acc += (p / l) * (np.abs(V[b, kh]).sum(axis=1) / D)
        loss = rnd(acc / Hq, dt)
        res[b] = int(np.argmin(loss))
    return res


# ---------------------------------------------------------------------------
# eviction scores and keep selection
# ---------------------------------------------------------------------------
def gqa_mean(q, Hk: int, dt: str):
    """Query heads -> KV heads by averaging each GQA group, rounded to `dt`
    (cache.py:60-66, scoring.py:17-26). q (Hq,T,D) -> (Hk,T,D)."""
    q = np.asarray(q, np.float64)
    Hq, T, D = q.shape
    if Hq == Hk:
        return q
    if Hq % Hk == 0:
        return rnd(q.reshape(Hk, Hq // Hk, T, D).mean(axis=1), dt)
    return np.broadcast_to(rnd(q.mean(axis=0, keepdims=True), dt), (Hk, T, D))


def hotcold_token_scores(q_obs, K, dt: str):
    """Hot/cold policy score (cache.py:55-69): GQA-mean query rows . K^T / sqrt(D),
    summed over the query rows, averaged over KV heads. q_obs (Hq,tq,D), K (Hk,S,D)
    -> (S,) float64."""
    K = np.asarray(K, np.float64)
    Hk, S, D = K.shape
    qb = gqa_mean(q_obs, Hk, dt)
    logits = np.einsum("htd,hsd->hts", qb, K) / math.sqrt(D)
    return logits.sum(axis=1).mean(axis=0)


def pool1d(x, kernel: int, pooling: str):
    """Stride-1 1-D pooling over the last axis with padding kernel//2
    (scoring.py:40-47: F.max_pool1d pads with -inf, F.avg_pool1d counts the zero
    padding in the mean)."""
    if kernel is None or kernel <= 1:
        return x
    pad = kernel // 2
    L = x.shape[-1]
    fill = -np.inf if pooling == "maxpool" else 0.0
    xp = np.concatenate([np.full(x.shape[:-1] + (pad,), fill), x, np.full(x.shape[:-1] + (pad,), fill)], axis=-1)
    win = np.stack([xp[..., i:i + L] for i in range(kernel)], axis=0)
    return win.max(axis=0) if pooling == "maxpool" else win.sum(axis=0) / kernel


def snapkv_token_scores(q_obs, K, scale: float, pool_kernel: int, pooling: str, dt: str):
    """SnapKV importance (scoring.py:50-79) reduced to one score per token by a mean
    over KV heads. The observation rows are the last tq tokens of the sequence;
    row r (position S-tq+r) is causally masked. q_obs (Hq,tq,D), K (Hk,S,D)."""
    K = np.asarray(K, np.float64)
    Hk, S, D = K.shape
    qb = gqa_mean(q_obs, Hk, dt)
    tq = qb.shape[1]
    logits = np.einsum("htd,hsd->hts", qb, K) * float(np.float32(scale))
    qpos = np.arange(S - tq, S)[:, None]
    kpos = np.arange(S)[None, :]
    logits = np.where(kpos > qpos, -np.inf, logits)
    mx = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - mx)
    probs = e / e.sum(axis=-1, keepdims=True)
    imp = pool1d(probs.sum(axis=1), pool_kernel, pooling)
    return imp.mean(axis=0)


def topk_lower_index(scores, k: int) -> np.ndarray:
    """Indices of the k largest scores; equal scores prefer the lower index.
    Returned ascending."""
    scores = np.asarray(scores, np.float64)
    order = np.lexsort((np.arange(scores.shape[0]), -scores))
    return np.sort(order[:k])


def boundary_gap(scores, k: int) -> float:
    """Relative gap between the k-th and (k+1)-th largest scores (inf if k==len)."""
    s = np.sort(np.asarray(scores, np.float64))[::-1]
    if k <= 0 or k >= s.shape[0]:
        return math.inf
    a, b = s[k - 1], s[k]
    den = max(abs(a), abs(b), 1e-300)
    return (a - b) / den


@dataclass
class Policy:
    """Eviction policy knobs. policy='hotcold' is cache.py:37-128;
    policy='snapkv' scores with scoring.py:50-79 and keeps with scoring.py:110-132."""
    policy: str = "hotcold"
    cap: int = 128            # max_capacity_prompt (the budget)
    recent: int = 32          # recent_size (snapkv: window)
    topk_ratio: float = 0.15
    pool_kernel: int = 7
    pooling: str = "maxpool"


def plan_keep(pol: Policy, S: int):
    """(prefix_len, n_top, n_obs) for a hot cache of S tokens, or None if no
    compression. n_obs caps the number of observation query rows used.
    hotcold: cache.py:44-57. snapkv: scoring.py:65,117-120 with trigger cache.py:44."""
    if S <= pol.cap:
        return None
    if pol.policy == "hotcold":
        recent = min(pol.recent, pol.cap, S)
        prefix_len = S - recent
        if prefix_len <= 0:
            return None
        n_top = max(1, min(int(pol.cap * pol.topk_ratio), prefix_len))
        return prefix_len, n_top, recent
    window = min(pol.recent, S)
    prefix_len = S - window
    n_top = max(0, min(pol.cap - window, prefix_len))
    return prefix_len, n_top, window


def token_scores(pol: Policy, q_obs, K, scale: float, dt: str):
    if pol.policy == "hotcold":
        return hotcold_token_scores(q_obs, K, dt)
    return snapkv_token_scores(q_obs, K, scale, pol.pool_kernel, pol.pooling, dt)


# ---------------------------------------------------------------------------
# cold store vectors  (controller.py:166-188)
# ---------------------------------------------------------------------------
def pad_or_crop(x, dim: int):
    x = np.asarray(x, np.float64)
    if x.shape[-1] > dim:
        return x[..., :dim]
    if x.shape[-1] < dim:
        return np.concatenate([x, np.zeros(x.shape[:-1] + (dim - x.shape[-1],))], axis=-1)
    return x


def key_index_vector(kpre_tok, faiss_dim: int, normalize: bool):
    """controller.py:178-182: mean over KV heads of the fp32 pre-RoPE key, pad/crop
    to faiss_dim, L2-normalise (F.normalize, eps 1e-12). kpre_tok (Hk,D)."""
    v = pad_or_crop(np.asarray(kpre_tok, np.float64).mean(axis=0), faiss_dim)
    if normalize:
        v = v / max(np.linalg.norm(v), 1e-12)
    return v.astype(np.float32).astype(np.float64)


def query_vector(q_rows, faiss_dim: int, normalize: bool, dt: str):
    """controller.py:184-188 in the model dtype: mean over heads (rounded), mean
    over pooled positions (rounded), pad/crop, F.normalize in the dtype (norm
    rounded, eps 1e-12 clamped in the dtype), then float32.
    q_rows (Hq, P, D) -> (faiss_dim,)."""
    q = np.asarray(q_rows, np.float64)
    m1 = rnd(q.mean(axis=0), dt)            # (P, D)
    m2 = rnd(m1.mean(axis=0), dt)           # (D,)
    x = pad_or_crop(m2, faiss_dim)
    if normalize:
        n = rnd(np.sqrt((x * x).sum()), dt)
        eps = float(rnd(1e-12, dt))
        x = rnd(x / max(n, eps), dt) if max(n, eps) > 0 else x / 0.0
    return x.astype(np.float32).astype(np.float64)


@dataclass
class ColdRing:
    """One (layer, sequence) cold store: a ring of `cap` tokens and the flat
    inner-product index over them, kept row-aligned (controller.py:190-238)."""
    cap: int
    kpre: deque = field(default_factory=deque)
    v: deque = field(default_factory=deque)
    pos: deque = field(default_factory=deque)
    vec: deque = field(default_factory=deque)

    def __len__(self):
        return len(self.pos)

    def add(self, kpre_list, v_list, pos_list, faiss_dim, normalize):
        for kp, vv, p in zip(kpre_list, v_list, pos_list):
            self.kpre.append(np.asarray(kp, np.float64))
            self.v.append(np.asarray(vv, np.float64))
            self.pos.append(int(p))
            self.vec.append(key_index_vector(kp, faiss_dim, normalize))
            while len(self.pos) > self.cap:
                self.kpre.popleft(); self.v.popleft(); self.pos.popleft(); self.vec.popleft()
        return min(len(pos_list), self.cap)

    def search(self, qvec, k: int):
        """Exact inner-product top-k (faiss IndexFlatIP.search, controller.py:274);
        ties prefer the lower ring slot. Returns (ids, scores) of min(k, n) hits."""
        n = len(self.pos)
        if n == 0:
            return np.zeros(0, np.int64), np.zeros(0)
        X = np.stack(list(self.vec), axis=0)
        sc = X @ np.asarray(qvec, np.float64)
        order = np.lexsort((np.arange(n), -sc))[: min(k, n)]
        return order.astype(np.int64), sc[order]


# ---------------------------------------------------------------------------
# one attention layer of the patched forward, deterministic retrieval schedule
# ---------------------------------------------------------------------------
DBG_KEYS = ("compress_calls", "evicted_tokens", "faiss_add", "retrieval_launched",
            "retrieval_launched_prefill", "retrieval_ready_cpu", "retrieval_skipped_no_cold",
            "retrieval_ready_empty", "prefetch_launched", "prefetch_ready", "prefetch_skipped_empty",
            "injection_used", "injection_new", "injection_skipped_no_valid",
            "triton_prefill_fallback")


class OracleLayer:
    """One decoder layer of the hot/cold path for B equal-length sequences.

    Follows patch.py:122-348 (the patched LlamaAttention.forward) with the
    hot tier of cache.py:37-151 and the cold tier of controller.py:190-442, with
    the retrieval worker run synchronously and its result staged at once, so a
    retrieval launched at step t is attended at step t (the rule the CUDA path
    implements). With retrieval_lag=1 a decode-step retrieval instead searches the
    cold store after step t's compression and is attended from step t+1: one of
    the orders the reference's asynchronous worker (controller.py:314-342) can
    take, the one the CUDA path's async_retrieval mode implements. Positions of
    prompt tokens are 0..T-1.
    """

    def __init__(self, *, Hq, Hk, D, dtype, inv_freq, attention_scaling=1.0,
                 policy: Policy, cpu_buffer_size=8192, faiss_dim=64, normalize_for_ip=True,
                 window_size=16, query_pool_size=4, lookahead_k=32, hold_retrieved=False,
                 retrieve_after_prefill=False, retrieval_lag=0):
        self.Hq, self.Hk, self.D, self.dt = Hq, Hk, D, dtype
        self.inv_freq = np.asarray(inv_freq, np.float32)
        self.att_scale = float(attention_scaling)
        self.pol = policy
        self.ccap = int(cpu_buffer_size)
        self.faiss_dim = int(faiss_dim)
        self.normalize = bool(normalize_for_ip)
        self.window_size = int(window_size)
        self.query_pool_size = int(query_pool_size)
        self.lookahead_k = int(lookahead_k)
        self.hold = bool(hold_retrieved)
        self.retrieve_after_prefill = bool(retrieve_after_prefill)
        if retrieval_lag not in (0, 1):
            raise ValueError("retrieval_lag is 0 or 1")
        self.retrieval_lag = int(retrieval_lag)
        self.scale = 1.0 / math.sqrt(D)
        self.dbg = {k: 0 for k in DBG_KEYS}
        self.step_count = 0
        self.qwin: deque = deque(maxlen=self.query_pool_size)   # entries (B,Hq,T,D)
        self.staged = None
        self.held = None
        self.B = None
        # records for tests
        self.events = []          # dicts per retrieval: step, ids, pos, valid, kmem
        self.compress_log = []    # dicts per compression: step, S, keep, evicted, gap
        # optional test hooks that may replace a selection of this restatement by another one
        # that differs only at a near-tie of its boundary (a parity test adopts the selection
        # of the implementation under test there and goes on comparing):
        #   resolve_keep(step, b, scores, prefix_len, n_top, top, P_b) -> top indices to keep
        #   resolve_hits(step, b, scores, ids, ring_pos) -> ring ids of the hits, best first
        self.resolve_keep = None
        self.resolve_hits = None

    # -- hot tier ------------------------------------------------------------
    def _compress(self, q_obs, step):
        """cache.py:37-128 (policy hotcold) / scoring composition (policy snapkv)."""
        B, Hk, S, D = self.K.shape
        plan = plan_keep(self.pol, S)
        if plan is None:
            return
        prefix_len, n_top, n_obs = plan
        q_obs = q_obs[:, :, -min(n_obs, q_obs.shape[2]):]
        keep_all, ev_all = [], []
        for b in range(B):
            sc = token_scores(self.pol, q_obs[b], self.K[b], self.scale, self.dt)
            top = topk_lower_index(sc[:prefix_len], n_top) if n_top > 0 else np.zeros(0, np.int64)
            if self.resolve_keep is not None:
                top = np.sort(np.asarray(self.resolve_keep(step, b, sc[:prefix_len], prefix_len, n_top, top,
                                                           self.P[b]), np.int64))
            keep = np.concatenate([top, np.arange(prefix_len, S)])
            ev = np.setdiff1d(np.arange(prefix_len), top)
            keep_all.append(keep)
            ev_all.append(ev)
            self.compress_log.append(dict(step=step, b=b, S=S, prefix_len=prefix_len, n_top=n_top,
                                          gap=boundary_gap(sc[:prefix_len], n_top),
                                          keep_pos=self.P[b, keep].copy(),
                                          evict_pos=self.P[b, ev].copy()))
        te_max = max(len(e) for e in ev_all)
        if te_max > 0:
            self.dbg["compress_calls"] += 1
            self.dbg["evicted_tokens"] += int(sum(len(e) for e in ev_all))
            for b in range(B):
                e = ev_all[b]
                if len(e) == 0:
                    continue
                self.dbg["faiss_add"] += self.cold[b].add(
                    [self.Kpre[b, :, t] for t in e], [self.V[b, :, t] for t in e],
                    [self.P[b, t] for t in e], self.faiss_dim, self.normalize)
        keep = np.stack(keep_all, axis=0)
        self.K = np.stack([self.K[b][:, keep[b]] for b in range(B)], 0)
        self.V = np.stack([self.V[b][:, keep[b]] for b in range(B)], 0)
        self.Kpre = np.stack([self.Kpre[b][:, keep[b]] for b in range(B)], 0)
        self.P = np.stack([self.P[b, keep[b]] for b in range(B)], 0)

    # -- cold tier -----------------------------------------------------------
    def cold_size(self):
        return 0 if self.B is None else sum(len(c) for c in self.cold)

    def _retrieve(self, q_rows_per_b, step):
        """controller.py:250-293 run synchronously, then staged (controller.py:344-380)."""
        B, Hk, D, R = self.B, self.Hk, self.D, self.lookahead_k
        kpre = np.zeros((B, Hk, R, D)); v = np.zeros((B, Hk, R, D))
        pos = np.zeros((B, R), np.int64); valid = np.zeros((B, R), bool)
        ids_all = []
        for b in range(B):
            n = len(self.cold[b])
            if n == 0:
                ids_all.append(np.zeros(0, np.int64))
                continue
            qv = query_vector(q_rows_per_b[b], self.faiss_dim, self.normalize, self.dt)
            ids, _ = self.cold[b].search(qv, R)
            if self.resolve_hits is not None:
                X = np.stack(list(self.cold[b].vec), axis=0)
                ids = np.asarray(self.resolve_hits(step, b, X @ np.asarray(qv, np.float64), ids,
                                                   np.asarray(self.cold[b].pos, np.int64)), np.int64)
            ids_all.append(ids)
            for j, i in enumerate(ids):
                kpre[b, :, j] = self.cold[b].kpre[i]
                v[b, :, j] = self.cold[b].v[i]
                pos[b, j] = self.cold[b].pos[i]
                valid[b, j] = True
        if not valid.any():
            self.dbg["retrieval_ready_empty"] += 1
            return
        self.dbg["retrieval_ready_cpu"] += 1
        # staging converts the fp32 pinned pack back to the model dtype (exact)
        self.staged = (rnd(kpre, self.dt), rnd(v, self.dt), pos, valid, step, ids_all)
        self.dbg["prefetch_launched"] += 1

    def _pooled_rows(self):
        """Query rows of every pooled entry, concatenated over positions (controller.py:243-248)."""
        return np.concatenate(list(self.qwin), axis=2)  # (B,Hq,P,D)

    # -- forward -------------------------------------------------------------
    def prefill(self, q_pre, k_pre, v):
        """Prompt forward (q_len = T > 1) on an empty cache: patch.py:151-233.
        Prompt attention itself is stock SDPA and not modelled."""
        q_pre = np.asarray(q_pre, np.float64)
        k_pre = np.asarray(k_pre, np.float64)
        v = np.asarray(v, np.float64)
        B, Hq, T, D = q_pre.shape
        self.B = B
        self.cold = [ColdRing(self.ccap) for _ in range(B)]
        pos = np.arange(T, dtype=np.int64)
        cos, sin = rope_cos_sin(pos, self.inv_freq, self.att_scale, self.dt)
        q_post = apply_rope(q_pre, cos, sin, self.dt)
        k_post = apply_rope(k_pre, cos, sin, self.dt)
        if self.query_pool_size >= self.window_size:
            self.qwin.append(q_pre)
        if self.lookahead_k > 0:
            self.step_count += 1   # a prefill forward counts as a step (controller.py:318)
            # a launch at step 1 needs window_size == 1; the cold tier is still empty then
            if self.step_count % self.window_size == 0:
                self.dbg["retrieval_skipped_no_cold"] += 1
        self.K, self.V, self.Kpre = k_post, v, k_pre
        self.P = np.broadcast_to(pos, (B, T)).copy()
        r = self.pol.recent
        q_obs = q_post if T <= r else q_post[:, :, -r:]
        self._compress(q_obs, step=0)
        self.dbg["triton_prefill_fallback"] += 1
        if self.retrieve_after_prefill and self.lookahead_k > 0:
            if self.cold_size() == 0:
                self.dbg["retrieval_skipped_no_cold"] += 1
            else:
                self._retrieve(q_pre[:, :, -self.query_pool_size:], step=0)
                self.dbg["retrieval_launched"] += 1
                self.dbg["retrieval_launched_prefill"] += 1

    def prefill_chunks(self, q_pre, k_pre, v, bounds):
        """A prompt forwarded in chunks [bounds[i], bounds[i+1]) (the reference rejects chunked
        prefill, patch.py:325-329; this is the semantics the CUDA path implements): each
        chunk's tokens join the hot tier after the ones already kept, and when the hot tier
        exceeds the budget it is compressed (cache.py:37-128 / the SnapKV composition) with the
        last recent_size post-RoPE queries of that chunk as the observation window. The whole
        prompt counts as one forward for the retrieval schedule; the prompt-end retrieval uses
        the last query_pool_size queries of the prompt. Needs query_pool_size < window_size
        (prompt queries stay out of the query pool). One chunk equals prefill()."""
        assert self.query_pool_size < self.window_size
        q_pre = np.asarray(q_pre, np.float64)
        k_pre = np.asarray(k_pre, np.float64)
        v = np.asarray(v, np.float64)
        B, Hq, T, D = q_pre.shape
        self.B = B
        self.cold = [ColdRing(self.ccap) for _ in range(B)]
        if self.lookahead_k > 0:
            self.step_count += 1
            if self.step_count % self.window_size == 0:
                self.dbg["retrieval_skipped_no_cold"] += 1
        r = self.pol.recent
        for ci, (c0, c1) in enumerate(zip(bounds[:-1], bounds[1:])):
            self.chunk_index = ci
            pos = np.arange(c0, c1, dtype=np.int64)
            cos, sin = rope_cos_sin(pos, self.inv_freq, self.att_scale, self.dt)
            q_post = apply_rope(q_pre[:, :, c0:c1], cos, sin, self.dt)
            k_post = apply_rope(k_pre[:, :, c0:c1], cos, sin, self.dt)
            if c0 == 0:
                self.K, self.V, self.Kpre = k_post, v[:, :, c0:c1], k_pre[:, :, c0:c1]
                self.P = np.broadcast_to(pos, (B, c1 - c0)).copy()
            else:
                self.K = np.concatenate([self.K, k_post], 2)
                self.V = np.concatenate([self.V, v[:, :, c0:c1]], 2)
                self.Kpre = np.concatenate([self.Kpre, k_pre[:, :, c0:c1]], 2)
                self.P = np.concatenate([self.P, np.broadcast_to(pos, (B, c1 - c0))], 1)
            q_obs = q_post if c1 - c0 <= r else q_post[:, :, -r:]
            self._compress(q_obs, step=0)
            self.dbg["triton_prefill_fallback"] += 1
        if self.retrieve_after_prefill and self.lookahead_k > 0:
            if self.cold_size() == 0:
                self.dbg["retrieval_skipped_no_cold"] += 1
            else:
                self._retrieve(q_pre[:, :, -self.query_pool_size:], step=0)
                self.dbg["retrieval_launched"] += 1
                self.dbg["retrieval_launched_prefill"] += 1

    def decode(self, q_pre, k_pre, v, step):
        """One decode step (q_len = 1): patch.py:151-315. q_pre (B,Hq,D),
        k_pre/v (B,Hk,D). `step` is 1-based; the position is T-1+step.
        Returns the attention output (B,Hq,D) in the model dtype."""
        q_pre = np.asarray(q_pre, np.float64)[:, :, None, :]
        k_pre = np.asarray(k_pre, np.float64)[:, :, None, :]
        v = np.asarray(v, np.float64)[:, :, None, :]
        B = self.B
        cur = self._next_pos
        cos, sin = rope_cos_sin(np.array([cur]), self.inv_freq, self.att_scale, self.dt)
        q_post = apply_rope(q_pre, cos, sin, self.dt)
        k_post = apply_rope(k_pre, cos, sin, self.dt)
        self.qwin.append(q_pre)
        deferred = False
        if self.lookahead_k > 0:
            self.step_count += 1
            if self.step_count % self.window_size == 0:
                if self.cold_size() == 0:
                    self.dbg["retrieval_skipped_no_cold"] += 1
                elif len(self.qwin):
                    if self.retrieval_lag:
                        deferred = True  # searched after this step's compression, attended next step
                    else:
                        self._retrieve(self._pooled_rows(), step=step)
                    self.dbg["retrieval_launched"] += 1
        # hot update (append then compress)
        self.K = np.concatenate([self.K, k_post], axis=2)
        self.V = np.concatenate([self.V, v], axis=2)
        self.Kpre = np.concatenate([self.Kpre, k_pre], axis=2)
        self.P = np.concatenate([self.P, np.full((B, 1), cur, np.int64)], axis=1)
        self._compress(q_post, step=step)
        # poll / inject
        mem = None
        if self.staged is not None:
            kpre_r, v_r, pos_r, valid_r, lstep, ids = self.staged
            self.staged = None
            self.dbg["prefetch_ready"] += 1
            cs, sn = rope_cos_sin(pos_r.reshape(-1), self.inv_freq, self.att_scale, self.dt)
            R = pos_r.shape[1]
            cs = cs.reshape(B, 1, R, self.D)
            sn = sn.reshape(B, 1, R, self.D)
            kmem = apply_rope(kpre_r, cs, sn, self.dt)
            mem = (kmem, v_r, pos_r, valid_r)
            self.events.append(dict(step=step, launched=lstep, ids=ids, pos=pos_r.copy(),
                                    valid=valid_r.copy(), kmem=kmem.copy()))
            if self.hold:
                self.held = mem
                self.dbg["injection_new"] += 1
        elif self.hold:
            mem = self.held
        Kc, Vc = self.K, self.V
        mask = np.ones((B, Kc.shape[2]), bool)
        if mem is not None:
            self.dbg["injection_used"] += 1
            keep_mem = mem[3] & (mem[2] <= cur)
            Kc = np.concatenate([mem[0], Kc], axis=2)
            Vc = np.concatenate([mem[1], Vc], axis=2)
            mask = np.concatenate([keep_mem, mask], axis=1)
        self._next_pos = cur + 1
        out = decode_attention(q_post[:, :, 0], Kc, Vc, mask, self.scale, self.dt)
        if deferred:
            self._retrieve(self._pooled_rows(), step=step + 1)
        return out

    def start_decode(self, T: int):
        self._next_pos = T

    # -- convenience ---------------------------------------------------------
    def hot_positions(self):
        return self.P.copy()

    def cold_positions(self):
        return [np.array(list(c.pos), np.int64) for c in self.cold]


def run_layer(inputs: dict, n_steps: int, chunks=None, follow=None, **kw):
    """Drive OracleLayer over `inputs` (synth.layer_inputs layout), the prompt whole or in
    chunks with the given boundaries. `follow`, a test object with attach(layer), installs
    the resolve_keep / resolve_hits hooks. Returns (layer, outs (n,B,Hq,D), hot_pos list per
    step)."""
    layer = OracleLayer(**kw)
    if follow is not None:
        follow.attach(layer)
    if chunks is None:
        layer.prefill(inputs["q_pre"], inputs["k_pre"], inputs["v"])
    else:
        layer.prefill_chunks(inputs["q_pre"], inputs["k_pre"], inputs["v"], chunks)
    T = inputs["q_pre"].shape[2]
    layer.start_decode(T)
    outs, hot = [], []
    for i in range(n_steps):
        outs.append(layer.decode(inputs["dq"][i], inputs["dk"][i], inputs["dv"][i], step=i + 1))
        hot.append(layer.hot_positions())
    return layer, np.stack(outs, 0), hot
