"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference sources (tarun931/hotcold-kv-cache);
HOTCOLD_REFERENCE_SRC must name their `src` directory (the one holding the
`hotcold_kv` package):

    HOTCOLD_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden.py [case ...]

It imports the reference's own modules and drives them on CPU with these shims
(none of them edits the reference; all live in this file):

 1. `faiss` is not installed: a stand-in module gives `IndexFlatIP(d)` (exact
    float32 inner product, search sorted by score with ties to the lower id),
    `add`, `search`, `remove_ids(IDSelectorRange)` and `ntotal`.
 2. Pinned host memory needs a CUDA driver: `pin_memory=True` is dropped
    (as tests/test_cold_store.py:33-36 of the reference does).
 3. transformers 5.x passes an int to `get_mask_sizes` (the reference was written
    for 4.57, cache.py:153-156): the int is accepted.
 4. The retrieval thread (controller.py:336-341) runs synchronously on start().
 5. Prefetch/poll (controller.py:344-442) stage the pack on CPU instead of a CUDA
    stream, converting to the model dtype exactly as the GPU path does, so the
    result is attended at the same forward (the reference on CPU never attends
    retrieved tokens: poll_staged_gpu returns ready=False without CUDA).

The snapkv-policy cases replace HotColdLayer._compress_if_needed with a
composition of the reference's own SnapKV functions (scoring.snapkv_importance,
scoring.keep_index): the per-KV-head importance is averaged over heads into one
token score, and the rest of the hot/cold eviction flow (cache.py:78-128) is
unchanged.

The single-layer cases call the patched LlamaAttention.forward with a stub
module whose projections return seeded synthetic pre-RoPE tensors
(hotcold_kv_cache_b200.synth.layer_inputs) and whose o_proj is the identity.
Seeds are chosen so that every top-k boundary of every compression and
retrieval has a relative score gap above GAP_MIN, which keeps multi-step
comparisons exact.
"""

from __future__ import annotations

import json
import math
import os
import sys
import threading
import types

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
REF_SRC = os.environ.get("HOTCOLD_REFERENCE_SRC")
if not REF_SRC or not os.path.isdir(os.path.join(REF_SRC, "hotcold_kv")):
    raise SystemExit("set HOTCOLD_REFERENCE_SRC to the reference's src directory (it holds hotcold_kv/)")

from hotcold_kv_cache_b200 import synth  # noqa: E402

# minimum relative gap at every top-k boundary: compression selections (scored in the
# model dtype by the reference) and cold searches (float32 inner products)
GAP_MIN = {"float32": 2e-4, "float16": 2e-3, "bfloat16": 2e-2}
SEARCH_GAP_MIN = 2e-4


# --------------------------------------------------------------------------- shim 1
class _IDSelectorRange:
    def __init__(self, lo, hi):
        self.lo, self.hi = int(lo), int(hi)


class _IndexFlatIP:
    def __init__(self, d):
        self.d = int(d)
        self._x = np.zeros((0, self.d), np.float32)

    @property
    def ntotal(self):
        return int(self._x.shape[0])

    def add(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.d)
        self._x = np.concatenate([self._x, x], axis=0)

    def remove_ids(self, sel):
        keep = np.ones(self.ntotal, bool)
        keep[sel.lo:sel.hi] = False
        n = int((~keep).sum())
        self._x = self._x[keep]
        return n

    def search(self, q, k):
        q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1, self.d)
        sc = (q.astype(np.float64) @ self._x.astype(np.float64).T).astype(np.float32)
        D = np.full((q.shape[0], k), -np.inf, np.float32)
        I = np.full((q.shape[0], k), -1, np.int64)
        for r in range(q.shape[0]):
            order = np.lexsort((np.arange(self.ntotal), -sc[r].astype(np.float64)))[:k]
            D[r, :len(order)] = sc[r, order]
            I[r, :len(order)] = order
            RECORD["search_gaps"].append(_gap(sc[r].astype(np.float64), min(k, self.ntotal)))
        return D, I


faiss_mod = types.ModuleType("faiss")
faiss_mod.Index = _IndexFlatIP
faiss_mod.IndexFlatIP = _IndexFlatIP
faiss_mod.IDSelectorRange = _IDSelectorRange
sys.modules["faiss"] = faiss_mod

# --------------------------------------------------------------------------- shim 2
if not torch.cuda.is_available():
    _zeros, _empty = torch.zeros, torch.empty
    torch.zeros = lambda *a, **k: _zeros(*a, **{x: y for x, y in k.items() if x != "pin_memory"})
    torch.empty = lambda *a, **k: _empty(*a, **{x: y for x, y in k.items() if x != "pin_memory"})

# record top-k boundaries (compression selection) to check score gaps
RECORD = {"topk_gaps": [], "search_gaps": []}
_topk = torch.topk


def _gap(scores: np.ndarray, k: int) -> float:
    s = np.sort(scores)[::-1]
    if k <= 0 or k >= s.shape[0]:
        return math.inf
    a, b = s[k - 1], s[k]
    return float((a - b) / max(abs(a), abs(b), 1e-300))


def _topk_rec(x, k, *a, **kw):
    xs = x.detach().double().reshape(-1, x.shape[-1]).numpy()
    for row in xs:
        RECORD["topk_gaps"].append(_gap(row, int(k)))
    return _topk(x, k, *a, **kw)


torch.topk = _topk_rec

sys.path.insert(0, REF_SRC)
import hotcold_kv  # noqa: E402
from hotcold_kv import controller as ref_ctrl  # noqa: E402
from hotcold_kv import cache as ref_cache  # noqa: E402
from hotcold_kv import patch as ref_patch  # noqa: E402
from hotcold_kv import kernels as ref_kernels  # noqa: E402
from hotcold_kv.datatypes import EvictedKV, RetrievedKV, _canon_br_2d, _canon_kv_4d  # noqa: E402
from hotcold_kv.baselines import scoring as ref_scoring  # noqa: E402
from transformers import LlamaConfig, LlamaForCausalLM  # noqa: E402
from transformers.cache_utils import Cache  # noqa: E402
from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding  # noqa: E402


# --------------------------------------------------------------------------- shim 3
def _get_mask_sizes(self, cache_position):
    q = cache_position if isinstance(cache_position, int) else int(cache_position.shape[0])
    return int(self.get_seq_length() + q), 0


ref_cache.HotColdLayer.get_mask_sizes = _get_mask_sizes


# --------------------------------------------------------------------------- shim 4
class _SyncThread:
    def __init__(self, target=None, args=(), kwargs=None, daemon=None):
        self._t, self._a, self._k = target, args, kwargs or {}

    def start(self):
        self._t(*self._a, **self._k)

    def is_alive(self):
        return False


# start() runs the worker while maybe_launch_async_retrieval holds _retrieval_lock
# (controller.py:332-341), so the shim hands out reentrant locks.
ref_ctrl.threading = types.SimpleNamespace(Thread=_SyncThread, Lock=threading.RLock, RLock=threading.RLock)


# --------------------------------------------------------------------------- shim 5
def _prefetch_cpu(self, layer_idx, device, dtype):
    li = int(layer_idx)
    with self._retrieval_lock[li]:
        pack = self._retrieval_ready_cpu[li]
        self._retrieval_ready_cpu[li] = None
    if pack is None:
        return
    kpre_cpu, v_cpu, pos_cpu, valid_cpu = pack
    if not bool(valid_cpu.any().item()):
        self.dbg["prefetch_skipped_empty"] += 1
        return
    staged = (kpre_cpu.to(dtype=dtype), v_cpu.to(dtype=dtype), pos_cpu.clone(), valid_cpu.clone())
    with self._stage_lock[li]:
        self._staged_gpu[li] = staged
        self._staged_event[li] = True
        self.dbg["prefetch_launched"] += 1


def _poll_cpu(self, layer_idx):
    li = int(layer_idx)
    empty = RetrievedKV(k_pre=torch.empty(0), v=torch.empty(0), pos=torch.empty(0, dtype=torch.long),
                        valid=torch.empty(0, dtype=torch.bool), ready=False)
    with self._stage_lock[li]:
        if self._staged_gpu[li] is None or self._staged_event[li] is None:
            return empty
        kpre, v, pos, valid = self._staged_gpu[li]
        self._staged_gpu[li] = None
        self._staged_event[li] = None
        self.dbg["prefetch_ready"] += 1
    if kpre.numel() == 0:
        return RetrievedKV(k_pre=kpre, v=v, pos=pos, valid=valid, ready=False)
    kpre = _canon_kv_4d(kpre, "staged.k_pre")
    v = _canon_kv_4d(v, "staged.v")
    pos = _canon_br_2d(pos, "staged.pos")
    valid = _canon_br_2d(valid, "staged.valid")
    RECORD["retrieved"].append(dict(pos=pos.numpy().copy(), valid=valid.numpy().copy()))
    if not bool(valid.any().item()):
        return RetrievedKV(k_pre=kpre, v=v, pos=pos, valid=valid, ready=False)
    return RetrievedKV(k_pre=kpre, v=v, pos=pos, valid=valid, ready=True)


ref_ctrl.KVController.maybe_prefetch_to_gpu = _prefetch_cpu
ref_ctrl.KVController.poll_staged_gpu = _poll_cpu

_rotate_orig = ref_patch._rotate_k_with_pos


def _rotate_rec(k_pre, pos_ids, head_dim):
    out = _rotate_orig(k_pre, pos_ids, head_dim)
    RECORD["kmem"].append(out.detach().float().numpy().copy())
    return out


ref_patch._rotate_k_with_pos = _rotate_rec


# --------------------------------------------------------------------------- snapkv policy
def _compress_snapkv_factory(pool_kernel, pooling):
    def _compress(self, layer_idx):
        """cache.py:37-128 with the score and keep set of scoring.py:50-79,110-132."""
        if self._last_q_post is None or self.keys is None:
            return
        B, Hk, S, D = self.keys.shape
        cap = self.kvctrl.max_capacity_prompt
        if S <= cap:
            return
        window = min(self.kvctrl.recent_size, S)
        prefix_len = S - window
        q = self._last_q_post
        tq = min(window, q.shape[2])
        q_full = torch.zeros(B, q.shape[1], S, D, dtype=q.dtype)
        q_full[:, :, S - tq:] = q[:, :, -tq:]
        imp = ref_scoring.snapkv_importance(q_full, self.keys, tq, 1.0 / math.sqrt(D), pool_kernel, pooling)
        token = imp.mean(dim=1, keepdim=True)
        keep_idx = ref_scoring.keep_index(token, window, cap)[:, 0]
        RECORD.setdefault("snap", []).append((token[:, 0].float().numpy().copy(), keep_idx.numpy().copy()))
        keep_len = keep_idx.shape[1]
        idx_k = keep_idx.unsqueeze(1).unsqueeze(-1).expand(B, Hk, keep_len, D)
        keys_new = self.keys.gather(2, idx_k)
        values_new = self.values.gather(2, idx_k)
        pre_new = self.pre_keys.gather(2, idx_k)
        pos_new = self.positions.gather(1, keep_idx)
        mask = torch.ones((B, prefix_len), dtype=torch.bool)
        top = keep_idx[:, : keep_len - window]
        if top.shape[1]:
            mask.scatter_(1, top, False)
        ev = [torch.nonzero(mask[b]).squeeze(-1) for b in range(B)]
        te_max = max(int(t.numel()) for t in ev)
        if te_max > 0:
            kp = torch.empty((B, Hk, te_max, D), dtype=torch.float32)
            vv = torch.empty((B, Hk, te_max, D), dtype=torch.float32)
            pp = torch.empty((B, te_max), dtype=torch.long)
            ii = torch.full((B, te_max), -1, dtype=torch.long)
            for b in range(B):
                t = ev[b]
                te = int(t.numel())
                if te == 0:
                    continue
                ii[b, :te] = t
                kp[b, :, :te] = self.pre_keys[b, :, t].float()
                vv[b, :, :te] = self.values[b, :, t].float()
                pp[b, :te] = self.positions[b, t]
            self.kvctrl.dbg["compress_calls"] += 1
            self.kvctrl.dbg["evicted_tokens"] += int((ii >= 0).sum().item())
            self.kvctrl.add_evicted_to_cold_store(layer_idx, EvictedKV(kp, vv, pp, ii))
        self.keys, self.values, self.pre_keys, self.positions = keys_new, values_new, pre_new, pos_new
    return _compress


_COMPRESS_HOTCOLD = ref_cache.HotColdLayer._compress_if_needed


# --------------------------------------------------------------------------- drivers
TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


class _Stub:
    """Stands in for a LlamaAttention module: projections return given tensors."""

    def __init__(self, Hq, Hk, D, layer_idx=0, n_layers=1):
        self.config = types.SimpleNamespace(num_attention_heads=Hq, num_key_value_heads=Hk,
                                            num_hidden_layers=n_layers, hidden_size=Hq * D)
        self.head_dim = D
        self.layer_idx = layer_idx
        self._q = self._k = self._v = None
        self.q_proj = lambda h: self._q
        self.k_proj = lambda h: self._k
        self.v_proj = lambda h: self._v
        self.o_proj = lambda x: x


def run_single_layer(case: dict, seed: int):
    """Drive the reference's patched forward for one layer. Returns arrays."""
    for k in RECORD:
        RECORD[k] = []
    RECORD["retrieved"], RECORD["kmem"] = [], []
    c = case
    B, Hq, Hk, D, T, n = c["B"], c["Hq"], c["Hk"], c["D"], c["T"], c["steps"]
    dt = TORCH_DT[c["dtype"]]
    inp = synth.layer_inputs(seed, B, Hq, Hk, D, T, n, c["dtype"])
    inp = {k: torch.from_numpy(np.ascontiguousarray(v).astype(np.float32)).to(dt) for k, v in inp.items()}
    if c["policy"] == "snapkv":
        ref_cache.HotColdLayer._compress_if_needed = _compress_snapkv_factory(c["pool_kernel"], "maxpool")
    else:
        ref_cache.HotColdLayer._compress_if_needed = _COMPRESS_HOTCOLD
    kv = hotcold_kv.KVController(
        max_capacity_prompt=c["cap"], topk_ratio=c["topk_ratio"], recent_size=c["recent"],
        cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], normalize_for_ip=True,
        window_size=c["window_size"], query_pool_size=c["pool"], lookahead_k=c["R"],
        hold_retrieved=c["hold"], retrieve_after_prefill=c["rap"], enable_asserts=True,
        profile_overlap=False)
    hotcold_kv.uninstall_monkeypatch()
    hotcold_kv.install_monkeypatch(enable_debug=False)
    fwd = ref_patch.modeling_llama.LlamaAttention.forward
    lc = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hk, head_dim=D,
                     num_hidden_layers=1, rope_theta=c["theta"], vocab_size=16, intermediate_size=16,
                     max_position_embeddings=max(4096, T + n + 8))
    rot = LlamaRotaryEmbedding(lc)
    hotcold_kv.set_active_rotary_emb(rot)
    hotcold_kv.set_active_kvctrl(kv)
    layer = ref_cache.HotColdLayer(kv)
    cache = Cache(layers=[layer])
    stub = _Stub(Hq, Hk, D)

    def proj(x, H):  # (B,H,t,D) -> (B,t,H*D)
        return x.transpose(1, 2).reshape(B, x.shape[2], H * D)

    stub._q, stub._k, stub._v = proj(inp["q_pre"], Hq), proj(inp["k_pre"], Hk), proj(inp["v"], Hk)
    pos = torch.arange(T).unsqueeze(0).expand(B, T)
    cos, sin = rot(torch.empty(B, T, Hq * D, dtype=dt), pos)
    hs = torch.zeros(B, T, 1, dtype=dt)
    with torch.inference_mode():
        fwd(stub, hs, (cos, sin), None, past_key_values=cache, cache_position=torch.arange(T))
    outs, hot = [], []
    for i in range(n):
        p = T + i
        stub._q = inp["dq"][i][:, None].reshape(B, 1, Hq * D)
        stub._k = inp["dk"][i][:, None].reshape(B, 1, Hk * D)
        stub._v = inp["dv"][i][:, None].reshape(B, 1, Hk * D)
        posd = torch.full((B, 1), p, dtype=torch.long)
        cos, sin = rot(torch.empty(B, 1, Hq * D, dtype=dt), posd)
        with torch.inference_mode():
            o, _ = fwd(stub, torch.zeros(B, 1, 1, dtype=dt), (cos, sin), None, past_key_values=cache,
                       cache_position=torch.tensor([p]))
        outs.append(o.reshape(B, Hq, D).float().numpy())
        hot.append(layer.positions.numpy().copy())
    hotcold_kv.uninstall_monkeypatch()
    cold = [np.array(list(kv.cpu_pos_ring[0][b]), np.int64) for b in range(B)]
    res = dict(outs=np.stack(outs, 0), hot_len=np.array([h.shape[1] for h in hot], np.int32),
               hot_pos=np.concatenate([h.reshape(B, -1) for h in hot], axis=1).astype(np.int32),
               cold_pos=np.stack(cold, 0) if len({len(x) for x in cold}) == 1 else np.zeros(0),
               dbg=json.dumps({k: v for k, v in kv.dbg.items() if not k.startswith("prefetch_copy")}))
    if RECORD["retrieved"]:
        res["ret_pos"] = np.stack([r["pos"] for r in RECORD["retrieved"]], 0)
        res["ret_valid"] = np.stack([r["valid"] for r in RECORD["retrieved"]], 0)
        res["kmem0"] = RECORD["kmem"][0].astype(np.float32)
    return res, _min_gap(c["dtype"])


def _min_gap(dtype):
    """Smallest boundary gap as a multiple of its threshold (>= 1 passes)."""
    g = [x / GAP_MIN[dtype] for x in RECORD["topk_gaps"]] + [x / SEARCH_GAP_MIN for x in RECORD["search_gaps"]]
    return min(g) if g else math.inf


CASES = {
    # hot/cold policy, fp32, Llama-3.1-8B head geometry; the prompt eviction is larger
    # than the ring (672 > 512) so the ring wraps; decode step 33 compresses again.
    "hotcold_f32": dict(B=1, Hq=32, Hk=8, D=128, T=768, steps=40, dtype="float32", policy="hotcold",
                        cap=128, recent=32, topk_ratio=0.5, pool_kernel=7, ccap=512, faiss_dim=128,
                        window_size=8, pool=4, R=32, hold=True, rap=True, theta=500000.0),
    # SnapKV policy (window 32, max-pool 7), prefill-end retrieval of 64 from the last
    # 8 queries, held; one eviction per decode step.
    "snapkv_f32": dict(B=1, Hq=32, Hk=8, D=128, T=1024, steps=24, dtype="float32", policy="snapkv",
                       cap=128, recent=32, topk_ratio=0.0, pool_kernel=7, ccap=2048, faiss_dim=128,
                       window_size=1000, pool=8, R=64, hold=True, rap=True, theta=500000.0),
    # batch of 2, fp16, eviction only. With B > 1 the reference cannot inject retrieved
    # tokens: _rotate_k_with_pos (patch.py:94-102) builds cos/sin of shape (B,1,R,D) and
    # apply_rotary_pos_emb unsqueezes them again, so k_mem becomes (B,B,Hk,R,D) and
    # _canon_kv_4d raises. Retrieval is therefore off here (lookahead_k = 0).
    "hotcold_f16_b2": dict(B=2, Hq=8, Hk=2, D=128, T=512, steps=30, dtype="float16", policy="hotcold",
                           cap=96, recent=32, topk_ratio=0.4, pool_kernel=7, ccap=1024, faiss_dim=64,
                           window_size=4, pool=4, R=0, hold=False, rap=False, theta=500000.0),
    # fp16, cropped index vectors (faiss_dim 64 < D), attend-once injection every 4 steps.
    "hotcold_f16_once": dict(B=1, Hq=8, Hk=2, D=128, T=512, steps=30, dtype="float16", policy="hotcold",
                             cap=96, recent=32, topk_ratio=0.4, pool_kernel=7, ccap=1024, faiss_dim=64,
                             window_size=4, pool=4, R=16, hold=False, rap=False, theta=500000.0),
}


# fp16 SnapKV prompt compression at the benchmark's head geometry. The CUDA path scores a
# prompt this long on the tensor cores (the logits do not fit its selection CTA). The
# reference computes the logits in fp16, which leaves the keep boundary of any long prompt at
# relative gaps of 1e-4 or below (often exact ties), so this case is not step-exact: it keeps
# the reference's token scores and keep set of the prompt compression, and the tests accept a
# different keep set only where the reference's own scores are within the fp16 band of its
# boundary.
SNAPKV_F16_PROMPT = dict(B=1, Hq=32, Hk=8, D=128, T=2048, steps=1, dtype="float16", policy="snapkv", cap=256,
                         recent=32, topk_ratio=0.0, pool_kernel=7, ccap=4096, faiss_dim=128, window_size=1 << 20,
                         pool=4, R=32, hold=True, rap=False, theta=500000.0)


def run_snapkv_prompt_f16(seed: int):
    RECORD["snap"] = []
    res, _ = run_single_layer(SNAPKV_F16_PROMPT, seed)
    token, keep = RECORD["snap"][0]
    return dict(token_scores=token.astype(np.float32), keep_idx=keep.astype(np.int32), hot_pos=res["hot_pos"],
                hot_len=res["hot_len"], case=json.dumps(dict(SNAPKV_F16_PROMPT, seed=seed)))


def run_scores(seed: int):
    """Function-level golden for the two eviction scores in fp16 and fp32:
    the hot/cold score (cache.py:55-69) and SnapKV importance (scoring.py:50-79,
    maxpool 7) averaged over KV heads, plus keep_index (scoring.py:110-132) and
    pool1d (scoring.py:40-47). Multi-step fp16 SnapKV runs always meet exact ties
    of the fp16-computed scores, so fp16 scoring is pinned here, value by value.
    Inputs come from synth.score_case_inputs(seed)."""
    out = {}
    Hq, Hk, D, W = 32, 8, 128, 32
    for dt, (qn, kn) in synth.score_case_inputs(seed).items():
        q = torch.from_numpy(qn.astype(np.float32)).to(TORCH_DT[dt])
        k = torch.from_numpy(kn.astype(np.float32)).to(TORCH_DT[dt])
        imp = ref_scoring.snapkv_importance(q, k, W, 1.0 / math.sqrt(D), 7, "maxpool").mean(dim=1)
        qf = q[:, :, -W:].reshape(1, Hk, Hq // Hk, W, D).mean(dim=2)
        hc = (torch.matmul(qf, k.transpose(2, 3)) / math.sqrt(D)).sum(dim=2).mean(dim=1)
        tag = "f32" if dt == "float32" else "f16"
        out[f"snap_{tag}"], out[f"hc_{tag}"] = imp.float().numpy(), hc.float().numpy()
    rng = np.random.default_rng(seed + 1)
    sc = torch.from_numpy(rng.standard_normal((2, 3, 100), dtype=np.float32))
    out["ki_scores"] = sc.numpy()
    out["ki_full"] = ref_scoring.keep_index(sc, 8, 30).numpy()
    x = torch.from_numpy(rng.standard_normal((2, 3, 57), dtype=np.float32))
    out["pool_x"] = x.numpy()
    out["pool_max"] = ref_scoring.pool1d(x, 7, "maxpool").numpy()
    out["pool_avg"] = ref_scoring.pool1d(x, 7, "avgpool").numpy()
    return out


def run_triton_kernel(seed: int):
    """The reference decode kernel itself (kernels.py:9-74) under the Triton
    interpreter, with the wrapper's post-processing (kernels.py:134-137).
    Inputs come from synth.attention_case_inputs(seed)."""
    qn, kn, vn, mn = synth.attention_case_inputs(seed)
    q, k, v, m = (torch.from_numpy(x) for x in (qn, kn, vn, mn))
    B, Hq, _, D = q.shape
    Hk, S = k.shape[1], k.shape[2]
    ao = torch.empty_like(q)
    tl_ = torch.zeros((B, Hq, S), dtype=torch.float32)
    tl1 = torch.zeros((B, Hq, 1), dtype=torch.float32)
    sc = 1.0 / math.sqrt(D)
    ref_kernels.evict_fwd_kernel[(B, Hq)](
        q, k, v, m, ao, tl_, tl1, sc, Hq // Hk, Hq,
        *q.stride()[:2], q.stride(3), *k.stride(), *v.stride(), *m.stride(),
        ao.stride(0), ao.stride(1), ao.stride(3), *tl_.stride(), *tl1.stride(),
        D_HEAD=D, SEQ_LEN_KV=S, BLOCK_S=64)
    final = (tl_ / tl1).mean(dim=1).to(q.dtype)
    return dict(out=ao.transpose(1, 2).contiguous().numpy(), evict_idx=torch.argmin(final, -1).numpy(),
                final_loss=final.numpy())


TINY_MODEL = dict(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=128, rope_theta=500000.0,
                  max_position_embeddings=1024, rms_norm_eps=1e-5)
TINY_RUN = dict(T=200, steps=16, cap=64, recent=16, topk_ratio=0.5, ccap=4096, faiss_dim=128,
                window_size=4, pool=2, R=8, hold=True, rap=True, model_seed=1234, token_seed=99)


def run_tiny_model():
    """A 2-layer random Llama through the reference's patched forward (prefill then
    teacher-forced decode), logits per step."""
    for k in RECORD:
        RECORD[k] = []
    RECORD["retrieved"], RECORD["kmem"] = [], []
    ref_cache.HotColdLayer._compress_if_needed = _COMPRESS_HOTCOLD
    r = TINY_RUN
    torch.manual_seed(r["model_seed"])
    model = LlamaForCausalLM(LlamaConfig(**TINY_MODEL)).eval()
    rng = np.random.default_rng(r["token_seed"])
    # distinct token ids: a repeated prompt token gives layer 0 identical pre-RoPE
    # keys, hence identical cold-index vectors and exact search ties
    ids = torch.from_numpy(rng.permutation(TINY_MODEL["vocab_size"])[: r["T"] + r["steps"]][None, :])
    kv = hotcold_kv.KVController(
        max_capacity_prompt=r["cap"], topk_ratio=r["topk_ratio"], recent_size=r["recent"],
        cpu_buffer_size=r["ccap"], faiss_dim=r["faiss_dim"], window_size=r["window_size"],
        query_pool_size=r["pool"], lookahead_k=r["R"], hold_retrieved=r["hold"],
        retrieve_after_prefill=r["rap"], enable_asserts=True, profile_overlap=False)
    hotcold_kv.uninstall_monkeypatch()
    hotcold_kv.set_active_rotary_emb(model.model.rotary_emb)
    hotcold_kv.install_monkeypatch(enable_debug=False)
    hotcold_kv.set_active_kvctrl(kv)
    cache = hotcold_kv.build_hotcold_cache(model, kv)
    T = r["T"]
    logits = []
    with torch.inference_mode():
        out = model(input_ids=ids[:, :T], use_cache=True, past_key_values=cache)
        logits.append(out.logits[0, -1].float().numpy())
        for i in range(r["steps"]):
            # explicit position ids: transformers 5.x would derive them from the cache's
            # get_seq_length(), the compressed hot length, where 4.57 (the reference's pin) took
            # them from cache_position
            out = model(input_ids=ids[:, T + i:T + i + 1], cache_position=torch.tensor([T + i]),
                        position_ids=torch.tensor([[T + i]]), past_key_values=cache, use_cache=True)
            logits.append(out.logits[0, -1].float().numpy())
    hotcold_kv.uninstall_monkeypatch()
    hotcold_kv.set_active_kvctrl(None)
    return dict(ids=ids.numpy(), logits=np.stack(logits, 0),
                dbg=json.dumps({k: v for k, v in kv.dbg.items() if not k.startswith("prefetch_copy")}),
                cold_sizes=np.array([kv.cold_size(i) for i in range(TINY_MODEL["num_hidden_layers"])])), \
        _min_gap("float32")


def main():
    only = sys.argv[1:]
    for name, case in CASES.items():
        if only and name not in only:
            continue
        seed = case.get("seed0", 1000)
        for attempt in range(120):
            res, gap = run_single_layer(case, seed)
            if gap >= 1.0:
                break
            print(f"{name}: seed {seed} min gap ratio {gap:.2e} < 1, next seed")
            seed += 1
        else:
            raise SystemExit(f"{name}: no seed with comfortable gaps")
        res["case"] = json.dumps(dict(case, seed=seed, min_gap=gap))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **res)
        print(f"{name}: seed {seed} min gap {gap:.2e} dbg {res['dbg']}")
    if not only or "snapkv_f16_prompt" in only:
        np.savez_compressed(os.path.join(HERE, "snapkv_f16_prompt.npz"), **run_snapkv_prompt_f16(2024))
        print("snapkv_f16_prompt: done")
    if not only or "scores" in only:
        np.savez_compressed(os.path.join(HERE, "scores.npz"), **run_scores(11))
        print("scores: done")
    if not only or "triton_kernel" in only:
        res = run_triton_kernel(7)
        np.savez_compressed(os.path.join(HERE, "triton_kernel.npz"), **res)
        print("triton_kernel: evict_idx", res["evict_idx"])
    if not only or "tiny_model" in only:
        res, gap = run_tiny_model()
        res["case"] = json.dumps(dict(model=TINY_MODEL, run=TINY_RUN, min_gap=gap))
        np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **res)
        print(f"tiny_model: min gap {gap:.2e} dbg {res['dbg']}")


if __name__ == "__main__":
    main()
