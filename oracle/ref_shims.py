"""Drive the reference implementation itself (tarun931/hotcold-kv-cache) for timing.

TEST AND BASELINE INFRASTRUCTURE ONLY. `bench.py` uses this module for its reference arm
(`--impl reference`), its `cpu_baseline` and the Triton bar; nothing on the product path
imports it. It imports the UNMODIFIED reference package `hotcold_kv` from `baseline/_ref`
(installed there with `pip install --no-deps --target baseline/_ref <reference checkout>`), or
from $HOTCOLD_REFERENCE_SRC, and runs it through its own public API: the patched
`LlamaAttention.forward` (patch.py:122-348) on a stub attention module whose projections
return seeded synthetic pre-RoPE tensors and whose o_proj is the identity.

Shims (none edits the reference's files; all are attribute replacements at run time):
 1. `faiss` (an unpinned dependency, controller.py:6) is not installed: `IndexFlatIP` is
    replaced by an exact float32 inner-product index (add, search sorted by score with ties
    to the lower id, remove_ids(IDSelectorRange), ntotal).
 2. transformers 5.x passes an int to `get_mask_sizes` (cache.py:153-156 expects 4.x's
    cache_position tensor): an int is accepted.
 3. On a host without CUDA (`cpu=True`): `pin_memory=True` is dropped, the retrieval thread
    (controller.py:336-341) runs synchronously on start(), and the prefetch/poll pair
    (controller.py:344-442) stages the retrieved pack on the host, so that retrieved tokens
    are attended (the reference's CPU path never attends them: poll_staged_gpu returns
    ready=False without CUDA).
 4. SnapKV policy: HotColdLayer._compress_if_needed is replaced by the composition of the
    reference's own SnapKV functions (scoring.snapkv_importance + keep_index, scoring.py:50-132)
    averaged over KV heads into one token score, with the rest of the hot/cold eviction flow
    (cache.py:78-128) unchanged. With policy="hotcold" the reference's method runs as is.
"""

from __future__ import annotations

import math
import os
import sys
import threading
import types

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_path() -> str | None:
    """Directory that holds the reference's `hotcold_kv` package, or None."""
    for cand in (os.environ.get("HOTCOLD_REFERENCE_SRC"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "hotcold_kv")):
            return cand
    return None


class _IDSelectorRange:
    def __init__(self, lo, hi):
        self.lo, self.hi = int(lo), int(hi)


class IndexFlatIP:
    """Exact float32 inner-product index with the calls the reference makes
    (controller.py:121-122, 223, 232, 274)."""

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
        sc = q @ self._x.T
        D = np.full((q.shape[0], k), -np.inf, np.float32)
        I = np.full((q.shape[0], k), -1, np.int64)
        for r in range(q.shape[0]):
            order = np.lexsort((np.arange(self.ntotal), -sc[r].astype(np.float64)))[:k]
            D[r, :len(order)] = sc[r, order]
            I[r, :len(order)] = order
        return D, I


class _SyncThread:
    def __init__(self, target=None, args=(), kwargs=None, daemon=None):
        self._t, self._a, self._k = target, args, kwargs or {}

    def start(self):
        self._t(*self._a, **self._k)

    def is_alive(self):
        return False


_LOADED = {}


def load_reference(cpu: bool):
    """Import the reference package with the shims above; cpu=True adds the host-only ones.
    Returns a namespace of its modules. Raises ImportError when it is not installed."""
    key = bool(cpu)
    if key in _LOADED:
        return _LOADED[key]
    path = reference_path()
    if path is None:
        raise ImportError("the reference is not installed under baseline/_ref (nor HOTCOLD_REFERENCE_SRC)")
    import torch
    if "faiss" not in sys.modules:
        fm = types.ModuleType("faiss")
        fm.Index = IndexFlatIP
        fm.IndexFlatIP = IndexFlatIP
        fm.IDSelectorRange = _IDSelectorRange
        sys.modules["faiss"] = fm
    if path not in sys.path:
        sys.path.insert(0, path)
    import hotcold_kv
    from hotcold_kv import cache as ref_cache
    from hotcold_kv import controller as ref_ctrl
    from hotcold_kv import patch as ref_patch
    from hotcold_kv.baselines import scoring as ref_scoring
    from hotcold_kv.datatypes import EvictedKV, RetrievedKV, _canon_br_2d, _canon_kv_4d

    def _get_mask_sizes(self, cache_position):
        q = cache_position if isinstance(cache_position, int) else int(cache_position.shape[0])
        return int(self.get_seq_length() + q), 0

    ref_cache.HotColdLayer.get_mask_sizes = _get_mask_sizes
    if cpu:
        if not torch.cuda.is_available():
            # page-locked host memory needs a CUDA driver (the reference's tests do the same,
            # tests/test_cold_store.py:33-36); this process only runs the reference then
            _zeros, _empty = torch.zeros, torch.empty
            torch.zeros = lambda *a, **k: _zeros(*a, **{x: y for x, y in k.items() if x != "pin_memory"})
            torch.empty = lambda *a, **k: _empty(*a, **{x: y for x, y in k.items() if x != "pin_memory"})
        ref_ctrl.threading = types.SimpleNamespace(Thread=_SyncThread, Lock=threading.RLock, RLock=threading.RLock)

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
            kpre, v = _canon_kv_4d(kpre, "staged.k_pre"), _canon_kv_4d(v, "staged.v")
            pos, valid = _canon_br_2d(pos, "staged.pos"), _canon_br_2d(valid, "staged.valid")
            return RetrievedKV(k_pre=kpre, v=v, pos=pos, valid=valid, ready=bool(valid.any().item()))

        ref_ctrl.KVController.maybe_prefetch_to_gpu = _prefetch_cpu
        ref_ctrl.KVController.poll_staged_gpu = _poll_cpu
    ns = types.SimpleNamespace(hotcold_kv=hotcold_kv, cache=ref_cache, controller=ref_ctrl, patch=ref_patch,
                               scoring=ref_scoring, EvictedKV=EvictedKV, path=path,
                               hotcold_compress=ref_cache.HotColdLayer._compress_if_needed)
    _LOADED[key] = ns
    return ns


def snapkv_compress(ref, pool_kernel: int = 7, pooling: str = "maxpool"):
    """HotColdLayer._compress_if_needed built from the reference's SnapKV functions: score =
    snapkv_importance (scoring.py:50-79) over the stashed observation queries, averaged over
    KV heads; keep = keep_index (scoring.py:110-132); then the reference's eviction flow
    (cache.py:78-128): gather the kept tokens, hand the evicted ones to the cold store."""
    import torch

    def _compress(self, layer_idx):
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
        q_full = torch.zeros(B, q.shape[1], S, D, dtype=q.dtype, device=q.device)
        q_full[:, :, S - tq:] = q[:, :, -tq:]
        imp = ref.scoring.snapkv_importance(q_full, self.keys, tq, 1.0 / math.sqrt(D), pool_kernel, pooling)
        token = imp.mean(dim=1, keepdim=True)
        keep_idx = ref.scoring.keep_index(token, window, cap)[:, 0]
        keep_len = keep_idx.shape[1]
        idx_k = keep_idx.unsqueeze(1).unsqueeze(-1).expand(B, Hk, keep_len, D)
        keys_new, values_new = self.keys.gather(2, idx_k), self.values.gather(2, idx_k)
        pre_new, pos_new = self.pre_keys.gather(2, idx_k), self.positions.gather(1, keep_idx)
        mask = torch.ones((B, prefix_len), dtype=torch.bool, device=self.keys.device)
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
                ii[b, :te] = t.cpu()
                kp[b, :, :te] = self.pre_keys[b, :, t].float().cpu()
                vv[b, :, :te] = self.values[b, :, t].float().cpu()
                pp[b, :te] = self.positions[b, t].cpu()
            self.kvctrl.dbg["compress_calls"] += 1
            self.kvctrl.dbg["evicted_tokens"] += int((ii >= 0).sum().item())
            self.kvctrl.add_evicted_to_cold_store(layer_idx, ref.EvictedKV(kp, vv, pp, ii))
        self.keys, self.values, self.pre_keys, self.positions = keys_new, values_new, pre_new, pos_new
    return _compress


class StubAttention:
    """Stands in for a LlamaAttention module: q/k/v projections return given tensors, o_proj
    is the identity."""

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


def time_reference_layer(c: dict, seed: int, warmup: int, steps: int, device: str = "cpu"):
    """One attention layer of the reference's patched forward on `device`: the prompt
    (untimed), `warmup` untimed and `steps` timed decode steps (time.perf_counter around each
    forward call, synchronised on CUDA). c: bench.py config(). Returns (us per timed
    layer-step, list of per-step us, dbg counters)."""
    import time

    import torch
    from transformers import LlamaConfig
    from transformers.cache_utils import Cache
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from hotcold_kv_cache_b200 import synth
    cpu = device == "cpu"
    ref = load_reference(cpu=cpu)
    hk = ref.hotcold_kv
    dev = torch.device(device)
    dt = {"float16": torch.float16, "float32": torch.float32, "bfloat16": torch.bfloat16}[c["dtype"]]
    Hq, Hk, D, T = c["Hq"], c["Hk"], c["D"], c["prompt"]
    n = warmup + steps
    inp = synth.layer_inputs(seed, 1, Hq, Hk, D, T, n, c["dtype"])
    inp = {k: torch.from_numpy(np.ascontiguousarray(v).astype(np.float32)).to(device=dev, dtype=dt)
           for k, v in inp.items()}
    ref.cache.HotColdLayer._compress_if_needed = (snapkv_compress(ref, c["pool_kernel"]) if c["policy"] == "snapkv"
                                                  else ref.hotcold_compress)
    kv = hk.KVController(max_capacity_prompt=c["budget"], topk_ratio=c["topk_ratio"], recent_size=c["recent"],
                         cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], normalize_for_ip=True,
                         window_size=c["window_size"], query_pool_size=c["query_pool_size"],
                         lookahead_k=c["lookahead_k"], hold_retrieved=c["hold"], retrieve_after_prefill=False,
                         enable_asserts=True, profile_overlap=False)
    hk.uninstall_monkeypatch()
    hk.install_monkeypatch(enable_debug=False)
    fwd = ref.patch.modeling_llama.LlamaAttention.forward
    lc = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hk, head_dim=D,
                     num_hidden_layers=1, rope_theta=c["theta"], vocab_size=16, intermediate_size=16,
                     max_position_embeddings=T + n + 8)
    rot = LlamaRotaryEmbedding(lc).to(dev)
    hk.set_active_rotary_emb(rot)
    hk.set_active_kvctrl(kv)
    layer = ref.cache.HotColdLayer(kv)
    cache = Cache(layers=[layer])
    stub = StubAttention(Hq, Hk, D)

    def proj(x, H):
        return x.transpose(1, 2).reshape(1, x.shape[2], H * D)

    stub._q, stub._k, stub._v = proj(inp["q_pre"], Hq), proj(inp["k_pre"], Hk), proj(inp["v"], Hk)
    pos = torch.arange(T, device=dev).unsqueeze(0)
    cos, sin = rot(torch.empty(1, T, Hq * D, dtype=dt, device=dev), pos)
    sync = (lambda: torch.cuda.synchronize(dev)) if not cpu else (lambda: None)
    times = []
    try:
        with torch.inference_mode():
            fwd(stub, torch.zeros(1, T, 1, dtype=dt, device=dev), (cos, sin), None, past_key_values=cache,
                cache_position=torch.arange(T, device=dev))
            for i in range(n):
                p = T + i
                stub._q = inp["dq"][i][:, None].reshape(1, 1, Hq * D)
                stub._k = inp["dk"][i][:, None].reshape(1, 1, Hk * D)
                stub._v = inp["dv"][i][:, None].reshape(1, 1, Hk * D)
                posd = torch.full((1, 1), p, dtype=torch.long, device=dev)
                cs, sn = rot(torch.empty(1, 1, Hq * D, dtype=dt, device=dev), posd)
                sync()
                t0 = time.perf_counter()
                fwd(stub, torch.zeros(1, 1, 1, dtype=dt, device=dev), (cs, sn), None, past_key_values=cache,
                    cache_position=torch.tensor([p], device=dev))
                sync()
                if i >= warmup:
                    times.append((time.perf_counter() - t0) * 1e6)
    finally:
        hk.uninstall_monkeypatch()
        hk.set_active_kvctrl(None)
        ref.cache.HotColdLayer._compress_if_needed = ref.hotcold_compress
    return float(np.mean(times)), times, dict(kv.dbg)
