"""HBM state of one attention layer and the C-ABI calls over it.

A LayerArena holds, for n_seq sequences, the hot slab (budget + 1 physical
slots with a logical-order table and a free-slot stack), the held segment of
retrieved tokens, the cold ring (payload + float32 index vectors), the query
pool and the device-resident counters, plus the descriptor array the kernels
read. All buffers are allocated once; every op afterwards is an asynchronous
launch on the current stream with no host synchronisation, so a decode step
can be captured in a CUDA graph.

The host keeps mirrors of the counters (hot length, cold count). They follow
from the schedule alone (compression plans depend only on lengths and
budgets), so the host never reads them back.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from ._lib import byref, call, ptr, size


# The last launch of this library on each stream, as (arena id, op name). hc_step may read part
# of a layer's state before its dependency wait (overlapping those copies with the launch before
# it) only when that launch wrote none of that state: see LayerArena._early_bits.
_LAST_OP: dict = {}
HC_STEP_EARLY_HOT, HC_STEP_EARLY_HELD = 1, 2


class Workspace:
    """Grow-only scratch buffer shared by the ops of one stream."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = torch.empty(0, dtype=torch.uint8, device=self.device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.empty(int(nbytes * 1.25) + 4096, dtype=torch.uint8, device=self.device)
        return self.buf


def plan_keep(policy: str, budget: int, recent: int, topk_ratio: float, S: int):
    """(prefix_len, n_top) of a compression of S hot tokens, or None when S <= budget.
    hot/cold: cache.py:44-53; SnapKV: scoring.py:117-120 with the trigger of cache.py:44."""
    if S <= budget:
        return None
    if policy == "hotcold":
        rec = min(recent, budget, S)
        prefix = S - rec
        if prefix <= 0:
            return None
        ntop = max(1, min(int(budget * topk_ratio), prefix))
        return prefix, ntop
    window = min(recent, S)
    prefix = S - window
    return prefix, max(0, min(budget - window, prefix))


class LayerArena:
    def __init__(self, *, n_seq: int, Hq: int, Hk: int, D: int, F: int, dtype, device, budgets, r_max: int,
                 ccap, p_max: int, policy: str, recent: int, topk_ratio: float, pool_kernel: int = 7,
                 pooling: str = "maxpool", normalize: bool = True, inv_freq: torch.Tensor, rope_scaling: float = 1.0,
                 workspace: Workspace | None = None, hot_cap_hint: int | None = None, cold_payload: str = "device"):
        """hot_cap_hint: initial physical hot slots when below budget + 1 (the slab grows on
        demand up to budget + 1, so a huge budget does not preallocate). cold_payload: "device"
        keeps the cold ring's pre-RoPE keys and values in HBM; "host" keeps them in page-locked
        host memory that the kernels address directly (evictions write it, retrievals gather
        their hits from it), for cold stores larger than HBM; the index vectors and positions
        stay in HBM either way, since every search scans them."""
        if cold_payload not in ("device", "host"):
            raise ValueError(f"cold_payload must be 'device' or 'host', not {cold_payload!r}")
        self.cold_payload = cold_payload
        _lib.load()
        dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("the hot/cold path runs on CUDA devices only")
        self.device, self.dtype = dev, dtype
        self.n_seq, self.Hq, self.Hk, self.D, self.F = n_seq, Hq, Hk, D, F
        budgets = [int(b) for b in (budgets if hasattr(budgets, "__len__") else [budgets] * n_seq)]
        ccaps = [int(c) for c in (ccap if hasattr(ccap, "__len__") else [ccap] * n_seq)]
        assert len(budgets) == n_seq and len(ccaps) == n_seq
        self.budgets, self.ccaps = budgets, ccaps
        self.policy, self.recent, self.topk_ratio = policy, int(recent), float(topk_ratio)
        self.r_max, self.p_max = int(r_max), int(p_max)
        caps = [b + 1 if hot_cap_hint is None else min(b + 1, max(int(hot_cap_hint), 1)) for b in budgets]
        self.caps = caps
        mc, R, C, P = max(caps), max(self.r_max, 1), max(max(ccaps), 1), max(self.p_max, 1)
        self.max_cap, self.max_ccap = mc, C
        z = dict(device=dev)
        self.hot_k = torch.empty((n_seq, Hk, mc, D), dtype=dtype, **z)
        self.hot_v = torch.empty((n_seq, Hk, mc, D), dtype=dtype, **z)
        self.hot_kpre = torch.empty((n_seq, Hk, mc, D), dtype=dtype, **z)
        self.hot_pos = torch.zeros((n_seq, mc), dtype=torch.int64, **z)
        self.hot_ord = torch.zeros((n_seq, mc), dtype=torch.int32, **z)
        self.hot_free = torch.zeros((n_seq, mc), dtype=torch.int32, **z)
        self.held_k = torch.zeros((n_seq, Hk, R, D), dtype=dtype, **z)
        self.held_v = torch.zeros((n_seq, Hk, R, D), dtype=dtype, **z)
        self.held_pos = torch.zeros((n_seq, R), dtype=torch.int64, **z)
        self.held_valid = torch.zeros((n_seq, R), dtype=torch.uint8, **z)
        self.held_src = torch.full((n_seq, R), -1, dtype=torch.int32, **z)
        self.cold_vec = torch.empty((n_seq, C, F), dtype=torch.float32, **z)
        if cold_payload == "host":
            self.cold_kpre = torch.empty((n_seq, C, Hk, D), dtype=dtype, pin_memory=True)
            self.cold_v = torch.empty((n_seq, C, Hk, D), dtype=dtype, pin_memory=True)
        else:
            self.cold_kpre = torch.empty((n_seq, C, Hk, D), dtype=dtype, **z)
            self.cold_v = torch.empty((n_seq, C, Hk, D), dtype=dtype, **z)
        self.cold_pos = torch.zeros((n_seq, C), dtype=torch.int64, **z)
        self.qwin = torch.zeros((n_seq, P, D), dtype=dtype, **z)
        self.st = torch.zeros((n_seq, 16), dtype=torch.int32, **z)
        self.counters = torch.zeros((n_seq * Hk,), dtype=torch.int32, **z)
        self.inv_freq = inv_freq.detach().to(device=dev, dtype=torch.float32).contiguous()
        self.q_post = torch.empty((n_seq, Hq, D), dtype=dtype, **z)
        self.out = torch.empty((n_seq, Hq, D), dtype=dtype, **z)
        self.ws = workspace or Workspace(dev)

        self.pool_kernel, self.pooling, self.normalize, self.rope_scaling = pool_kernel, pooling, normalize, rope_scaling
        self._step_ok: dict = {}
        self._dirty = True  # host-side (torch) writes since the last launch: no early reads next step
        self.launches = 0  # kernels launched by the decode-path ops (append/compress/retrieve/attend/step)
        self._build_descriptors()
        # host mirrors: hot and cold lengths, and the entries ever appended to each cold ring (the
        # ring's oldest live entry sits at slot (cold_pushed - cold_count) % ccap)
        self.n_hot = np.zeros(n_seq, np.int64)
        self.cold_count = np.zeros(n_seq, np.int64)
        self.cold_pushed = np.zeros(n_seq, np.int64)

    def _build_descriptors(self):
        n_seq, caps, budgets, ccaps = self.n_seq, self.caps, self.budgets, self.ccaps
        mc, C = self.max_cap, self.max_ccap
        descs = (_lib.HcSeqDesc * n_seq)()
        for s in range(n_seq):
            d = descs[s]
            d.hot_k = self.hot_k[s].data_ptr()
            d.hot_v = self.hot_v[s].data_ptr()
            d.hot_kpre = self.hot_kpre[s].data_ptr()
            d.hot_pos = self.hot_pos[s].data_ptr()
            d.hot_ord = self.hot_ord[s].data_ptr()
            d.hot_free = self.hot_free[s].data_ptr()
            d.held_k = self.held_k[s].data_ptr()
            d.held_v = self.held_v[s].data_ptr()
            d.held_pos = self.held_pos[s].data_ptr()
            d.held_valid = self.held_valid[s].data_ptr()
            d.held_src = self.held_src[s].data_ptr()
            d.cold_vec = self.cold_vec[s].data_ptr()
            d.cold_kpre = self._device_address(self.cold_kpre[s])
            d.cold_v = self._device_address(self.cold_v[s])
            d.cold_pos = self.cold_pos[s].data_ptr()
            d.qwin = self.qwin[s].data_ptr()
            d.st = self.st[s].data_ptr()
            d.cap, d.budget, d.r_max, d.ccap, d.p_max = caps[s], budgets[s], self.r_max, ccaps[s], self.p_max
        raw = bytes(ctypes.string_at(ctypes.addressof(descs), ctypes.sizeof(descs)))
        self.desc = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
        L = _lib.HcLayer()
        L.desc = self.desc.data_ptr()
        L.inv_freq = self.inv_freq.data_ptr()
        L.counters = self.counters.data_ptr()
        L.topk_ratio = self.topk_ratio
        L.n_seq, L.Hq, L.Hk, L.D, L.F = n_seq, self.Hq, self.Hk, self.D, self.F
        L.dtype = _lib.dtype_code(self.dtype)
        L.policy = _lib.HC_POLICY_HOTCOLD if self.policy == "hotcold" else _lib.HC_POLICY_SNAPKV
        L.recent = self.recent
        L.pool_kernel = int(self.pool_kernel)
        L.pooling = _lib.HC_POOL_MAX if self.pooling == "maxpool" else _lib.HC_POOL_AVG
        L.normalize = 1 if self.normalize else 0
        L.max_cap, L.max_r, L.max_ccap = mc, self.r_max, C
        L.scale = 1.0 / math.sqrt(self.D)
        L.rope_scaling = float(self.rope_scaling)
        L.kmaps = self._encode_kmaps()
        self.L = L
        self._Lref = byref(L)
        self._caps_np = np.asarray(self.caps, np.int64)
        self._plan_cache = {}
        self._dirty = True

    def _device_address(self, t: torch.Tensor) -> int:
        """The address kernels use for `t`: its own for device memory, the mapped device address
        of page-locked host memory."""
        if t.is_cuda:
            return t.data_ptr()
        dev = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("hc_host_device_pointer", t.data_ptr(), ctypes.byref(dev))
        return int(dev.value)

    def _encode_kmaps(self):
        """TMA tensor maps for the fused step's 16-bit path, all sequences as rows of D: the hot
        K slab (64-row boxes), the held K rows (8-row boxes), the hot V slab (16-row boxes) and
        the held V rows (8-row boxes); 0 when unavailable."""
        self.kmaps = None
        if self.dtype not in (torch.float16, torch.bfloat16):
            return 0
        buf = (ctypes.c_uint8 * 512)()
        code = _lib.dtype_code(self.dtype)
        lib = _lib.load()
        rc = 0
        for i, (t, box) in enumerate(((self.hot_k, 64), (self.held_k, 8), (self.hot_v, 16), (self.held_v, 8))):
            if rc == 0:
                rc = lib.hc_encode_kmap(ctypes.addressof(buf) + 128 * i, t.data_ptr(), code, t.numel() // self.D,
                                        self.D, box)
        if rc != 0:
            return 0
        self.kmaps = torch.frombuffer(bytearray(bytes(buf)), dtype=torch.uint8).to(self.device)
        return self.kmaps.data_ptr()

    def ensure_hot_capacity(self, need):
        """Grow the physical hot slab so that sequence s can hold need[s] tokens (capped at
        budget + 1). Contents, logical order and free slots carry over; runs only when the
        slab is too small, never in a steady decode loop."""
        need = np.broadcast_to(np.asarray(need, np.int64), (self.n_seq,))
        new_caps = [min(self.budgets[s] + 1, max(self.caps[s], int(need[s]))) for s in range(self.n_seq)]
        if new_caps == self.caps:
            return
        grown = [max(c, min(self.budgets[s] + 1, 2 * self.caps[s])) if c > self.caps[s] else c
                 for s, c in enumerate(new_caps)]
        mc_old, mc = self.max_cap, max(grown)
        if mc > mc_old:
            def grow(t, dim, fill=None):
                shape = list(t.shape)
                shape[dim] = mc
                n = torch.empty(shape, dtype=t.dtype, device=t.device) if fill is None else \
                    torch.full(shape, fill, dtype=t.dtype, device=t.device)
                n.narrow(dim, 0, mc_old).copy_(t)
                return n
            # per-sequence regions are [Hk][cap][D] with the sequence's own cap: re-lay them
            for name in ("hot_k", "hot_v", "hot_kpre"):
                old = getattr(self, name)
                new = torch.empty((self.n_seq, self.Hk, mc, self.D), dtype=old.dtype, device=old.device)
                for s in range(self.n_seq):
                    c = self.caps[s]
                    src = old[s].reshape(-1)[: self.Hk * c * self.D].view(self.Hk, c, self.D)
                    new[s].reshape(-1)[: self.Hk * grown[s] * self.D].view(self.Hk, grown[s], self.D)[:, :c] \
                        .copy_(src)
                setattr(self, name, new)
            self.hot_pos = grow(self.hot_pos, 1, 0)
            self.hot_ord = grow(self.hot_ord, 1, 0)
            self.hot_free = grow(self.hot_free, 1, 0)
        else:
            for name in ("hot_k", "hot_v", "hot_kpre"):
                t = getattr(self, name)
                for s in range(self.n_seq):
                    c, g = self.caps[s], grown[s]
                    if g != c:
                        buf = t[s].reshape(-1)
                        tmp = buf[: self.Hk * c * self.D].view(self.Hk, c, self.D).clone()
                        buf[: self.Hk * g * self.D].view(self.Hk, g, self.D)[:, :c].copy_(tmp)
        for s in range(self.n_seq):
            c, g = self.caps[s], grown[s]
            if g > c:
                nf = c - int(self.n_hot[s])
                self.hot_free[s, nf: nf + g - c] = torch.arange(g - 1, c - 1, -1, dtype=torch.int32,
                                                                device=self.device)
                self.st[s, 1] += g - c
        self.caps = grown
        self.max_cap = mc
        self._step_ok = {}
        self._build_descriptors()

    # ------------------------------------------------------------------ helpers
    def _stream(self):
        return _lib.stream_of(self.device)

    _hc_step = None  # the library's hc_step, looked up once

    def _launched(self, op: str, stream=None):
        """Record that `op` of this arena was the last launch on the stream."""
        _LAST_OP[stream if stream is not None else self._stream()] = (id(self), op)

    def _early_bits(self, stream) -> int:
        """HC_STEP_EARLY_* bits for a step about to launch on `stream`: what of this layer's
        state the launch before it left alone. Another layer's launch (or none of this library)
        writes nothing of it; this layer's decode retrieval writes the held segment only; any
        other op of this layer, or a host-side write, may write all of it."""
        if self._dirty:
            return 0
        last = _LAST_OP.get(stream)
        if last is None or last[0] != id(self):
            return HC_STEP_EARLY_HOT | HC_STEP_EARLY_HELD
        return HC_STEP_EARLY_HOT if last[1] == "retrieve_decode" else 0

    def _fast_rows(self, t: torch.Tensor, rows: int):
        """(tensor, sequence stride) of a (n_seq, rows, D) operand without copies when it is
        contiguous and 16-byte aligned; else the general _row_major path."""
        if t.is_contiguous() and t.numel() == self.n_seq * rows * self.D and t.data_ptr() % 16 == 0:
            return t, rows * self.D
        return self._row_major(t, rows)

    def _step_plan(self):
        """Evictions of every sequence when each holds one more token than now (the host
        mirror of the fused step's compression), cached by the hot lengths (the cache is reset
        when the capacities change): (ev, total, total capped by the cold capacities, whether
        every sequence has a free slot for the new token, the hot lengths after the step)."""
        key = self.n_hot.tobytes()
        e = self._plan_cache.get(key)
        if e is None:
            ev = np.zeros(self.n_seq, np.int64)
            for s in range(self.n_seq):
                p = self.plan(s, int(self.n_hot[s]) + 1)
                if p is not None:
                    ev[s] = p[0] - p[1]
            fits = not bool((self.n_hot >= self._caps_np).any())
            e = (ev, int(ev.sum()), int(np.minimum(ev, np.asarray(self.ccaps)).sum()), fits, self.n_hot + 1 - ev)
            if len(self._plan_cache) < 4096:
                self._plan_cache[key] = e
        return e

    def _ccaps_arr(self):
        c = getattr(self, "_ccaps_np", None)
        if c is None:
            c = self._ccaps_np = np.asarray(self.ccaps, np.int64)
        return c

    def _row_major(self, t: torch.Tensor, rows: int) -> tuple[torch.Tensor, int]:
        """(n_seq, rows, D) view with contiguous, 16-byte aligned rows; returns (tensor, seq stride)."""
        t = t.reshape(self.n_seq, rows, self.D) if t.dim() != 3 else t
        if t.stride(2) != 1 or t.stride(1) != self.D:
            t = t.contiguous()
        if t.data_ptr() % 16 or (t.stride(0) * t.element_size()) % 16:
            t = t.clone(memory_format=torch.contiguous_format)
        return t, t.stride(0)

    def plan(self, s: int, S: int):
        return plan_keep(self.policy, self.budgets[s], self.recent, self.topk_ratio, S)

    # ------------------------------------------------------------------ ops
    def store_prompt(self, k_post, v, k_pre, pos):
        """Prompt of T <= budget tokens into the slab (cache.py:145-148). Tensors (n_seq,Hk,T,D)."""
        T = k_post.shape[2]
        call("hc_store_prompt", byref(self.L), T, ptr(k_post), ptr(v), ptr(k_pre), *self._strides(k_post, v, k_pre),
             ptr(pos.contiguous()), self._stream())
        self._launched("store_prompt")
        self.n_hot[:] = T

    def _strides(self, k, v, kp):
        st = k.stride()
        if v.stride() != st or kp.stride() != st or st[3] != 1:
            raise ValueError("k_post, v and k_pre must share strides with unit stride over head_dim")
        return st[0], st[1], st[2]

    def hot_dense(self):
        """The hot tokens of every sequence in logical order as dense (n_seq, Hk, n_hot, D)
        tensors (k_post, v, k_pre) and positions (n_seq, n_hot); all sequences must hold the
        same number of tokens. Device gathers, no host synchronisation."""
        n = int(self.n_hot[0])
        if (self.n_hot != n).any():
            raise ValueError("hot_dense needs equal hot lengths")
        outs = []
        for name in ("hot_k", "hot_v", "hot_kpre"):
            t = getattr(self, name)
            rows = []
            for s in range(self.n_seq):
                c = self.caps[s]
                slab = t[s].reshape(-1)[: self.Hk * c * self.D].view(self.Hk, c, self.D)
                rows.append(slab.index_select(1, self.hot_ord[s, :n].long()))
            outs.append(torch.stack(rows, 0))
        pos = torch.stack([self.hot_pos[s].index_select(0, self.hot_ord[s, :n].long()) for s in range(self.n_seq)], 0)
        return outs[0], outs[1], outs[2], pos

    def _seq_view(self, s: int):
        """hc_layer over sequence s alone: the descriptor array and counters from its entry on,
        n_seq = 1 (every per-sequence buffer is reached through the descriptor)."""
        L = _lib.HcLayer()
        ctypes.memmove(ctypes.addressof(L), ctypes.addressof(self.L), ctypes.sizeof(L))
        L.desc = self.desc.data_ptr() + s * ctypes.sizeof(_lib.HcSeqDesc)
        L.counters = self.counters.data_ptr() + s * self.Hk * 4
        L.n_seq = 1
        L.kmaps = None
        return L

    def compress_prompt(self, q_obs, k_post, v, k_pre, pos, seq: int | None = None):
        """Prompt of T tokens into an empty slab: sequences with T > budget score, keep and
        evict into the cold ring (cache.py:37-128 on the prompt); the others keep the whole
        prompt. Tensors (n_seq,Hk,T,D), q_obs (n_seq,Hq,tq,D). With `seq`, the tensors hold
        that one sequence of a ragged batch (leading dimension 1). Returns evicted counts."""
        T = k_post.shape[2]
        seqs = range(self.n_seq) if seq is None else [int(seq)]
        need = np.asarray(self.caps, np.int64).copy() if seq is not None else np.zeros(self.n_seq, np.int64)
        for s in seqs:
            need[s] = min(T, self.budgets[s]) + 1
        self.ensure_hot_capacity(need)
        L = self.L if seq is None else self._seq_view(int(seq))
        tq = q_obs.shape[2]
        qs = q_obs.stride()
        nbytes = size("hc_compress_scratch_bytes", byref(L), T, tq)
        ws = self.ws.get(nbytes)
        pos = pos.contiguous()
        call("hc_compress_ex", byref(L), ptr(q_obs), qs[0], qs[1], qs[2], tq, T, ptr(k_post), ptr(v), ptr(k_pre),
             *self._strides(k_post, v, k_pre), ptr(pos), ptr(ws), ws.numel(), 1 << 30, self._stream())
        self._launched("compress_prompt")
        ev = np.zeros(self.n_seq, np.int64)
        for s in seqs:
            p = self.plan(s, T)
            if p is None:
                self.n_hot[s] = T
                continue
            prefix, ntop = p
            ev[s] = prefix - ntop
            self.n_hot[s] = T - ev[s]
        self._cold_push(ev)
        return ev

    def append(self, q_pre, k_pre, v, cos, sin, pos):
        """Decode-step RoPE + append + query-pool push. q_pre (n_seq,Hq,D), k_pre/v (n_seq,Hk,D),
        cos/sin (n_seq,D) or None, pos (n_seq,) int64. Returns q_post (n_seq,Hq,D)."""
        if (self.n_hot + 1 > np.asarray(self.caps)).any():
            self.ensure_hot_capacity(self.n_hot + 1)
        q, qss = self._row_major(q_pre, self.Hq)
        k, kss = self._row_major(k_pre, self.Hk)
        vv, vss = self._row_major(v, self.Hk)
        if vss != kss:
            k, vv = k.contiguous(), vv.contiguous()
            kss = k.stride(0)
        if cos is not None:
            cos = cos.reshape(self.n_seq, self.D).contiguous()
            sin = sin.reshape(self.n_seq, self.D).contiguous()
        call("hc_append", byref(self.L), ptr(q), qss, ptr(k), ptr(vv), kss, ptr(cos), ptr(sin), ptr(pos),
             ptr(self.q_post), self._stream())
        self._launched("append")
        self.launches += 1
        self.n_hot += 1
        return self.q_post

    def step_supported(self, use_held: bool) -> bool:
        """Whether the fused decode step fits this layer (one 16-CTA cluster per sequence)."""
        key = bool(use_held)
        if key not in self._step_ok:
            ok = self.n_seq >= 1 and self.Hk <= 16 and 16 % self.Hk == 0 and self.Hq // self.Hk in (1, 2, 4, 8)
            if ok:
                with torch.cuda.device(self.device):
                    ok = _lib.load().hc_step_check(byref(self.L), 1 if key else 0) == 0
            self._step_ok[key] = ok
        return self._step_ok[key]

    def step(self, q_pre, k_pre, v, cos, sin, pos, use_held: bool, overflow_nan: bool = True, out=None):
        """Fused decode step: append + compression with eviction + attention over [held | hot]
        in one launch (hc_step). Returns (output (n_seq,Hq,D), evicted counts), or None when
        the fused kernel does not fit this layer (nothing launched; use append/compress/attend).
        `out`, when given, is a contiguous (n_seq,Hq,D) tensor of the layer dtype to write."""
        plan = self._step_plan()
        if not plan[3] or not self.step_supported(use_held):
            return None
        q, qss = self._fast_rows(q_pre, self.Hq)
        k, kss = self._fast_rows(k_pre, self.Hk)
        vv, vss = self._fast_rows(v, self.Hk)
        if vss != kss:
            k, vv = k.contiguous(), vv.contiguous()
            kss = k.stride(0)
        if cos is not None and not (cos.is_contiguous() and sin.is_contiguous()
                                    and cos.numel() == self.n_seq * self.D == sin.numel()):
            cos = cos.reshape(self.n_seq, self.D).contiguous()
            sin = sin.reshape(self.n_seq, self.D).contiguous()
        o = self.out if out is None else out
        stream = self._stream()
        fn = self._hc_step
        if fn is None:
            fn = self._hc_step = _lib.load().hc_step
        rc = fn(self._Lref, q.data_ptr(), qss, k.data_ptr(), vv.data_ptr(), kss, ptr(cos), ptr(sin), pos.data_ptr(),
                1 if use_held else 0, o.data_ptr(), 1 if overflow_nan else 0, self._early_bits(stream), stream)
        if rc == 3:  # HC_ERR_UNSUPPORTED: nothing was launched
            self._step_ok[bool(use_held)] = False
            return None
        if rc != 0:
            raise RuntimeError(f"hc_step failed (code {rc}): {_lib.load().hc_last_error().decode()}")
        self._launched("step", stream)
        self._dirty = False
        self.launches += 1
        ev, tot, capped, _, n_after = plan
        self.last_ev = (tot, capped)
        self.n_hot[:] = n_after
        if tot:
            self.cold_pushed += ev
            np.minimum(self.cold_count + ev, self._ccaps_arr(), out=self.cold_count)
        return o, ev

    def append_rotated(self, k_post, k_pre, v, pos):
        if (self.n_hot + 1 > np.asarray(self.caps)).any():
            self.ensure_hot_capacity(self.n_hot + 1)
        k, kss = self._row_major(k_post, self.Hk)
        kp = k_pre.reshape(self.n_seq, self.Hk, self.D).contiguous()
        vv = v.reshape(self.n_seq, self.Hk, self.D).contiguous()
        k = k.contiguous()
        call("hc_append_rotated", byref(self.L), ptr(k), ptr(kp), ptr(vv), k.stride(0), ptr(pos), self._stream())
        self._launched("append_rotated")
        self.n_hot += 1

    def compress_decode(self, q_obs):
        """Compression of the slab when a sequence holds more than its budget. q_obs
        (n_seq,Hq,tq,D). Returns evicted counts per sequence (all zero when no sequence
        compresses; nothing is launched then)."""
        ev = np.zeros(self.n_seq, np.int64)
        active = False
        for s in range(self.n_seq):
            p = self.plan(s, int(self.n_hot[s]))
            if p is not None:
                active = True
                ev[s] = p[0] - p[1]
        if not active:
            return ev
        tq = q_obs.shape[2]
        qs = q_obs.stride()
        nbytes = size("hc_compress_scratch_bytes", byref(self.L), self.max_cap, tq)
        ws = self.ws.get(nbytes)
        call("hc_compress_ex", byref(self.L), ptr(q_obs), qs[0], qs[1], qs[2], tq, 0, None, None, None, 0, 0, 0, None,
             ptr(ws), ws.numel(), int(ev.max()), self._stream())
        self._launched("compress_decode")
        self.launches += 2 + (1 if int(ev.max()) > 32 else 0)
        self.n_hot -= ev
        self._cold_push(ev)
        return ev

    def retrieve(self, q_dense=None, n_pool: int = 0, extra_sum=None, extra_n: int = 0, qvec=None, ws=None,
                 stream=None):
        """Search + gather + re-RoPE into the held segment. `stream` (a torch.cuda.Stream) and its
        Workspace `ws`: where it runs when that is not the current stream (a side stream)."""
        nbytes = size("hc_retrieve_scratch_bytes", byref(self.L))
        ws = (ws or self.ws).get(nbytes)
        sh = stream.cuda_stream if stream is not None else self._stream()
        qd = (0, 0, 0)
        P = 0
        if q_dense is not None:
            qd = q_dense.stride()[:3]
            P = q_dense.shape[2]
        mc = int(self.cold_count.max())
        call("hc_retrieve_ex", byref(self.L), ptr(q_dense), qd[0], qd[1], qd[2], P, int(n_pool), ptr(extra_sum),
             int(extra_n), ptr(qvec), ptr(ws), ws.numel(), mc, sh)
        self._launched("retrieve", sh)
        self.launches += 1 if self._retr_fused() else (3 if qvec is not None else 4)

    def retrieve_sharded(self, searcher, q_dense=None, n_pool: int = 0, extra_sum=None, extra_n: int = 0,
                         qvec=None, ws=None):
        """hc_retrieve with the scan divided by token range over the ranks of `searcher` (a
        shard.ShardedColdSearch): pooled query (hc_retrieve_query), this rank's range of every
        sequence's cold entries scored and cut to its top R (hc_cold_topk), the all-gather and
        merge to the global top R, then the same splice on every rank (hc_splice_hits). A
        token range is a range of ages (0 = the oldest live entry); on a ring that has wrapped
        it covers at most two runs of contiguous slots (shard.age_runs), searched separately
        and merged on this rank before the exchange. `ws`: the Workspace of the stream it runs on,
        when that is not the arena's (a side stream)."""
        if qvec is None:
            qvec = torch.empty((self.n_seq, self.F), dtype=torch.float32, device=self.device)
            qd, P = (0, 0, 0), 0
            if q_dense is not None:
                qd, P = q_dense.stride()[:3], q_dense.shape[2]
            call("hc_retrieve_query", byref(self.L), ptr(q_dense), qd[0], qd[1], qd[2], P, int(n_pool),
                 ptr(extra_sum), int(extra_n), ptr(qvec), self._stream())
            self.launches += 1
        from .shard import age_runs, token_range
        runs, n = [], []
        heads = self.cold_head()
        for s in range(self.n_seq):
            c = int(self.cold_count[s])
            lo, hi = token_range(c, searcher.rank, searcher.world)
            runs.append([(self.cold_vec[s, s0:s0 + cnt], age0)
                         for s0, cnt, age0 in age_runs(int(heads[s]), self.ccaps[s], lo, hi)])
            n.append(c)
        searcher.ws = ws or self.ws
        k = max(self.r_max, 1)
        ids = searcher.search(runs, n, qvec, k)
        call("hc_splice_hits", byref(self.L), ptr(ids), k, self._stream())
        self._launched("retrieve_sharded")
        # per sequence: scan + merge per run, a merge of two runs, the merge of the ranks; one splice
        self.launches += sum(2 * max(len(r), 1) + (len(r) == 2) for r in runs) + \
            (self.n_seq if searcher.world > 1 else 0) + 1

    def _retr_fused(self) -> bool:
        """Whether hc_retrieve runs as the one-launch cluster kernel (its shared memory fits)."""
        p2 = lambda x: 1 << max(0, int(x) - 1).bit_length()
        nloc2 = p2(max(32, -(-self.max_ccap // 16)))
        R2 = p2(max(1, self.r_max))
        r16 = lambda b: (b + 15) // 16 * 16
        nr = 1
        while nr * 32 < nloc2:
            nr <<= 1
        RL = max(R2, 32)
        smem = (r16(self.Hq * self.D * 4) + r16(self.F * 4) + 128 + r16(max(nloc2, 32) * 8 + RL * 8)
                + r16(nr * RL * 8) + r16(16 * RL * 8) + 2 * r16(R2 * 4) + r16(-(-R2 // 16) * self.D * 4 + 16))
        return smem <= 200 * 1024 and self.F <= 4096 and R2 <= 256

    def retrieve_decode(self, q_pre, n_pool: int) -> bool:
        """One-launch search + gather + re-RoPE with this step's q_pre (n_seq, Hq, D) as the
        newest query-pool entry plus the n_pool newest pool entries. False when the fused
        retrieval kernel does not fit (nothing launched)."""
        nbytes = size("hc_retrieve_scratch_bytes", byref(self.L))
        ws = self.ws.get(nbytes)
        q, qss = self._row_major(q_pre, self.Hq)
        rc = _lib.load().hc_retrieve_decode(byref(self.L), ptr(q), qss, int(n_pool), ptr(ws), ws.numel(),
                                            self._stream())
        if rc == 3:
            return False
        if rc != 0:
            raise RuntimeError(f"hc_retrieve_decode failed (code {rc}): {_lib.load().hc_last_error().decode()}")
        self._launched("retrieve_decode")
        self.launches += 1
        return True

    def prompt_query_sum(self, q_dense):
        """Sum over the prompt's positions of its head-mean pre-RoPE queries (n_seq, D) fp32."""
        out = torch.empty((self.n_seq, self.D), dtype=torch.float32, device=self.device)
        qs = q_dense.stride()
        ws = self.ws.get(size("hc_prompt_query_sum_scratch_bytes", byref(self.L)))
        call("hc_prompt_query_sum", byref(self.L), ptr(q_dense), qs[0], qs[1], qs[2], q_dense.shape[2], ptr(out),
             ptr(ws), ws.numel(), self._stream())
        self._launched("prompt_query_sum")
        return out

    def attend(self, q_post, cur_pos, use_held: bool, overflow_nan: bool = True, out=None):
        nbytes = size("hc_attend_scratch_bytes", byref(self.L))
        ws = self.ws.get(nbytes)
        q = q_post if q_post.is_contiguous() else q_post.contiguous()
        o = self.out if out is None else out
        call("hc_attend", byref(self.L), ptr(q), ptr(cur_pos), 1 if use_held else 0, ptr(o),
             1 if overflow_nan else 0, ptr(ws), ws.numel(), self._stream())
        self._launched("attend")
        self.launches += 1
        return o

    def cold_append(self, k_pre, v, pos, evicted_idx):
        """Evicted tokens (n_seq,Hk,Te,D) into the cold ring (controller.py:190-238)."""
        Te = k_pre.shape[2]
        st = k_pre.stride()
        if v.stride() != st:
            v = v.contiguous()
            k_pre = k_pre.contiguous()
            st = k_pre.stride()
        idx = evicted_idx.to(device=self.device, dtype=torch.int64).contiguous()
        call("hc_cold_append", byref(self.L), ptr(k_pre), ptr(v), st[0], st[1], st[2],
             ptr(pos.to(device=self.device, dtype=torch.int64).contiguous()), ptr(idx), Te, self._stream())
        self._launched("cold_append")
        m = (evicted_idx >= 0).sum(dim=1).cpu().numpy()
        self._cold_push(m)
        return m

    def _cold_push(self, ev):
        """Host mirror of ev[s] entries appended to each cold ring (the device ring keeps the
        newest ccap: hc_seq_state cold_head/cold_count)."""
        ev = np.asarray(ev, np.int64)
        self.cold_pushed += ev
        np.minimum(self.cold_count + ev, self._ccaps_arr(), out=self.cold_count)

    def cold_head(self) -> np.ndarray:
        """Physical slot of each ring's oldest live entry (host mirror, no synchronisation)."""
        return (self.cold_pushed - self.cold_count) % np.maximum(self._ccaps_arr(), 1)

    # ------------------------------------------------------------------ views (API, not the hot path)
    # ------------------------------------------------------------------ persistence
    _STATE_TENSORS = ("hot_k", "hot_v", "hot_kpre", "hot_pos", "hot_ord", "hot_free", "held_k", "held_v",
                      "held_pos", "held_valid", "held_src", "cold_vec", "cold_kpre", "cold_v", "cold_pos", "qwin",
                      "st", "counters")

    def state_dict(self, pin: bool = True) -> dict:
        """The arena's HBM contents and host mirrors, copied to host memory (page-locked when
        `pin`): the hot slab with its order table and free stack, the held segment, the cold
        ring (payload, index vectors, positions), the query pool and the device counters.
        Synchronises the current stream."""
        out = {"geometry": dict(n_seq=self.n_seq, Hq=self.Hq, Hk=self.Hk, D=self.D, F=self.F,
                                dtype=str(self.dtype), budgets=list(self.budgets), ccaps=list(self.ccaps),
                                r_max=self.r_max, p_max=self.p_max, policy=self.policy, recent=self.recent),
               "caps": list(self.caps), "n_hot": self.n_hot.copy(), "cold_count": self.cold_count.copy()}
        for name in self._STATE_TENSORS:
            t = getattr(self, name)
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin)
            h.copy_(t, non_blocking=pin)
            out[name] = h
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def load_state_dict(self, sd: dict) -> None:
        """Restore a state_dict() into this arena (same geometry; the hot slab grows to the
        saved capacity first). Host-to-device copies on the current stream."""
        g = sd["geometry"]
        mine = dict(n_seq=self.n_seq, Hq=self.Hq, Hk=self.Hk, D=self.D, F=self.F, dtype=str(self.dtype),
                    budgets=list(self.budgets), ccaps=list(self.ccaps), r_max=self.r_max, p_max=self.p_max,
                    policy=self.policy, recent=self.recent)
        if g != mine:
            raise ValueError(f"arena geometry differs: saved {g}, here {mine}")
        self.ensure_hot_capacity(sd["caps"])
        if list(self.caps) != list(sd["caps"]):
            raise ValueError("hot slab capacity differs from the saved one")
        for name in self._STATE_TENSORS:
            getattr(self, name).copy_(sd[name], non_blocking=True)
        self.n_hot[:] = sd["n_hot"]
        self.cold_count[:] = sd["cold_count"]
        # entries ever appended, up to a multiple of the ring size: head + count
        self.cold_pushed[:] = sd["st"][:, 2].numpy().astype(np.int64) + self.cold_count
        self._plan_cache = {}
        self._dirty = True

    def logical_order(self, s: int) -> torch.Tensor:
        return self.hot_ord[s, : int(self.n_hot[s])].long()

    def hot_view(self, which: str) -> torch.Tensor:
        """(n_seq, Hk, S, D) of the hot tier in logical order (all sequences of equal length)."""
        src = {"k": self.hot_k, "v": self.hot_v, "kpre": self.hot_kpre}[which]
        return torch.stack([src[s].index_select(1, self.logical_order(s)) for s in range(self.n_seq)], 0)

    def hot_positions(self) -> torch.Tensor:
        return torch.stack([self.hot_pos[s].index_select(0, self.logical_order(s)) for s in range(self.n_seq)], 0)

    def cold_order(self, s: int) -> torch.Tensor:
        """Physical ring slots of sequence s, oldest first (device tensor)."""
        st = self.st[s].cpu()
        head, count = int(st[2]), int(st[3])
        return (torch.arange(count, device=self.device) + head) % self.ccaps[s]

    def device_state(self) -> np.ndarray:
        """Counters as the kernels see them (synchronises)."""
        return self.st.cpu().numpy()
