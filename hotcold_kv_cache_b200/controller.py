"""KVController: the cold store, the retrieval schedule and the held set.

Same constructor, members and counters as the reference KVController
(controller.py:14-442 of src/hotcold_kv). What changes is where things live:
the cold tier is an HBM ring per (layer, sequence) with float32 index vectors
instead of host deques plus a CPU FAISS index, the search is a CUDA scan +
exact top-k instead of a daemon thread, and retrieved tokens go straight into
a held segment in HBM instead of a pinned buffer and a side-stream copy.

Schedule. A retrieval that fires at a decode step (every `window_size` forward
calls, controller.py:314-342) is attended at that same step; the prompt-end
retrieval (patch.py:231-233) is attended at decode step 1. The reference's
asynchronous thread makes that step nondeterministic; this is the
deterministic order its synchronous path would give. With async_retrieval the
search instead runs on a side stream after the step's compression, overlapping
the next layers, and is attended from the layer's next step (another order the
thread can give, as deterministic). Nothing here blocks the host: every op is an
asynchronous launch on the current stream (or, for those searches, a side
stream joined by events).
"""

from __future__ import annotations

from collections import deque
from typing import List, Optional

import numpy as np
import torch
import torch.nn.functional as F

from .arena import LayerArena, Workspace
from .datatypes import EvictedKV, RetrievedKV, _canon_br_2d, _canon_kv_4d

DBG_KEYS = (
    "compress_calls", "evicted_tokens", "faiss_add",
    "retrieval_launched", "retrieval_launched_prefill", "retrieval_ready_cpu", "retrieval_skipped_no_cold",
    "retrieval_ready_empty",
    "prefetch_launched", "prefetch_ready", "prefetch_skipped_empty",
    "injection_used", "injection_new", "injection_skipped_no_valid",
    "prefetch_copy_ms_sum", "prefetch_copy_ms_count", "prefetch_not_ready_checks", "main_waited_for_prefetch",
    "triton_decode_calls", "triton_prefill_fallback",
)


def _no_hook(name, phase):
    return None


class _RingView:
    """Read-only view of one cold ring in age order (the reference's cpu_*_ring deques)."""

    def __init__(self, ctrl: "KVController", li: int, b: int, field: str):
        self.c, self.li, self.b, self.field = ctrl, li, b, field

    def __len__(self):
        return int(self.c.arenas[self.li].cold_count[self.b])

    def __getitem__(self, i):
        a = self.c.arenas[self.li]
        n = len(self)
        if i < 0:
            i += n
        if not 0 <= i < n:
            raise IndexError(i)
        slot = int(a.cold_order(self.b)[i])
        if self.field == "kpre":
            return a.cold_kpre[self.b, slot]
        if self.field == "v":
            return a.cold_v[self.b, slot]
        return int(a.cold_pos[self.b, slot])


class _IndexView:
    """The reference's per-(layer, sequence) FAISS index, reduced to ntotal."""

    def __init__(self, ctrl, li, b):
        self.c, self.li, self.b = ctrl, li, b

    @property
    def ntotal(self):
        return int(self.c.arenas[self.li].cold_count[self.b])


class KVController:
    def __init__(
        self,
        max_capacity_prompt: int = 128,
        topk_ratio: float = 0.15,
        recent_size: int = 32,
        cpu_buffer_size: int = 8192,
        faiss_dim: int = 64,
        normalize_for_ip: bool = True,
        window_size: int = 16,
        query_pool_size: int = 4,
        lookahead_k: int = 32,
        hold_retrieved: bool = False,
        retrieve_after_prefill: bool = False,
        enable_asserts: bool = True,
        profile_overlap: bool = True,
        force_wait_for_prefetch_diagnostic: bool = False,
        *,
        policy: str = "hotcold",
        pool_kernel: int = 7,
        pooling: str = "maxpool",
        overflow_nan: bool = True,
        cold_payload: str = "device",
        async_retrieval: bool = False,
    ):
        """Reference arguments (controller.py:15-34) plus:
        policy: "hotcold" (cache.py:37-128) or "snapkv" (SnapKV score, scoring.py:50-132,
            with recent_size as the observation/recent window);
        pool_kernel, pooling: SnapKV pooling (scoring.py:40-47);
        overflow_nan: reproduce the reference kernel's NaN on fp32 exp overflow;
        cold_payload: "device" (HBM) or "host": the cold rings' pre-RoPE keys and values in
            page-locked host RAM that the kernels read and write directly, the reference's CPU
            cold tier (docs/design.md:59-64) for stores larger than HBM; the index stays in HBM;
        async_retrieval: a decode-step search runs on a side stream after that step's
            compression, while the following layers decode, and is attended from the layer's
            next step (the reference's worker thread, controller.py:314-342, in one of its
            orders); False searches before the step and attends the hits at once."""
        if policy not in ("hotcold", "snapkv"):
            raise ValueError(f"unknown policy {policy!r}")
        if pooling not in ("maxpool", "avgpool"):
            raise ValueError(f"unknown pooling {pooling!r}")
        self.max_capacity_prompt = int(max_capacity_prompt)
        self.topk_ratio = float(topk_ratio)
        self.recent_size = int(recent_size)
        self.cpu_buffer_size = int(cpu_buffer_size)
        self.faiss_dim = int(faiss_dim)
        self.normalize_for_ip = bool(normalize_for_ip)
        self.window_size = int(window_size)
        self.query_pool_size = int(query_pool_size)
        self.lookahead_k = int(lookahead_k)
        self.hold_retrieved = bool(hold_retrieved)
        self.retrieve_after_prefill = bool(retrieve_after_prefill)
        self.enable_asserts = bool(enable_asserts)
        self.profile_overlap = bool(profile_overlap)
        self.force_wait_for_prefetch_diagnostic = bool(force_wait_for_prefetch_diagnostic)
        self.policy, self.pool_kernel, self.pooling = policy, int(pool_kernel), pooling
        self.overflow_nan = bool(overflow_nan)
        if cold_payload not in ("device", "host"):
            raise ValueError(f"cold_payload must be 'device' or 'host', not {cold_payload!r}")
        self.cold_payload = cold_payload
        self.async_retrieval = bool(async_retrieval)
        self._pending: List[Optional[torch.cuda.Event]] = []  # per layer: its search on a side stream
        self._side = None  # [(stream, workspace)] of the side streams, made on first use
        self._events = None  # per layer: (fork, done) events of its searches on a side stream
        self._n_pending = 0

        self._inited = False
        self.B = self.Hk = self.D = self.n_layers = None
        self.step_count: List[int] = []
        self.arenas: List[Optional[LayerArena]] = []
        self._qpool: List[deque] = []
        self._prompt_qsum: List[Optional[torch.Tensor]] = []
        self._staged: List[bool] = []
        self._held_active: List[bool] = []
        self._retrieval_ready_cpu: List[Optional[tuple]] = []
        self.last_injected_len = 0
        self.workspace: Optional[Workspace] = None
        self.rotary = None  # (inv_freq tensor, attention_scaling); else the active rotary module
        # optional callable(op_name, "begin"|"end") around each op of decode_layer (timing probes)
        self.op_hook = None
        # decode steps without a search run as one fused launch (hc_step) when the layer fits
        self.fused_step = True
        # ragged batches: per-sequence budgets and cold capacities (set_ragged), else the
        # scalar settings above apply to every sequence
        self.seq_budgets = None
        self.seq_ccaps = None
        self._tails: List[dict] = []
        # a shard.ShardedColdSearch: cold searches scan only this rank's token range and merge
        # the ranks' candidates (every rank runs the same decode); None = search the whole ring
        self._cold_search = None
        self.dbg = {k: (0.0 if k == "prefetch_copy_ms_sum" else 0) for k in DBG_KEYS}

    @property
    def cold_search(self):
        return self._cold_search

    @cold_search.setter
    def cold_search(self, searcher):
        """Attach a shard.ShardedColdSearch (or None). Its limits on the top k are checked here,
        against lookahead_k, instead of at the first retrieval deep in a decode."""
        if searcher is not None and self.lookahead_k > 0:
            searcher.check_k(self.lookahead_k)
        self._cold_search = searcher

    # ------------------------------------------------------------------ setup
    def _lazy_init(self, k_pre: torch.Tensor, n_layers: int):
        """controller.py:124-158: geometry and per-layer state; device buffers follow on the
        first forward of each layer."""
        if self._inited:
            return
        B, Hk, _, D = k_pre.shape
        self._init_dims(int(B), int(Hk), int(D), int(n_layers), k_pre.device)

    def _init_dims(self, B: int, Hk: int, D: int, n_layers: int, device):
        self.B, self.Hk, self.D, self.n_layers = B, Hk, D, n_layers
        L = self.n_layers
        self.step_count = [0] * L
        self.arenas = [None] * L
        self._qpool = [deque(maxlen=max(self.query_pool_size, 1)) for _ in range(L)]
        self._prompt_qsum = [None] * L
        self._staged = [False] * L
        self._held_active = [False] * L
        self._retrieval_ready_cpu = [None] * L
        self._tails = [dict() for _ in range(L)]
        self._seen = [0] * L  # tokens each layer has processed (prompt + decode steps)
        self._pending = [None] * L
        self._n_pending = 0
        self._side = self._events = None
        self.workspace = Workspace(device)
        self._inited = True

    def set_ragged(self, budgets, ccaps, Hk: int, D: int, n_layers: int, device):
        """A ragged batch of len(budgets) independent sequences with their own budgets and cold
        ring capacities. Each sequence's prompt goes through prefill_sequence (any length),
        then finish_prefill per layer; decode_layer then steps all of them at once."""
        if self._inited:
            raise RuntimeError("set_ragged must come before the first forward")
        if self.query_pool_size >= self.window_size:
            raise ValueError("ragged prompts need query_pool_size < window_size (prompt queries stay out of the pool)")
        if len(budgets) != len(ccaps):
            raise ValueError("one budget and one cold capacity per sequence")
        self.seq_budgets = [int(b) for b in budgets]
        self.seq_ccaps = [int(c) for c in ccaps]
        self._init_dims(len(budgets), int(Hk), int(D), int(n_layers), device)

    def set_rotary(self, inv_freq: torch.Tensor, attention_scaling: float = 1.0):
        """Rotary parameters for re-rotating retrieved keys (instead of the active module)."""
        self.rotary = (inv_freq, float(attention_scaling))

    def _rotary_params(self):
        if self.rotary is not None:
            return self.rotary
        from . import patch
        rot = patch.ACTIVE_ROTARY_EMB
        if rot is None:
            raise RuntimeError("ACTIVE_ROTARY_EMB is None. Call set_active_rotary_emb(model.model.rotary_emb).")
        return rot.inv_freq, float(getattr(rot, "attention_scaling", 1.0))

    def arena(self, layer_idx: int, Hq: int, dtype, device) -> LayerArena:
        li = int(layer_idx)
        a = self.arenas[li]
        if a is None:
            inv_freq, sc = self._rotary_params()
            a = LayerArena(n_seq=self.B, Hq=int(Hq), Hk=self.Hk, D=self.D, F=self.faiss_dim, dtype=dtype,
                           device=device, budgets=self.seq_budgets or self.max_capacity_prompt,
                           r_max=max(self.lookahead_k, 0), ccap=self.seq_ccaps or self.cpu_buffer_size,
                           p_max=max(self.query_pool_size, 1), policy=self.policy,
                           recent=self.recent_size, topk_ratio=self.topk_ratio, pool_kernel=self.pool_kernel,
                           pooling=self.pooling, normalize=self.normalize_for_ip, inv_freq=inv_freq,
                           rope_scaling=sc, workspace=self.workspace, cold_payload=self.cold_payload,
                           hot_cap_hint=None if max(self.seq_budgets or [self.max_capacity_prompt]) < (1 << 16)
                           else 4096)
            self.arenas[li] = a
        return a

    def seen_tokens(self, layer_idx: int) -> int:
        """Tokens layer `layer_idx` has processed so far (the next token's absolute position when
        positions start at 0); the hot tier's physical length is shorter once compressed."""
        return self._seen[int(layer_idx)] if self._inited else 0

    # ------------------------------------------------------------------ cold store
    def cold_size(self, layer_idx: int) -> int:
        if not self._inited or self.arenas[int(layer_idx)] is None:
            return 0
        return int(self.arenas[int(layer_idx)].cold_count.sum())

    def _count_eviction(self, ev: np.ndarray, totals=None):
        """dbg counters of one compression; `totals` = (evicted, evicted capped by the cold
        capacities) when the caller has them."""
        if totals is not None:
            tot, capped = totals
            if tot:
                self.dbg["compress_calls"] += 1
                self.dbg["evicted_tokens"] += tot
                self.dbg["faiss_add"] += capped
            return
        if int(ev.max(initial=0)) > 0:
            self.dbg["compress_calls"] += 1
            self.dbg["evicted_tokens"] += int(ev.sum())
            self.dbg["faiss_add"] += int(np.minimum(ev, self.seq_ccaps or self.cpu_buffer_size).sum())

    def add_evicted_to_cold_store(self, layer_idx: int, ev: EvictedKV):
        """controller.py:190-238: append evicted tokens (host or device tensors) to the
        layer's cold rings; tokens whose evicted_idx is negative are skipped."""
        if not self._inited:
            raise RuntimeError("KVController not initialized")
        li = int(layer_idx)
        a = self.arenas[li]
        if a is None:
            dev = ev.k_pre_cpu.device if ev.k_pre_cpu.is_cuda else self.workspace.device
            a = self.arena(li, self.Hk, ev.k_pre_cpu.dtype if ev.k_pre_cpu.is_floating_point() else torch.float32,
                           dev)
        kp = ev.k_pre_cpu.to(device=a.device, dtype=a.dtype)
        vv = ev.v_cpu.to(device=a.device, dtype=a.dtype)
        m = a.cold_append(kp, vv, ev.pos_cpu, ev.evicted_idx)
        self.dbg["faiss_add"] += int(np.minimum(m, self.seq_ccaps or self.cpu_buffer_size).sum())

    @property
    def cpu_kpre_ring(self):
        return [[_RingView(self, li, b, "kpre") for b in range(self.B)] for li in range(self.n_layers or 0)]

    @property
    def cpu_v_ring(self):
        return [[_RingView(self, li, b, "v") for b in range(self.B)] for li in range(self.n_layers or 0)]

    @property
    def cpu_pos_ring(self):
        return [[_RingView(self, li, b, "pos") for b in range(self.B)] for li in range(self.n_layers or 0)]

    @property
    def index(self):
        return [[_IndexView(self, li, b) for b in range(self.B)] for li in range(self.n_layers or 0)]

    # ------------------------------------------------------------------ vectors (host helpers)
    def _pad_or_crop(self, x: torch.Tensor, dim: int) -> torch.Tensor:
        if x.shape[-1] > dim:
            return x[..., :dim]
        if x.shape[-1] < dim:
            return F.pad(x, (0, dim - x.shape[-1]))
        return x

    def _normalize(self, x: torch.Tensor, dim: int = -1) -> torch.Tensor:
        return F.normalize(x, dim=dim) if self.normalize_for_ip else x

    def _k_token_to_vec_np(self, kpre_token: torch.Tensor) -> np.ndarray:
        """controller.py:178-182 (host helper): head-mean, pad/crop, normalise."""
        v = kpre_token.detach().float().cpu().mean(dim=0)
        v = self._normalize(self._pad_or_crop(v, self.faiss_dim), dim=0)
        return v.numpy().astype("float32", copy=False)

    def _q_to_vecs_np(self, q_pre: torch.Tensor) -> np.ndarray:
        """controller.py:184-188 (host helper)."""
        q = q_pre.detach().mean(dim=1).mean(dim=1)
        q = self._normalize(self._pad_or_crop(q, self.faiss_dim), dim=-1)
        return q.float().cpu().numpy().astype("float32", copy=False)

    # ------------------------------------------------------------------ query pool and retrieval
    def update_query_window(self, layer_idx: int, q_pre: torch.Tensor):
        """controller.py:240-241: push a (B,Hq,T,D) pre-RoPE query into the pool. The decode
        path pushes inside its append kernel; this entry serves direct callers."""
        li = int(layer_idx)
        a = self.arena(li, q_pre.shape[1], q_pre.dtype, q_pre.device)
        T = int(q_pre.shape[2])
        if T == 1:
            m = q_pre.detach().mean(dim=1)[:, 0]  # (B,D), model dtype
            head = a.st[:, 6].long()
            a.qwin[torch.arange(a.n_seq, device=a.device), head] = m.to(a.dtype)
            a.st[:, 6] = ((head + 1) % a.p_max).to(torch.int32)
            self._qpool[li].append(1)
        else:
            self._prompt_qsum[li] = a.prompt_query_sum(q_pre)
            self._qpool[li].append(("prompt", T))

    def _pool(self, li: int):
        n_pool, extra_n = 0, 0
        for e in self._qpool[li]:
            if isinstance(e, tuple):
                extra_n = e[1]
            else:
                n_pool += 1
        return n_pool, (self._prompt_qsum[li] if extra_n else None), extra_n

    def _retrieve(self, li: int, side: bool = False, **kw):
        a = self.arenas[li]
        if side:
            # on a side stream, after everything this stream has launched; the layer's next
            # step waits for it (_wait_search). A sharded search's collective runs there too:
            # every rank launches its layers, hence their searches, in the same order
            stream, ws = self._side_stream(li, a.device)
            fork, done = self._events[li]
            fork.record(torch.cuda.current_stream(a.device))
            stream.wait_event(fork)
            if self.cold_search is not None:
                with torch.cuda.stream(stream):
                    a.retrieve_sharded(self.cold_search, ws=ws, **kw)
            else:
                a.retrieve(ws=ws, stream=stream, **kw)
            done.record(stream)
            self._pending[li] = done
            self._n_pending += 1
        elif self.cold_search is not None:
            a.retrieve_sharded(self.cold_search, **kw)
        else:
            a.retrieve(**kw)
        self.dbg["retrieval_ready_cpu"] += 1   # some sequence has a non-empty ring: hits are valid
        self.dbg["prefetch_launched"] += 1
        self._staged[li] = True

    def _side_stream(self, li: int, device):
        """(stream, workspace) for layer li's searches in async_retrieval mode: four side
        streams taken round robin over the layers, so that searches of different layers run at
        the same time, each with its own scratch."""
        if self._side is None:
            self._side = [(torch.cuda.Stream(device=device), Workspace(device)) for _ in range(4)]
            # per layer, reused: each layer's next search comes after its last one was waited for
            self._events = [(torch.cuda.Event(), torch.cuda.Event()) for _ in range(self.n_layers)]
        return self._side[li % len(self._side)]

    def _wait_search(self, li: int):
        """The current stream waits for the search layer li launched at its previous step."""
        ev = self._pending[li] if self._n_pending else None
        if ev is not None:
            a = self.arenas[li]
            torch.cuda.current_stream(a.device).wait_event(ev)
            a._dirty = True  # its held segment was written on another stream: no early reads
            self._pending[li] = None
            self._n_pending -= 1

    def join_searches(self):
        """Make the current stream wait for every search still running on a side stream. The
        last layer's decode_layer does this every step, so a step captured as a CUDA graph
        rejoins its side streams; call it before reading a layer's held segment on the host
        between layers."""
        if self._n_pending:
            for li in range(len(self._pending)):
                self._wait_search(li)

    def launch_retrieval_now(self, layer_idx: int, q_pre: torch.Tensor):
        """controller.py:295-312: one retrieval from the given pre-RoPE queries
        (B,Hq,P,D), used at the end of the prompt."""
        if self.lookahead_k <= 0 or not self._inited:
            return
        li = int(layer_idx)
        if self.cold_size(li) == 0:
            self.dbg["retrieval_skipped_no_cold"] += 1
            return
        self._retrieve(li, q_dense=q_pre)
        self.dbg["retrieval_launched"] += 1
        self.dbg["retrieval_launched_prefill"] += 1

    def maybe_launch_async_retrieval(self, layer_idx: int, deferred: bool = False):
        """controller.py:314-342: count the forward call; every window_size calls search
        the cold store with the pooled queries. `deferred`: called after the step's attention
        in async_retrieval mode, the search runs on a side stream."""
        if self.lookahead_k <= 0:
            return
        li = int(layer_idx)
        self.step_count[li] += 1
        if self.step_count[li] % self.window_size != 0:
            return
        if not self._inited:
            return
        if self.cold_size(li) == 0:
            self.dbg["retrieval_skipped_no_cold"] += 1
            return
        n_pool, extra, extra_n = self._pool(li)
        if n_pool == 0 and extra_n == 0:
            return
        self._retrieve(li, side=deferred, n_pool=n_pool, extra_sum=extra, extra_n=extra_n)
        self.dbg["retrieval_launched"] += 1

    def maybe_prefetch_to_gpu(self, layer_idx: int, device=None, dtype=None):
        """controller.py:344-380. The cold tier already lives in HBM and retrieval writes the
        held segment directly, so there is nothing to copy."""
        return None

    def _retrieval_worker(self, layer_idx: int, q_vecs):
        """controller.py:250-293 with given query vectors (B, faiss_dim): search, gather and
        re-rotate into the held segment; the gathered pre-RoPE pack is also kept in
        _retrieval_ready_cpu[layer_idx] as (k_pre, v, pos, valid) device tensors."""
        li = int(layer_idx)
        a = self.arenas[li]
        if a is None:
            return
        qv = torch.as_tensor(np.asarray(q_vecs, dtype=np.float32)).to(a.device).reshape(a.n_seq, self.faiss_dim)
        if self.cold_size(li) == 0:
            self._retrieval_ready_cpu[li] = None
            self.dbg["retrieval_ready_empty"] += 1
            return
        if self.cold_search is not None:
            a.retrieve_sharded(self.cold_search, qvec=qv.contiguous())
        else:
            a.retrieve(qvec=qv.contiguous())
        self._retrieval_ready_cpu[li] = self._held_pack(li)
        self._staged[li] = True
        self.dbg["retrieval_ready_cpu"] += 1

    def _held_pack(self, li: int):
        a = self.arenas[li]
        R = a.r_max
        src = a.held_src[:, :R].long()
        valid = a.held_valid[:, :R].bool()
        idx = src.clamp(min=0).to(a.cold_kpre.device)
        kpre = torch.stack([a.cold_kpre[b].index_select(0, idx[b]) for b in range(a.n_seq)], 0).to(a.device)
        vv = torch.stack([a.cold_v[b].index_select(0, idx[b]) for b in range(a.n_seq)], 0).to(a.device)
        m = valid[:, :, None, None]
        kpre = torch.where(m, kpre, torch.zeros_like(kpre)).permute(0, 2, 1, 3).contiguous()
        vv = torch.where(m, vv, torch.zeros_like(vv)).permute(0, 2, 1, 3).contiguous()
        return kpre, vv, a.held_pos[:, :R].clone(), valid

    def poll_staged_gpu(self, layer_idx: int) -> RetrievedKV:
        """controller.py:382-442: the retrieved set staged since the last poll, if any."""
        li = int(layer_idx)
        if not self._inited or not self._staged[li]:
            return RetrievedKV(k_pre=torch.empty(0), v=torch.empty(0), pos=torch.empty(0, dtype=torch.long),
                               valid=torch.empty(0, dtype=torch.bool), ready=False)
        self._staged[li] = False
        self.dbg["prefetch_ready"] += 1
        kpre, vv, pos, valid = self._held_pack(li)
        return RetrievedKV(k_pre=kpre, v=vv, pos=pos, valid=valid, ready=True)

    @property
    def held_mem(self):
        """Per layer: (k_post, v, pos, valid) of the held set while it is attended, else None
        (patch.py:252-261)."""
        out = []
        for li in range(self.n_layers or 0):
            a = self.arenas[li]
            if a is None or not self._held_active[li]:
                out.append(None)
            else:
                R = a.r_max
                out.append((a.held_k[:, :, :R], a.held_v[:, :, :R], a.held_pos[:, :R], a.held_valid[:, :R].bool()))
        return out

    # ------------------------------------------------------------------ the per-layer hot path
    def prefill_layer(self, layer_idx: int, q_pre, q_post, k_pre, k_post, v, positions):
        """The prompt forward of one layer (patch.py:159-233): query pool, schedule,
        compression of the prompt into the hot slab with eviction into the cold ring,
        and the prompt-end retrieval. Tensors (B,H,T,D); positions (B,T) int64."""
        li = int(layer_idx)
        a = self.arena(li, q_pre.shape[1], k_post.dtype, k_post.device)
        T = int(k_post.shape[2])
        if self.query_pool_size >= self.window_size:
            self.update_query_window(li, q_pre)
        self.maybe_launch_async_retrieval(li)
        r = self.recent_size
        q_obs = q_post if T <= r else q_post[:, :, -r:, :]
        ev = a.compress_prompt(q_obs, k_post, v, k_pre, positions.to(k_post.device, torch.int64))
        self._count_eviction(ev)
        self._seen[li] = T
        self.dbg["triton_prefill_fallback"] += 1
        if self.query_pool_size < self.window_size:
            # the query tail a later chunk of this prompt extends (prefill_chunk)
            self._tails[li]["chunk"] = q_pre[:, :, -self.query_pool_size:, :] if self.query_pool_size > 0 \
                else q_pre[:, :, :0, :]
        if self.retrieve_after_prefill:
            self.launch_retrieval_now(li, q_pre[:, :, -self.query_pool_size:, :])

    def prefill_chunk(self, layer_idx: int, q_pre, q_post, k_pre, k_post, v, positions, last: bool):
        """One chunk of a prompt forwarded in pieces (the reference rejects chunked prefill,
        patch.py:325-329). The chunk's tokens join the hot tier after the ones already kept;
        when the tier exceeds the budget it is compressed with the chunk's last recent_size
        post-RoPE queries as the observation window, evicting into the cold ring. The whole
        prompt counts as one forward for the retrieval schedule; after the `last` chunk the
        prompt-end retrieval uses the prompt's last query_pool_size queries. Needs
        query_pool_size < window_size. A single chunk is prefill_layer. Tensors (B,H,T_c,D);
        positions (B,T_c)."""
        li = int(layer_idx)
        if self.query_pool_size >= self.window_size:
            raise ValueError("chunked prefill needs query_pool_size < window_size")
        a = self.arena(li, q_pre.shape[1], k_post.dtype, k_post.device)
        first = int(a.n_hot.max()) == 0 and int(a.cold_count.max()) == 0
        if first:
            self.maybe_launch_async_retrieval(li)  # the prompt's forward, counted once
        r = self.recent_size
        T = int(k_post.shape[2])
        q_obs = q_post if T <= r else q_post[:, :, -r:, :]
        pos = positions.to(k_post.device, torch.int64)
        if first:
            ev = a.compress_prompt(q_obs, k_post, v, k_pre, pos)
        else:
            hk, hv, hp, hpos = a.hot_dense()
            ev = a.compress_prompt(q_obs, torch.cat([hk, k_post], 2), torch.cat([hv, v], 2),
                                   torch.cat([hp, k_pre], 2), torch.cat([hpos, pos], 1))
        self._count_eviction(ev)
        self._seen[li] += T
        self.dbg["triton_prefill_fallback"] += 1
        P = self.query_pool_size
        tail = self._tails[li].get("chunk")
        tail = q_pre if tail is None else torch.cat([tail, q_pre], 2)
        self._tails[li]["chunk"] = tail[:, :, -P:, :] if P > 0 else tail[:, :, :0, :]
        if last and self.retrieve_after_prefill:
            # the prompt's last query_pool_size queries so far (the tail is kept: a later chunk
            # of the same prompt extends it and searches again; its result replaces this one)
            self.launch_retrieval_now(li, self._tails[li]["chunk"])

    def prefill_sequence(self, layer_idx: int, b: int, q_pre, q_post, k_pre, k_post, v, positions):
        """The prompt forward of sequence b of a ragged batch (set_ragged) in one layer:
        compression of its prompt into its hot slab with eviction into its cold ring (the
        per-sequence form of prefill_layer). Tensors (1,H,T_b,D); positions (1,T_b)."""
        li, b = int(layer_idx), int(b)
        if self.seq_budgets is None:
            raise RuntimeError("prefill_sequence needs set_ragged")
        a = self.arena(li, q_pre.shape[1], k_post.dtype, k_post.device)
        T = int(k_post.shape[2])
        r = self.recent_size
        q_obs = q_post if T <= r else q_post[:, :, -r:, :]
        ev = a.compress_prompt(q_obs, k_post, v, k_pre, positions.to(k_post.device, torch.int64), seq=b)
        self._count_eviction(ev)
        self.dbg["triton_prefill_fallback"] += 1
        if self.retrieve_after_prefill:
            self._tails[li][b] = q_pre[:, :, -self.query_pool_size:, :]

    def finish_prefill(self, layer_idx: int):
        """After every sequence of a ragged batch went through prefill_sequence in this layer:
        the prompt-end retrieval of all of them in one search (patch.py:232)."""
        li = int(layer_idx)
        tails = self._tails[li]
        if self.retrieve_after_prefill and tails:
            if len(tails) != self.B or len({t.shape[2] for t in tails.values()}) != 1:
                raise ValueError("every sequence needs a prompt of at least query_pool_size tokens")
            self.launch_retrieval_now(li, torch.cat([tails[b] for b in range(self.B)], 0))
        self._tails[li] = {}

    def decode_layer(self, layer_idx: int, q_pre, k_pre, v, cos, sin, pos, out=None):
        """One decode step of one layer (patch.py:151-315): RoPE + append + query-pool push,
        scheduled retrieval into the held segment, compression with eviction, and
        attention over [held | hot]. q_pre (B,Hq,D), k_pre/v (B,Hk,D), cos/sin (B,D) in the
        model dtype or None, pos (B,) int64 on the device. Returns (B,Hq,D): `out` when given
        (a contiguous tensor of that shape and the model dtype), else the layer's own buffer."""
        li = int(layer_idx)
        a = self.arena(li, q_pre.shape[1], k_pre.dtype, k_pre.device)
        self._wait_search(li)
        self._seen[li] += 1
        hook = self.op_hook or _no_hook
        if self.fused_step:
            res = self._decode_fused(li, a, hook, q_pre, k_pre, v, cos, sin, pos, out)
            if res is not None:
                self._end_of_layer(li)
                return res
        hook("append", "begin")
        q_post = a.append(q_pre, k_pre, v, cos, sin, pos)
        hook("append", "end")
        self._qpool[li].append(1)
        if not self.async_retrieval:
            hook("retrieve", "begin")
            self.maybe_launch_async_retrieval(li)
            hook("retrieve", "end")
        hook("compress", "begin")
        ev = a.compress_decode(q_post.view(a.n_seq, a.Hq, 1, a.D))
        self._count_eviction(ev)
        hook("compress", "end")
        use_held = self._poll_use_held(li)
        self._count_injection(a, use_held)
        self.dbg["triton_decode_calls"] += 1
        hook("attend", "begin")
        res = a.attend(q_post, pos, use_held, self.overflow_nan, out=out)
        hook("attend", "end")
        if self.async_retrieval:
            self.maybe_launch_async_retrieval(li, deferred=True)
        self._end_of_layer(li)
        return res

    def _end_of_layer(self, li: int):
        """After the model's last layer: the decode stream rejoins the side streams' searches."""
        if self.async_retrieval and li == self.n_layers - 1:
            self.join_searches()

    def _decode_fused(self, li, a, hook, q_pre, k_pre, v, cos, sin, pos, out=None):
        """The decode step as one hc_step launch, preceded on search steps by one fused
        retrieval launch whose pooled query takes this step's q_pre as the newest entry (its
        query-pool push happens inside hc_step). Returns None, with nothing launched and no
        counter changed, when the fused kernels do not fit; the caller then runs the split ops."""
        fires = not self.async_retrieval and self._retrieval_fires(li)
        if fires and self.cold_search is not None:
            return None  # the sharded search runs with the split ops
        if fires:
            pool = list(self._qpool[li]) + [1]
            pool = pool[-(self._qpool[li].maxlen or len(pool)):]
            if any(isinstance(e, tuple) for e in pool) or not a.step_supported(self._poll_peek(li, True)):
                return None  # the prompt's queries are still in the pool: the split ops handle it
            hook("retrieve", "begin")
            ok = a.retrieve_decode(q_pre, len(pool) - 1)
            hook("retrieve", "end")
            if not ok:
                return None
            # the bookkeeping of maybe_launch_async_retrieval + _retrieve for a search that fired
            self.step_count[li] += 1
            self.dbg["retrieval_ready_cpu"] += 1
            self.dbg["prefetch_launched"] += 1
            self.dbg["retrieval_launched"] += 1
            self._staged[li] = True
        use_held = self._poll_use_held(li)
        hook("step", "begin")
        res = a.step(q_pre, k_pre, v, cos, sin, pos, use_held, self.overflow_nan, out=out)
        hook("step", "end")
        if res is None:
            self._undo_poll(li, use_held)
            if fires:
                raise RuntimeError("hc_step refused a layer after its retrieval ran")
            return None
        self._qpool[li].append(1)
        if not fires:
            # counts the call; in async_retrieval mode a search that fires runs on a side stream
            self.maybe_launch_async_retrieval(li, deferred=self.async_retrieval)
        o, ev = res
        self._count_eviction(ev, a.last_ev)
        self._count_injection(a, use_held)
        self.dbg["triton_decode_calls"] += 1
        return o

    def _poll_peek(self, li: int, staged_now: bool) -> bool:
        """Whether this step attends the held segment (what _poll_use_held will return),
        without changing any state."""
        if staged_now or self._staged[li]:
            return True
        return bool(self.hold_retrieved and self._held_active[li])

    def _retrieval_fires(self, li: int) -> bool:
        """Whether the next maybe_launch_async_retrieval(li) launches a search."""
        if self.lookahead_k <= 0 or (self.step_count[li] + 1) % self.window_size != 0:
            return False
        if self.cold_size(li) == 0:
            return False
        n_pool, _, extra_n = self._pool(li)
        return n_pool + 1 > 0 or extra_n > 0

    def _poll_use_held(self, li: int) -> bool:
        """patch.py:241-261: attend the retrieved set staged since the last step (and keep it
        when holding), or the held set."""
        self._poll_undo = (self._staged[li], self._held_active[li], self.dbg["prefetch_ready"],
                           self.dbg["injection_new"])
        use_held = False
        if self._staged[li]:
            self._staged[li] = False
            self.dbg["prefetch_ready"] += 1
            use_held = True
            if self.hold_retrieved:
                self._held_active[li] = True
                self.dbg["injection_new"] += 1
        elif self.hold_retrieved and self._held_active[li]:
            use_held = True
        if not self.hold_retrieved:
            self._held_active[li] = use_held
        return use_held

    def _undo_poll(self, li: int, use_held: bool):
        self._staged[li], self._held_active[li], pr, inj = self._poll_undo
        self.dbg["prefetch_ready"], self.dbg["injection_new"] = pr, inj

    def _count_injection(self, a, use_held: bool):
        self.last_injected_len = a.r_max if use_held else 0
        if use_held:
            self.dbg["injection_used"] += 1

    # ------------------------------------------------------------------ persistence
    def state_dict(self, pin: bool = True) -> dict:
        """Everything a later process needs to continue decoding from this point: every
        layer's arena (LayerArena.state_dict, host copies) and the host schedule (step
        counts, query-pool entries, staged/held flags, the prompt query sums, dbg counters).
        The result can go through torch.save. Synchronises."""
        if not self._inited:
            raise RuntimeError("KVController not initialized")
        self.join_searches()
        return {
            "dims": dict(B=self.B, Hk=self.Hk, D=self.D, n_layers=self.n_layers),
            "seq_budgets": self.seq_budgets, "seq_ccaps": self.seq_ccaps,
            "arenas": [None if a is None else a.state_dict(pin) for a in self.arenas],
            "arena_meta": [None if a is None else (a.Hq, str(a.dtype)) for a in self.arenas],
            "step_count": list(self.step_count),
            "qpool": [list(q) for q in self._qpool],
            "prompt_qsum": [None if t is None else t.cpu() for t in self._prompt_qsum],
            "staged": list(self._staged), "held_active": list(self._held_active),
            "dbg": dict(self.dbg), "last_injected_len": self.last_injected_len, "seen": list(self._seen),
        }

    def load_state_dict(self, sd: dict, device) -> None:
        """Restore a state_dict() into a controller built with the same settings (and the
        same rotary parameters) before its first forward."""
        if self._inited:
            raise RuntimeError("load_state_dict must come before the first forward")
        dm = sd["dims"]
        self.seq_budgets, self.seq_ccaps = sd["seq_budgets"], sd["seq_ccaps"]
        self._init_dims(dm["B"], dm["Hk"], dm["D"], dm["n_layers"], torch.device(device))
        dtypes = {str(t): t for t in (torch.float32, torch.float16, torch.bfloat16)}
        for li, (st, meta) in enumerate(zip(sd["arenas"], sd["arena_meta"])):
            if st is None:
                continue
            a = self.arena(li, meta[0], dtypes[meta[1]], torch.device(device))
            a.load_state_dict(st)
        self.step_count = list(sd["step_count"])
        for li, entries in enumerate(sd["qpool"]):
            self._qpool[li].clear()
            self._qpool[li].extend(tuple(e) if isinstance(e, (tuple, list)) else e for e in entries)
        self._prompt_qsum = [None if t is None else t.to(device) for t in sd["prompt_qsum"]]
        self._staged = list(sd["staged"])
        self._held_active = list(sd["held_active"])
        self.dbg = dict(sd["dbg"])
        self.last_injected_len = sd["last_injected_len"]
        self._seen = list(sd.get("seen", [0] * self.n_layers))

    def device_status(self) -> int:
        """OR of the device status words of every layer (synchronises): HC_DEV_* bits."""
        bits = 0
        for a in self.arenas:
            if a is not None:
                bits |= int(np.bitwise_or.reduce(a.st[:, 8].cpu().numpy()))
        return bits
