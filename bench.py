"""Benchmark of the per-layer decode step of the hot/cold KV path.

Workload (BASELINE configs[1] geometry): Llama-3.1-8B attention shapes (32 query /
8 KV heads, head_dim 128, fp16), 32 layers, batch 1, an 8192-token prompt per
layer compressed to a budget of 512 with the evicted tokens in the HBM cold
store, retrieval of the top 64 every 16 steps, held until replaced. The
pre-RoPE q/k/v of every layer and step are seeded N(0,1) draws resident in HBM
(no weights or dataset exist here; the hot path's cost does not depend on the
values). Default eviction policy: SnapKV scoring (window 32, max-pool 7), which
evicts one token into the cold store every decode step, so each step runs
attention + eviction + (every 16th step) cold top-k and re-RoPE inject.

One step = one decode step through all layers. Every timed step is captured as
a CUDA graph right before it is replayed (capture is outside the timed region),
L2 is flushed before each replay, and each replay is bracketed by CUDA events
on the launching stream. value = device time / layer-steps (us per layer-step,
lower is better), max over ranks at N > 1 (each rank runs its own replica).

Three more workloads (--workload); the first two also run as sub-results of the default line
("ragged", "cold_shard"; --no-partitioned skips them), so every N of a scaling run times them:
  ragged      the ragged continuous batch: 64 sequences of lengths
              uniform in [2048, 32768] with budgets cycling 512/1024/2048, one layer,
              partitioned over the N ranks by balanced token count, no collective on the
              decode path; value = us per sequence-layer-step of the whole batch.
  cold-shard  the long cold store (BASELINE configs[4] shape): a 131072-token prompt per
              layer compressed to budget 2048 (about 129k cold entries), top-256 retrieval
              from 8 query states every step, the cold index scanned by token range over the
              N ranks and the candidates merged after an NCCL all-gather; every rank runs the
              same decode. value = us per layer-step.
  prefill     SnapKV compression of one layer's prompt (window 32, max-pool 7, budget 512,
              fp16, 32/8 heads) with eviction of the rest into the cold ring: the prompt-side
              use of the scoring kernels (tcgen05 observation x prefix product). value = us per
              prompt-layer; also the scoring's algorithmic TFLOP/s.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                       [--workload decode|ragged|cold-shard|prefill]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-step µs/layer (attn+evict+cold top-k) at 8k ctx; HBM GB/s vs peak"
UNIT = "us/layer-step"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--policy", default="snapkv", choices=["snapkv", "hotcold"])
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--prompt", type=int, default=None, help="default 8192 (decode), 131072 (cold-shard)")
    p.add_argument("--budget", type=int, default=None, help="default 512 (decode), 2048 (cold-shard)")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--cpu-steps", type=int, default=16)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", default="decode", choices=["decode", "ragged", "cold-shard", "prefill", "model"])
    p.add_argument("--seqs", type=int, default=64)
    p.add_argument("--retrieval", default="async", choices=["sync", "async"],
                   help="decode-step searches in the decode stream before the step (sync), or on side "
                        "streams after it, attended from the next step (async: KVController(async_retrieval=True))")
    p.add_argument("--no-partitioned", action="store_true",
                   help="skip the ragged-batch and sharded-cold-store sub-results of the default line")
    return p.parse_args()


def config(a):
    recent = 32 if a.policy == "snapkv" else 128
    ratio = 0.0 if a.policy == "snapkv" else max(0.05, 0.75 - recent / (a.budget or 512))  # run_baselines.py:86-87
    return dict(Hq=32, Hk=8, D=128, theta=500000.0, layers=a.layers, prompt=a.prompt or 8192, budget=a.budget or 512,
                policy=a.policy, recent=recent, topk_ratio=ratio, pool_kernel=7, ccap=32768, faiss_dim=128,
                window_size=16, query_pool_size=4, lookahead_k=64, hold=True, dtype="float16",
                async_retrieval=getattr(a, "retrieval", "async") == "async")


def workload_config(c, extra=None):
    d = {"workload": "llama3.1-8b-geometry hot/cold decode step, 32 layers, 8k prompt, budget 512",
         "layers": c["layers"], "prompt_tokens": c["prompt"], "budget": c["budget"], "policy": c["policy"],
         "recent": c["recent"], "lookahead_k": c["lookahead_k"], "retrieval_every": c["window_size"],
         "hold_retrieved": c["hold"], "cold_ring": c["ccap"], "batch": 1, "heads": "32q/8kv", "head_dim": 128,
         "retrieval": ("async: side streams after the step, attended from the next step" if c.get("async_retrieval")
                       else "sync: in the decode stream before the step, attended at once"),
         "l2": "flushed (256 MiB write) before every timed step"}
    if extra:
        d.update(extra)
    return d


# ------------------------------------------------------------------------------------------
# clocks
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.gpu_id is not None:
            cmd += ["-i", str(self.gpu_id)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(", ") for r in self.lines if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def source_sha(name: str) -> str:
    """First 12 hex digits of the SHA-1 of a kernel source file (csrc/<name>)."""
    import hashlib
    with open(os.path.join(ROOT, "hotcold_kv_cache_b200", "csrc", name), "rb") as f:
        return hashlib.sha1(f.read()).hexdigest()[:12]


def profiled_traffic(kernel: str, source: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary (profiles/traffic.txt),
    with where it comes from. DRAM counters cannot be read inside this run, so the figure is
    the one ncu measured; it is withheld (None) when the kernel's source file changed since
    that capture (the summary records the file's SHA-1)."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    val = sha = None
    try:
        for line in open(path):
            if line.startswith(f"traffic[{kernel}]"):
                val = int(float(line.split("=", 1)[1].split()[0]))
            elif line.startswith(f"source_sha[{kernel}]"):
                sha = line.split("=", 1)[1].strip()
    except OSError:
        return None, "no ncu summary"
    now = source_sha(source)
    if val is None:
        return None, "no ncu figure for this kernel"
    if sha != now:
        return None, f"stale: {source} changed since the ncu capture (sha {sha} vs {now})"
    return val, f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, profiles/traffic.txt ({source} sha {now})"


# ------------------------------------------------------------------------------------------
# CUDA runtime helpers (graph upload, event nodes recorded inside a capture)
# ------------------------------------------------------------------------------------------
_RT = None


def _rt():
    global _RT
    if _RT is None:
        import ctypes
        rt = ctypes.CDLL("libcudart.so.12")
        rt.cudaGraphUpload.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        rt.cudaEventCreate.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
        rt.cudaEventRecordWithFlags.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint]
        rt.cudaEventElapsedTime.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_void_p, ctypes.c_void_p]
        rt.cudaEventDestroy.argtypes = [ctypes.c_void_p]
        _RT = rt
    return _RT


def _handle(x) -> int:
    import ctypes
    if isinstance(x, int):
        return x
    try:
        return int(x)
    except TypeError:
        get = ctypes.pythonapi.PyCapsule_GetPointer
        get.restype, get.argtypes = ctypes.c_void_p, [ctypes.py_object, ctypes.c_char_p]
        return get(x, None)


def graph_upload(g, stream) -> None:
    """Upload an instantiated graph so that its first launch does not pay for it."""
    rc = _rt().cudaGraphUpload(_handle(g.raw_cuda_graph_exec()), stream.cuda_stream)
    if rc != 0:
        raise RuntimeError(f"cudaGraphUpload failed ({rc})")


class EventPool:
    """Events recorded as graph nodes (cudaEventRecordExternal) during a capture."""

    def __init__(self):
        import ctypes
        self.ct = ctypes
        self.events = []

    def record(self, stream_handle: int):
        ev = self.ct.c_void_p()
        if _rt().cudaEventCreate(self.ct.byref(ev)) != 0:
            raise RuntimeError("cudaEventCreate failed")
        if _rt().cudaEventRecordWithFlags(ev, self.ct.c_void_p(stream_handle), 1) != 0:
            raise RuntimeError("cudaEventRecordWithFlags failed")
        self.events.append(ev)
        return ev

    def elapsed_us(self, a, b) -> float:
        ms = self.ct.c_float()
        if _rt().cudaEventElapsedTime(self.ct.byref(ms), a, b) != 0:
            raise RuntimeError("cudaEventElapsedTime failed")
        return ms.value * 1e3

    def close(self):
        for ev in self.events:
            _rt().cudaEventDestroy(ev)
        self.events = []


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------
class Workload:
    """32 layers of prompt + decode inputs in HBM and the controller holding their state."""

    def __init__(self, c, steps, seed, device):
        import torch
        from transformers import LlamaConfig
        from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, apply_rotary_pos_emb

        from hotcold_kv_cache_b200 import KVController
        self.torch = torch
        self.c, self.dev = c, device
        L, T, Hq, Hk, D = c["layers"], c["prompt"], c["Hq"], c["Hk"], c["D"]
        dt = torch.float16
        g = torch.Generator(device=device).manual_seed(seed)
        cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hk, head_dim=D,
                          num_hidden_layers=L, rope_theta=c["theta"], vocab_size=16, intermediate_size=16,
                          max_position_embeddings=1 << 17)
        self.rot = LlamaRotaryEmbedding(cfg).to(device)
        self.ctrl = KVController(max_capacity_prompt=c["budget"], topk_ratio=c["topk_ratio"],
                                 recent_size=c["recent"], cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"],
                                 window_size=c["window_size"], query_pool_size=c["query_pool_size"],
                                 lookahead_k=c["lookahead_k"], hold_retrieved=c["hold"],
                                 retrieve_after_prefill=False, policy=c["policy"], pool_kernel=c["pool_kernel"],
                                 profile_overlap=False, async_retrieval=c.get("async_retrieval", False))
        self.ctrl.set_rotary(self.rot.inv_freq, self.rot.attention_scaling)
        pos = torch.arange(T, device=device)[None]
        cos, sin = self.rot(torch.empty(1, dtype=dt, device=device), pos)
        for li in range(L):
            q = torch.randn((1, Hq, T, D), generator=g, device=device, dtype=dt)
            k = torch.randn((1, Hk, T, D), generator=g, device=device, dtype=dt)
            v = torch.randn((1, Hk, T, D), generator=g, device=device, dtype=dt)
            if li == 0:
                self.ctrl._lazy_init(k, n_layers=L)
            qp, kp = apply_rotary_pos_emb(q, k, cos, sin)
            self.ctrl.prefill_layer(li, q, qp, k, kp, v, pos)
            del q, k, v, qp, kp
        self.n = steps
        self.dq = torch.randn((steps, L, 1, Hq, D), generator=g, device=device, dtype=dt)
        self.dk = torch.randn((steps, L, 1, Hk, D), generator=g, device=device, dtype=dt)
        self.dv = torch.randn((steps, L, 1, Hk, D), generator=g, device=device, dtype=dt)
        p = torch.arange(T, T + steps, device=device)
        cs, sn = self.rot(torch.empty(1, dtype=dt, device=device), p[None])
        self.cos, self.sin = cs[0].contiguous(), sn[0].contiguous()   # (steps, D)
        self.pos = p.view(steps, 1).contiguous()
        self.out = torch.empty((L, 1, Hq, D), dtype=dt, device=device)
        # size the shared scratch for every op now, so that no allocation happens in a capture
        from hotcold_kv_cache_b200._lib import byref, size
        a0 = self.ctrl.arenas[0]
        need = max(size("hc_attend_scratch_bytes", byref(a0.L)), size("hc_retrieve_scratch_bytes", byref(a0.L)),
                   size("hc_compress_scratch_bytes", byref(a0.L), a0.max_cap, 1))
        self.ctrl.workspace.get(need)
        if self.ctrl.async_retrieval:
            for li in range(min(L, 4)):
                self.ctrl._side_stream(li, device)[1].get(need)
        torch.cuda.synchronize(device)

    def step(self, i):
        """Decode step i through all layers (the public per-layer API). Each layer's output
        stays in its arena's output buffer."""
        c = self.c
        for li in range(c["layers"]):
            self.ctrl.decode_layer(li, self.dq[i, li], self.dk[i, li], self.dv[i, li], self.cos[i:i + 1],
                                   self.sin[i:i + 1], self.pos[i])


def kernel_launches(ctrl) -> int:
    """Kernels launched so far by the decode-path ops of every layer (each op counts its own)."""
    return sum(a.launches for a in ctrl.arenas if a is not None)


def run_ours(a, rank, world):
    import torch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    c = config(a)
    K, W = a.steps, a.warmup
    total_steps = W + K
    wl = Workload(c, total_steps + K, a.seed + rank, dev)
    ctrl = wl.ctrl
    # warm-up: eager steps (grow the workspace, fill the query pool, land a retrieval)
    for i in range(W):
        wl.step(i)
    torch.cuda.synchronize(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    times = []
    launches0 = kernel_launches(ctrl)
    gpu_id = None
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gpu_id = None
    clocks = ClockSampler(gpu_id if rank == 0 else None)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    if rank == 0:
        clocks.start()
    cur = torch.cuda.current_stream(dev)
    step_launches = []
    for i in range(W, total_steps):
        g = torch.cuda.CUDAGraph()
        la = kernel_launches(ctrl)
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                wl.step(i)
        step_launches.append(kernel_launches(ctrl) - la)
        graph_upload(g, cur)
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        g.replay()
        e1.record(cur)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        del g
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop() if rank == 0 else None
    launches = kernel_launches(ctrl) - launches0
    step_ms = float(sum(times) / len(times))
    tot = torch.tensor([sum(times)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(tot, op=torch.distributed.ReduceOp.MAX)
    max_total_ms = float(tot.item())
    layer_steps_all = world * K * c["layers"]
    value = max_total_ms * 1e3 / layer_steps_all
    status = ctrl.device_status()
    if status:
        raise RuntimeError(f"device status word set: {status}")

    # ---- per-op device time inside the captured steps (event nodes around each op) --------
    ops = per_op_live(wl, total_steps, min(K, 16), dev)

    # ---- end to end through the public API with host buffers ------------------------------
    e2e = run_e2e(wl, total_steps + 0, min(K, 8), dev)

    peak, peak_kind = measured_peaks()
    # the dominant kernel: the fused step when it runs, else the split attention
    key, kname = ("step", "step_kernel (hc_step)") if "step" in ops else ("attend", "attn_kernel (hc_attend)")
    att = ops[key]
    us_launch, timing = att["us"], "event nodes around the op inside captured steps"
    if key == "step":
        # a step without retrieval is exactly one step_kernel launch per layer: its replay time
        # per layer is the kernel's duration in the programmatic-launch chain, unperturbed by
        # event nodes
        plain = [t for t, n in zip(times, step_launches) if n == c["layers"]]
        if plain:
            us_launch = statistics.median(plain) * 1e3 / c["layers"]
            timing = f"median replay time / layers over the {len(plain)} timed steps without retrieval"
    gbs = att["bytes"] / (us_launch * 1e-6) / 1e9
    traffic, traffic_src = profiled_traffic(key, "hc_step.cu" if key == "step" else "hc_attention.cu")
    roof = {"bound": "hbm", "kernel": kname, "achieved": round(gbs, 1),
            "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
            "traffic": traffic, "traffic_source": traffic_src, "peak_source": f"{peak_kind} hbm_gbs",
            "bytes_per_launch": att["bytes"], "us_per_launch": round(us_launch, 3), "timing": timing}
    res = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
           "ms_per_step": round(step_ms, 4), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
           "dtype": "f16", "data": "synthetic N(0,1) pre-RoPE q/k/v, seeded; no weights or dataset",
           "config": workload_config(c, {"parallelism": f"replicas{world}"}),
           "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "clocks": clk,
           "ops_us_per_layer_step": {k: round(v["us"], 3) for k, v in ops.items() if not k.startswith("_")},
           "hbm_gbs_per_layer_step": round(ops["_step_bytes"] / (value * 1e-6) / 1e9, 1)}
    return res


def op_times(ctrl, step_fn, start, n, dev):
    """Device time of each op of a layer-step inside captured decode steps: event nodes
    (cudaEventRecordExternal) bracket every op of every layer, the graph is uploaded, L2 is
    flushed, the step is replayed once. Returns {op: [us of each layer-step where the op
    launched kernels]}."""
    import torch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    rec = {k: [] for k in ("step", "append", "retrieve", "compress", "attend")}
    for i in range(start, start + n):
        pool = EventPool()
        marks = []

        def hook(name, phase):
            h = torch.cuda.current_stream(dev).cuda_stream
            if phase == "begin":
                marks.append([name, pool.record(h), None, (ctrl.dbg["retrieval_launched"], ctrl.dbg["compress_calls"])])
            else:
                m = marks[-1]
                m[2] = pool.record(h)
                r0, c0 = m[3]
                m[3] = not ((name == "retrieve" and ctrl.dbg["retrieval_launched"] == r0) or
                            (name == "compress" and ctrl.dbg["compress_calls"] == c0))

        ctrl.op_hook = hook
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    step_fn(i)
        finally:
            ctrl.op_hook = None
        graph_upload(g, cur)
        flush.zero_()
        g.replay()
        torch.cuda.synchronize(dev)
        for name, a, b, launched in marks:
            if launched:
                rec[name].append(pool.elapsed_us(a, b))
        pool.close()
        del g
    return rec


def ops_median(rec):
    return {k: round(float(np.median(v)), 3) for k, v in rec.items() if v}


def per_op_live(wl, start, n, dev):
    """op_times over the decode workload, with each op's algorithmic bytes and GB/s."""
    ctrl, c = wl.ctrl, wl.c
    rec = op_times(ctrl, wl.step, start, n, dev)
    Hk, D, R, Hq = c["Hk"], c["D"], c["lookahead_k"], c["Hq"]
    a = ctrl.arenas[0]
    n_hot, n_cold = int(a.n_hot[0]), int(a.cold_count[0])
    bytes_ = {
        # fused step: K/V rows of held + hot tokens once, q/k/v in, output out, the new token's
        # three slab rows, one evicted token's payload + index vector, the logical order
        "step": float((n_hot + R) * Hk * D * 2 * 2 + (Hq + 2 * Hk) * D * 2 + Hq * D * 2 + 3 * Hk * D * 2
                      + (2 * Hk * D * 2) * 2 + c["faiss_dim"] * 4 + n_hot * 4 * 2),
        # K and V rows of the held and hot tokens, plus the query in and the output
        "attend": float((n_hot + R) * Hk * D * 2 * 2 + 2 * Hq * D * 2),
        # pre-RoPE q/k/v in, q_post out, k_post/k_pre/v into the slab
        "append": float((Hq + 2 * Hk) * D * 2 + Hq * D * 2 + 3 * Hk * D * 2),
        # post-RoPE keys scored once, one evicted token's payload + index vector
        "compress": float(n_hot * Hk * D * 2 + 2 * Hk * D * 2 * 2 + c["faiss_dim"] * 4),
        # index scan over the live ring, gather of R hits (k_pre, v), held segment written
        "retrieve": float(n_cold * c["faiss_dim"] * 4 + R * Hk * D * 2 * 4),
    }
    out = {}
    for k, v in rec.items():
        if not v:
            continue
        us = float(np.median(v))
        out[k] = {"us": us, "bytes": bytes_[k], "gbs": bytes_[k] / (us * 1e-6) / 1e9, "n": len(v)}
    step_bytes = bytes_["step"] + bytes_["retrieve"] / c["window_size"]
    out["_step_bytes"] = step_bytes
    return out


def run_e2e(wl, start, n, dev):
    """Per step: pinned host -> device copy of every layer's q/k/v, the public per-layer
    decode call for all layers, device -> host read of every layer's attention output."""
    import torch
    c = wl.c
    L = c["layers"]
    hq = wl.dq[start:start + n].cpu().pin_memory()
    hk = wl.dk[start:start + n].cpu().pin_memory()
    hv = wl.dv[start:start + n].cpu().pin_memory()
    hout = torch.empty((L, 1, c["Hq"], c["D"]), dtype=torch.float16).pin_memory()
    dq, dk, dv = torch.empty_like(wl.dq[0]), torch.empty_like(wl.dk[0]), torch.empty_like(wl.dv[0])
    # the per-layer views of the device input and output buffers, made once (a model holds its
    # per-layer activations the same way)
    views = [(li, dq[li], dk[li], dv[li], wl.out[li]) for li in range(L)]
    steps = [(wl.cos[i:i + 1], wl.sin[i:i + 1], wl.pos[i]) for i in range(start, start + n)]
    decode = wl.ctrl.decode_layer
    times = []
    for j in range(n):
        cs, sn, ps = steps[j]
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dq.copy_(hq[j], non_blocking=True)
        dk.copy_(hk[j], non_blocking=True)
        dv.copy_(hv[j], non_blocking=True)
        for li, q, k, v, o in views:
            decode(li, q, k, v, cs, sn, ps, out=o)
        hout.copy_(wl.out, non_blocking=True)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = float(np.mean(times))
    h2d = (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 2
    return {"value": round(ms * 1e3 / L, 3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(hout.numel() * 2),
            "api": "KVController.decode_layer per layer, eager, outputs written into one (layers,1,Hq,D) buffer",
            "steps": n}


# ------------------------------------------------------------------------------------------
# extra workloads: ragged batch over ranks, token-range sharded cold search
# ------------------------------------------------------------------------------------------
def _rotary(Hq, Hk, D, theta, dev):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hk, head_dim=D,
                      num_hidden_layers=1, rope_theta=theta, vocab_size=16, intermediate_size=16,
                      max_position_embeddings=1 << 18)
    return LlamaRotaryEmbedding(cfg).to(dev)


def _prefill_inputs(g, Hq, Hk, T, D, dev, rot):
    import torch
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    dt = torch.float16
    q = torch.randn((1, Hq, T, D), generator=g, device=dev, dtype=dt)
    k = torch.randn((1, Hk, T, D), generator=g, device=dev, dtype=dt)
    v = torch.randn((1, Hk, T, D), generator=g, device=dev, dtype=dt)
    pos = torch.arange(T, device=dev)[None]
    cos, sin = rot(torch.empty(1, dtype=dt, device=dev), pos)
    qp, kp = apply_rotary_pos_emb(q, k, cos, sin)
    return q, qp, k, kp, v, pos


def _timed_graph_steps(step_fn, first, K, dev, world):
    """Capture each of K steps as a CUDA graph and replay it between CUDA events after an
    L2 flush; returns (per-step ms, sum of the max over ranks)."""
    import torch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    times = []
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    for i in range(first, first + K):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                step_fn(i)
        graph_upload(g, cur)
        flush.zero_()
        if world > 1:
            # ranks capture at different host speeds: line them up outside the timed region so a
            # collective inside the step does not time the other rank's capture
            torch.cuda.synchronize(dev)
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        g.replay()
        e1.record(cur)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
        del g
    torch.cuda.synchronize(dev)
    tot = torch.tensor([sum(times)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.all_reduce(tot, op=torch.distributed.ReduceOp.MAX)
    return times, float(tot.item())


def run_ragged(a, rank, world):
    import torch
    from hotcold_kv_cache_b200 import KVController, synth
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    Hq, Hk, D = 32, 8, 128
    items = synth.ragged_batch(a.seed, a.seqs)
    mine = synth.balanced_partition(items, world)[rank]
    n = len(mine)
    rot = _rotary(Hq, Hk, D, 500000.0, dev)
    ctrl = KVController(max_capacity_prompt=2048, topk_ratio=0.0, recent_size=32, cpu_buffer_size=32768,
                        faiss_dim=128, window_size=1 << 20, query_pool_size=8, lookahead_k=64, hold_retrieved=True,
                        retrieve_after_prefill=True, policy="snapkv", pool_kernel=7, profile_overlap=False)
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    ctrl.set_ragged([items[i][1] for i in mine], [items[i][0] for i in mine], Hk, D, 1, dev)
    for b, i in enumerate(mine):
        g = torch.Generator(device=dev).manual_seed(a.seed * 1000 + i)
        q, qp, k, kp, v, pos = _prefill_inputs(g, Hq, Hk, items[i][0], D, dev, rot)
        ctrl.prefill_sequence(0, b, q, qp, k, kp, v, pos)
        del q, qp, k, kp, v
    ctrl.finish_prefill(0)
    K, W = a.steps, a.warmup
    g = torch.Generator(device=dev).manual_seed(a.seed + 7 + rank)
    dq = torch.randn((W + K, n, Hq, D), generator=g, device=dev, dtype=torch.float16)
    dk = torch.randn((W + K, n, Hk, D), generator=g, device=dev, dtype=torch.float16)
    dv = torch.randn((W + K, n, Hk, D), generator=g, device=dev, dtype=torch.float16)
    lens = torch.tensor([items[i][0] for i in mine], device=dev)
    pos = torch.stack([lens + i for i in range(W + K)], 0).contiguous()  # (steps, n)
    cs, sn = rot(torch.empty(1, dtype=torch.float16, device=dev), pos)
    cs, sn = cs.contiguous(), sn.contiguous()

    def step(i):
        ctrl.decode_layer(0, dq[i], dk[i], dv[i], cs[i], sn[i], pos[i])

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    a0 = ctrl.arenas[0]
    l0 = a0.launches
    times, max_total = _timed_graph_steps(step, W, K, dev, world)
    launches = a0.launches - l0
    ops = ops_median(op_times(ctrl, step, W + K - 2, 2, dev)) if K >= 2 else {}
    if ctrl.device_status():
        raise RuntimeError("device status word set")
    units = len(items) * K
    value = max_total * 1e3 / units
    # per sequence-layer-step: K/V of the held + hot tokens, the eviction's key scan and payload
    hot = np.asarray(a0.n_hot, np.float64)
    byts = float(((hot + a0.r_max) * Hk * D * 2 * 2 + hot * Hk * D * 2 + 2 * Hk * D * 2 * 2).sum())
    tot_b = torch.tensor([byts], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(tot_b)
    gbs = float(tot_b.item()) * K / (max_total * 1e-3) / 1e9
    return {"metric": "ragged batch decode: us per sequence-layer-step (64 seqs, attn+evict)", "value": round(value, 3),
            "unit": "us/sequence-layer-step", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(max_total / K, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,1) pre-RoPE q/k/v, seeded per sequence",
            "config": {"workload": "ragged batch: 64 sequences, lengths U[2048,32768], budgets 512/1024/2048, 1 layer",
                       "seqs_this_rank": n, "tokens_this_rank": int(sum(items[i][0] for i in mine)),
                       "partition": "balanced token count (LPT)", "parallelism": f"sequences over {world} ranks",
                       "l2": "flushed before every timed step"},
            "aggregate_hbm_gbs": round(gbs, 1), "gpu_launches": int(launches), "ops_us_per_step": ops}


def run_cold_shard(a, rank, world):
    import torch
    from hotcold_kv_cache_b200 import KVController
    from hotcold_kv_cache_b200.shard import ShardedColdSearch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    Hq, Hk, D = 32, 8, 128
    T, budget, R, layers = a.prompt or 131072, a.budget or 2048, 256, a.layers
    rot = _rotary(Hq, Hk, D, 500000.0, dev)
    ctrl = KVController(max_capacity_prompt=budget, topk_ratio=0.0, recent_size=32, cpu_buffer_size=T + 1024,
                        faiss_dim=128, window_size=1, query_pool_size=8, lookahead_k=R, hold_retrieved=True,
                        retrieve_after_prefill=False, policy="snapkv", pool_kernel=7, profile_overlap=False,
                        async_retrieval=getattr(a, "retrieval", "async") == "async")
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    ctrl.cold_search = ShardedColdSearch()
    g = torch.Generator(device=dev).manual_seed(a.seed)  # the same draws on every rank: replicas
    for li in range(layers):
        q, qp, k, kp, v, pos = _prefill_inputs(g, Hq, Hk, T, D, dev, rot)
        if li == 0:
            ctrl._lazy_init(k, n_layers=layers)
        ctrl.prefill_layer(li, q, qp, k, kp, v, pos)
        del q, qp, k, kp, v
    K, W = a.steps, a.warmup
    dq = torch.randn((W + K, layers, 1, Hq, D), generator=g, device=dev, dtype=torch.float16)
    dk = torch.randn((W + K, layers, 1, Hk, D), generator=g, device=dev, dtype=torch.float16)
    dv = torch.randn((W + K, layers, 1, Hk, D), generator=g, device=dev, dtype=torch.float16)
    p = torch.arange(T, T + W + K, device=dev)
    cs, sn = rot(torch.empty(1, dtype=torch.float16, device=dev), p[None])
    cs, sn = cs[0].contiguous(), sn[0].contiguous()
    pos = p.view(-1, 1).contiguous()

    def step(i):
        for li in range(layers):
            ctrl.decode_layer(li, dq[i, li], dk[i, li], dv[i, li], cs[i:i + 1], sn[i:i + 1], pos[i])

    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    l0 = sum(x.launches for x in ctrl.arenas)
    times, max_total = _timed_graph_steps(step, W, K, dev, world)
    launches = sum(x.launches for x in ctrl.arenas) - l0
    ops = ops_median(op_times(ctrl, step, W + K - 2, 2, dev)) if K >= 2 else {}
    if ctrl.device_status():
        raise RuntimeError("device status word set")
    a0 = ctrl.arenas[0]
    n_cold = int(a0.cold_count[0])
    value = max_total * 1e3 / (K * layers)
    return {"metric": "sharded cold store decode: us per layer-step (attn+evict+top-256 search every step)",
            "value": round(value, 3), "unit": "us/layer-step", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(max_total / K, 4), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,1) pre-RoPE q/k/v, seeded",
            "config": {"workload": f"cold-store sharding: {layers} layer(s), {T}-token prompt, budget {budget}, "
                                   f"top-{R} every step from 8 queries", "cold_entries_per_layer": n_cold,
                       "index_rows_scanned_per_rank": -(-n_cold // world),
                       "parallelism": f"cold index by token range over {world} ranks, NCCL all-gather of "
                                      f"{world}x{R} candidates, decode replicated",
                       "retrieval": ("async: side streams after the step, attended from the next step"
                                     if ctrl.async_retrieval else "sync: before the step, attended at once"),
                       "l2": "flushed before every timed step"},
            "gpu_launches": int(launches), "ops_us_per_layer_step": ops}


def run_model(a, rank, world):
    """BASELINE configs[1] end to end through the reference-facing entry point: a random-init
    32-layer Llama-3.1-8B in fp16, install_monkeypatch + build_hotcold_cache, an 8192-token
    uniform-random prompt, budget 512 (SnapKV, window 32, max-pool 7), top-64 retrieval every 16
    steps, held; teacher-forced decode of uniform-random tokens. Per decode token: the eager call
    a user makes (CUDA events around model(...)), and the device time of the same step captured
    as a CUDA graph (the host's Python out of the picture). Each rank runs its own replica."""
    import torch
    import hotcold_kv_cache_b200 as hc
    from hotcold_kv_cache_b200 import synth
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    model = synth.llama8b_random(dev, seed=a.seed + rank)
    T, K, W = a.prompt or 8192, a.steps, a.warmup
    ctrl = hc.KVController(max_capacity_prompt=a.budget or 512, topk_ratio=0.0, recent_size=32,
                           cpu_buffer_size=32768, faiss_dim=128, window_size=16, query_pool_size=4, lookahead_k=64,
                           hold_retrieved=True, retrieve_after_prefill=False, policy="snapkv", pool_kernel=7,
                           profile_overlap=False)
    g = torch.Generator().manual_seed(a.seed + 100 + rank)
    n = W + 2 * K
    ids = torch.randint(0, model.config.vocab_size, (1, T + n), generator=g).to(dev)
    hc.uninstall_monkeypatch()
    hc.set_active_rotary_emb(model.model.rotary_emb)
    hc.install_monkeypatch(enable_debug=False)
    hc.set_active_kvctrl(ctrl)
    try:
        cache = hc.build_hotcold_cache(model, ctrl)
        with torch.inference_mode():
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            model(input_ids=ids[:, :T], use_cache=True, past_key_values=cache, logits_to_keep=1)
            e1.record()
            e1.synchronize()
            prefill_ms = e0.elapsed_time(e1)

            def step(i):
                return model(input_ids=ids[:, T + i:T + i + 1], cache_position=torch.arange(T + i, T + i + 1, device=dev),
                             past_key_values=cache, use_cache=True, logits_to_keep=1).logits

            for i in range(W):
                step(i)
            torch.cuda.synchronize(dev)
            eager = []
            for i in range(W, W + K):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                lg = step(i)
                tok = lg[0, -1].argmax().item()  # the token a generation loop would read back
                e1.record()
                e1.synchronize()
                eager.append(e0.elapsed_time(e1))
            stream = torch.cuda.Stream(dev)
            flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
            graphed = []
            for i in range(W + K, W + 2 * K):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(gr, stream=stream):
                        step(i)
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                gr.replay()
                e1.record()
                e1.synchronize()
                graphed.append(e0.elapsed_time(e1))
                del gr
        if ctrl.device_status():
            raise RuntimeError("device status word set")
        del tok
    finally:
        hc.uninstall_monkeypatch()
        hc.set_active_kvctrl(None)
    eg, gp = statistics.median(eager), statistics.median(graphed)
    res = {"metric": "decode ms per token through the patched Llama-3.1-8B forward (32 layers, random init)",
           "value": round(eg, 3), "unit": "ms/token", "higher_is_better": False, "scaling": "weak",
           "steps": K, "warmup": W, "graph_ms_per_token": round(gp, 3), "prefill_ms": round(prefill_ms, 1),
           "config": {"workload": f"random-init Llama-3.1-8B fp16, {T}-token prompt, budget {a.budget or 512}, "
                                  "top-64 every 16 steps, held, SnapKV", "api": "install_monkeypatch + "
                                  "build_hotcold_cache + model(...) per token; argmax read back per token (eager)",
                      "graph": "the same decode step captured as a CUDA graph, L2 flushed before each replay"}}
    del model, cache, ctrl
    return res


def run_prefill(a, rank, world):
    import torch
    from hotcold_kv_cache_b200 import KVController
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    Hq, Hk, D, W = 32, 8, 128, 32
    T, budget = a.prompt or 8192, a.budget or 512
    rot = _rotary(Hq, Hk, D, 500000.0, dev)
    ctrl = KVController(max_capacity_prompt=budget, topk_ratio=0.0, recent_size=W, cpu_buffer_size=T,
                        faiss_dim=128, window_size=1 << 20, query_pool_size=8, lookahead_k=64, hold_retrieved=True,
                        retrieve_after_prefill=False, policy="snapkv", pool_kernel=7, profile_overlap=False)
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    g = torch.Generator(device=dev).manual_seed(a.seed + rank)
    q, qp, k, kp, v, pos = _prefill_inputs(g, Hq, Hk, T, D, dev, rot)
    ctrl._lazy_init(k, n_layers=1)
    ctrl.prefill_layer(0, q, qp, k, kp, v, pos)
    ar = ctrl.arenas[0]
    q_obs = qp[:, :, -W:, :]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    l0 = ar.launches
    times = []
    for i in range(a.warmup + a.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ar.compress_prompt(q_obs, kp, v, k, pos)  # the whole prompt again, from an empty slab
        e1.record()
        e1.synchronize()
        if i >= a.warmup:
            times.append(e0.elapsed_time(e1) * 1e3)
    us = float(statistics.median(times))
    flops = 2.0 * Hk * W * T * D
    kv_bytes = 3.0 * Hk * T * D * 2  # k_post scored, k_pre and v of every token copied once
    return {"metric": "SnapKV prompt compression: us per prompt-layer (score + pool + top-k + evict)",
            "value": round(us, 2), "unit": "us/prompt-layer", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) pre-RoPE q/k/v, seeded",
            "config": {"workload": f"{T}-token prompt, 32/8 heads, D 128, window {W}, max-pool 7, budget {budget}",
                       "l2": "flushed before every timed call"},
            "scoring_tflops": round(flops / (us * 1e-6) / 1e12, 3),
            "hbm_gbs": round(kv_bytes / (us * 1e-6) / 1e9, 1)}


def triton_bar(c, dev, sets: int = 32, reps: int = 10):
    """The reference's own GPU decode attention, triton_evict_attention_forward (kernels.py:77-137,
    called as patch.py:295 calls it), against this library's drop-in of the same call
    (kernels.triton_evict_attention_forward: hc_attention_dense + evict_idx), on this GPU at the
    benchmark's attended rows (budget + 1 hot + R held), fp16, 32/8 heads. Each is captured as
    one CUDA graph of `sets` calls over distinct K/V buffers, replayed after an L2 flush; us per
    call = median replay / sets."""
    import torch
    try:
        from oracle.ref_shims import load_reference
        ref = load_reference(cpu=False).hotcold_kv
    except Exception as e:  # the reference is not installed next to the repo
        return {"unavailable": f"reference not importable: {e}"}
    from hotcold_kv_cache_b200.kernels import triton_evict_attention_forward as ours
    S, Hq, Hk, D = c["budget"] + 1 + c["lookahead_k"], c["Hq"], c["Hk"], c["D"]
    g = torch.Generator(device=dev).manual_seed(5)
    bufs = [(torch.randn((1, Hq, 1, D), generator=g, device=dev, dtype=torch.float16),
             torch.randn((1, Hk, S, D), generator=g, device=dev, dtype=torch.float16),
             torch.randn((1, Hk, S, D), generator=g, device=dev, dtype=torch.float16)) for _ in range(sets)]
    mask = torch.ones((1, S), dtype=torch.bool, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)
    out = {"rows": S, "calls_per_graph": sets, "dtype": "f16"}
    for name, fn in (("reference_triton_us", ref.triton_evict_attention_forward), ("hc_dropin_us", ours)):
        def run():
            for q, k, v in bufs:
                fn(q, k, v, mask, Hq // Hk, 1.0 / math.sqrt(D))
        run()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            run()  # warm the allocator on the capture stream
            with torch.cuda.graph(graph, stream=stream):
                run()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            graph.replay()
            e1.record(cur)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3 / sets)
        out[name] = round(statistics.median(times), 3)
        del graph
    out["speedup"] = round(out["reference_triton_us"] / out["hc_dropin_us"], 2)
    return out


# ------------------------------------------------------------------------------------------
# CPU arm: the reference's own code (baseline/_ref), else the oracle port, on one layer
# ------------------------------------------------------------------------------------------
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_cpu(c, seed, warmup, steps):
    """The reference's own CPU path (patched forward with its SDPA decode fallback, its cache and
    controller, SnapKV as the composition of its scoring functions, faiss -> exact flat-IP
    stand-in; oracle/ref_shims.py) on ONE layer of the workload with every host thread: prompt
    untimed, `warmup` + `steps` decode steps, the latter timed. Falls back to the oracle port
    when the reference is not installed. Returns (us per layer-step, cpu_baseline dict)."""
    import torch
    thr = host_threads()
    torch.set_num_threads(thr)
    try:
        from oracle.ref_shims import time_reference_layer
        us, _, dbg = time_reference_layer(c, seed, warmup, steps, "cpu")
        sample = (f"1 of {c['layers']} layers: {c['prompt']}-token prompt (untimed), {warmup} warm-up + {steps} timed "
                  f"decode steps ({dbg['retrieval_launched']} cold searches among them), the reference's own "
                  f"patched forward on the CPU (SDPA decode fallback), faiss unavailable: exact flat-IP stand-in")
        return us, {"value": round(us, 1), "unit": UNIT, "cores": thr, "kind": "reference", "sample": sample}
    except ImportError:
        us, thr = cpu_port(c, max(warmup + steps, 1), seed)
        return us, {"value": round(us, 1), "unit": UNIT, "cores": thr, "kind": "port",
                    "sample": f"1 of {c['layers']} layers, {warmup + steps} decode steps, numpy restatement in "
                              f"oracle/ (the reference is not installed under baseline/_ref)"}


# ------------------------------------------------------------------------------------------
# CPU port: the oracle restatement of the reference path on one layer
# ------------------------------------------------------------------------------------------
def cpu_port(c, n_steps, seed):
    """Time the CPU restatement of the reference per-layer decode step (torch-free numpy port)
    on ONE layer of the workload: prompt compressed into hot + cold tiers (untimed), then
    n_steps decode steps timed with perf_counter. Returns (us per layer-step, threads)."""
    from hotcold_kv_cache_b200 import synth
    from oracle import hotcold_oracle as O
    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        threads = 1
    inp = synth.layer_inputs(seed, 1, c["Hq"], c["Hk"], c["D"], c["prompt"], n_steps, c["dtype"])
    layer = O.OracleLayer(Hq=c["Hq"], Hk=c["Hk"], D=c["D"], dtype=c["dtype"],
                          inv_freq=synth.rope_inv_freq(c["D"], c["theta"]),
                          policy=O.Policy(c["policy"], cap=c["budget"], recent=c["recent"],
                                          topk_ratio=c["topk_ratio"], pool_kernel=c["pool_kernel"]),
                          cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], window_size=c["window_size"],
                          query_pool_size=c["query_pool_size"], lookahead_k=c["lookahead_k"],
                          hold_retrieved=c["hold"], retrieve_after_prefill=False)
    layer.prefill(inp["q_pre"], inp["k_pre"], inp["v"])
    layer.start_decode(c["prompt"])
    ts = []
    for i in range(n_steps):
        t0 = time.perf_counter()
        layer.decode(inp["dq"][i], inp["dk"][i], inp["dv"][i], step=i + 1)
        ts.append(time.perf_counter() - t0)
    return float(np.mean(ts)) * 1e6, threads


def cpu_baseline_obj(c, n_steps, seed):
    return reference_cpu(c, seed, 0, n_steps)[1]


def sub_result(r: dict) -> dict:
    """A workload's line, reduced to what a sub-result of the default line needs."""
    keep = ("metric", "value", "unit", "higher_is_better", "scaling", "ms_per_step", "steps", "warmup", "config",
            "aggregate_hbm_gbs", "gpu_launches", "ops_us_per_step", "ops_us_per_layer_step")
    return {k: r[k] for k in keep if k in r}


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if a.impl == "reference":
        if rank != 0:
            return 0
        c = config(a)
        us, cb = reference_cpu(c, a.seed, a.warmup, a.steps)
        out = {"impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": UNIT, "n_gpus": a.gpus,
               "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(us * c["layers"] / 1e3, 3),
               "ms_per_step_note": "per layer-step time x layers (one layer of the workload is timed)",
               "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
               "data": "synthetic N(0,1) pre-RoPE q/k/v, seeded",
               "config": workload_config(c, {"parallelism": "cpu"}),
               "cpu_baseline": cb,
               "e2e": {"value": round(us, 1), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(out))
        return 0
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    if a.workload != "decode":
        run = {"ragged": run_ragged, "cold-shard": run_cold_shard, "prefill": run_prefill, "model": run_model}[a.workload]
        res = run(a, rank, world)
        if world > 1:
            import torch
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        if rank == 0:
            print(json.dumps(res))
        return 0
    import torch
    res = run_ours(a, rank, world)
    if not a.no_partitioned:
        # the partitioned configurations at this N, timed in the same run (every rank takes part)
        torch.cuda.empty_cache()
        res["ragged"] = sub_result(run_ragged(a, rank, world))
        torch.cuda.empty_cache()
        res["cold_shard"] = sub_result(run_cold_shard(a, rank, world))
        torch.cuda.empty_cache()
    if rank == 0:
        res["triton_reference"] = triton_bar(config(a), torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
    if rank == 0 and not a.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_obj(config(a), a.cpu_steps, a.seed)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
