"""Drive the CUDA hot path of one layer the way oracle.run_layer drives the
restatement: a prompt forward, then decode steps, recording the attention
output, the hot positions and the held set after every step."""

import math

import numpy as np
import torch
from transformers import LlamaConfig
from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding, apply_rotary_pos_emb

from hotcold_kv_cache_b200.controller import KVController

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def rotary(Hq, D, theta, device, max_pos=1 << 20):
    cfg = LlamaConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=1, head_dim=D,
                      num_hidden_layers=1, rope_theta=theta, vocab_size=16, intermediate_size=16,
                      max_position_embeddings=max_pos)
    return LlamaRotaryEmbedding(cfg).to(device)


def controller_kwargs(case):
    c = case
    return dict(max_capacity_prompt=c["cap"], topk_ratio=c["topk_ratio"], recent_size=c["recent"],
                cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], normalize_for_ip=True,
                window_size=c["window_size"], query_pool_size=c["pool"], lookahead_k=c["R"],
                hold_retrieved=c["hold"], retrieve_after_prefill=c["rap"], policy=c["policy"],
                pool_kernel=c.get("pool_kernel", 7), pooling=c.get("pooling", "maxpool"),
                async_retrieval=c.get("async", False))


def run_cuda_layer(case, inputs, n_steps, device="cuda:0", model_cos=True, fused=True, chunks=None, searcher=None):
    """Returns dict(outs (n,B,Hq,D) float64, hot [per-step (B,S) int64], held {step: (pos, valid, k)},
    ctrl). model_cos=True passes HF's cos/sin tables to the append kernel (what the patched
    forward does); False lets the kernel compute them from inv_freq. `searcher(ctrl)`, when
    given, makes the sharded cold search the controller uses."""
    c = case
    dev = torch.device(device)
    dt = TORCH_DT[c["dtype"]]
    B, Hq, Hk, D, T = c["B"], c["Hq"], c["Hk"], c["D"], c["T"]

    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x).astype(np.float32)).to(device=dev, dtype=dt)

    rot = rotary(Hq, D, c["theta"], dev)
    ctrl = KVController(**controller_kwargs(c))
    ctrl.fused_step = fused
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    if searcher is not None:
        ctrl.cold_search = searcher(ctrl)
    q_pre, k_pre, v = t(inputs["q_pre"]), t(inputs["k_pre"]), t(inputs["v"])
    ctrl._lazy_init(k_pre, n_layers=1)
    pos = torch.arange(T, device=dev).unsqueeze(0).expand(B, T)
    cos, sin = rot(torch.empty(1, dtype=dt, device=dev), pos)
    q_post, k_post = apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
    hot0 = []  # hot positions after the prompt (after each chunk of a chunked prompt)
    if chunks is None:
        ctrl.prefill_layer(0, q_pre, q_post, k_pre, k_post, v, pos)
        hot0.append(ctrl.arenas[0].hot_positions().cpu().numpy())
    else:
        for c0, c1 in zip(chunks[:-1], chunks[1:]):
            ctrl.prefill_chunk(0, q_pre[:, :, c0:c1], q_post[:, :, c0:c1], k_pre[:, :, c0:c1], k_post[:, :, c0:c1],
                               v[:, :, c0:c1], pos[:, c0:c1], last=c1 == chunks[-1])
            hot0.append(ctrl.arenas[0].hot_positions().cpu().numpy())
    outs, hot, held, launched = [], [], {}, set()
    dq, dk, dv = t(inputs["dq"]), t(inputs["dk"]), t(inputs["dv"])
    for i in range(n_steps):
        p = T + i
        pd = torch.full((B,), p, device=dev, dtype=torch.long)
        if model_cos:
            c1, s1 = rot(torch.empty(1, dtype=dt, device=dev), pd[:, None])
            c1, s1 = c1.reshape(B, D), s1.reshape(B, D)
        else:
            c1 = s1 = None
        ready_before = ctrl.dbg["prefetch_ready"]
        launched_before = ctrl.dbg["retrieval_launched"]
        o = ctrl.decode_layer(0, dq[i], dk[i], dv[i], c1, s1, pd)
        if ctrl.dbg["retrieval_launched"] != launched_before:
            launched.add(i + 1)
        outs.append(o.double().cpu().numpy())
        a = ctrl.arenas[0]
        hot.append(a.hot_positions().cpu().numpy())
        if ctrl.dbg["prefetch_ready"] != ready_before:
            R = a.r_max
            held[i + 1] = (a.held_pos[:, :R].cpu().numpy(), a.held_valid[:, :R].cpu().numpy().astype(bool),
                           a.held_k[:, :, :R].double().cpu().numpy())
    torch.cuda.synchronize(dev)
    return dict(outs=np.stack(outs, 0), hot=hot, held=held, hot0=hot0, launched=launched, ctrl=ctrl)


def run_cuda_layers(case, layer_inputs, n_steps, device="cuda:0", fused=True):
    """Several layers of one model the way a decode loop runs them: every layer's prompt,
    then per step every layer's decode_layer back to back (no host synchronisation between
    layers, so each layer's step is chained to the previous layer's). Returns one dict per
    layer, as run_cuda_layer."""
    c = case
    dev = torch.device(device)
    dt = TORCH_DT[c["dtype"]]
    B, Hq, Hk, D, T = c["B"], c["Hq"], c["Hk"], c["D"], c["T"]
    L = len(layer_inputs)

    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x).astype(np.float32)).to(device=dev, dtype=dt)

    rot = rotary(Hq, D, c["theta"], dev)
    ctrl = KVController(**controller_kwargs(c))
    ctrl.fused_step = fused
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    pos = torch.arange(T, device=dev).unsqueeze(0).expand(B, T)
    cos, sin = rot(torch.empty(1, dtype=dt, device=dev), pos)
    res = [dict(outs=[], hot=[], held={}, hot0=[], launched=set(), ctrl=ctrl) for _ in range(L)]
    for li, inp in enumerate(layer_inputs):
        q_pre, k_pre, v = t(inp["q_pre"]), t(inp["k_pre"]), t(inp["v"])
        if li == 0:
            ctrl._lazy_init(k_pre, n_layers=L)
        q_post, k_post = apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
        ctrl.prefill_layer(li, q_pre, q_post, k_pre, k_post, v, pos)
        res[li]["hot0"].append(ctrl.arenas[li].hot_positions().cpu().numpy())
        del q_pre, k_pre, v, q_post, k_post
    dq = torch.stack([t(inp["dq"]) for inp in layer_inputs], 1)  # (steps, L, B, Hq, D)
    dk = torch.stack([t(inp["dk"]) for inp in layer_inputs], 1)
    dv = torch.stack([t(inp["dv"]) for inp in layer_inputs], 1)
    out = torch.empty((L, B, Hq, D), dtype=dt, device=dev)
    for i in range(n_steps):
        pd = torch.full((B,), T + i, device=dev, dtype=torch.long)
        c1, s1 = rot(torch.empty(1, dtype=dt, device=dev), pd[:, None])
        c1, s1 = c1.reshape(B, D).contiguous(), s1.reshape(B, D).contiguous()
        ready = [ctrl.dbg["prefetch_ready"]]
        for li in range(L):
            n0 = ctrl.dbg["retrieval_launched"]
            ctrl.decode_layer(li, dq[i, li], dk[i, li], dv[i, li], c1, s1, pd, out=out[li])
            ready.append(ctrl.dbg["prefetch_ready"])
            if ctrl.dbg["retrieval_launched"] != n0:
                res[li]["launched"].add(i + 1)
        o = out.double().cpu().numpy()
        for li in range(L):
            a = ctrl.arenas[li]
            r = res[li]
            r["outs"].append(o[li])
            r["hot"].append(a.hot_positions().cpu().numpy())
            if ready[li + 1] != ready[li]:
                R = a.r_max
                r["held"][i + 1] = (a.held_pos[:, :R].cpu().numpy(), a.held_valid[:, :R].cpu().numpy().astype(bool),
                                    a.held_k[:, :, :R].double().cpu().numpy())
    torch.cuda.synchronize(dev)
    for r in res:
        r["outs"] = np.stack(r["outs"], 0)
    return res


def cold_positions(ctrl, li=0):
    a = ctrl.arenas[li]
    return [a.cold_pos[b].index_select(0, a.cold_order(b)).cpu().numpy() for b in range(a.n_seq)]


def run_cuda_ragged(case, seq_inputs, budgets, ccaps, n_steps, device="cuda:0", fused=True):
    """A ragged batch through one controller: sequence b has its own prompt (seq_inputs[b],
    B=1 arrays of layer_inputs), budget and cold capacity; prompts go in one at a time
    (prefill_sequence + finish_prefill), decode steps run all sequences at once with their
    own positions. Returns dict(outs [per-step (n_seq,Hq,D)], hot [per-step list of arrays], ctrl)."""
    c = case
    dev = torch.device(device)
    dt = TORCH_DT[c["dtype"]]
    Hq, Hk, D = c["Hq"], c["Hk"], c["D"]
    n = len(seq_inputs)

    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x).astype(np.float32)).to(device=dev, dtype=dt)

    rot = rotary(Hq, D, c["theta"], dev)
    ctrl = KVController(**controller_kwargs(c))
    ctrl.fused_step = fused
    ctrl.set_rotary(rot.inv_freq, rot.attention_scaling)
    ctrl.set_ragged(budgets, ccaps, Hk, D, 1, dev)
    Ts = []
    for b, inp in enumerate(seq_inputs):
        q_pre, k_pre, v = t(inp["q_pre"]), t(inp["k_pre"]), t(inp["v"])
        T = q_pre.shape[2]
        Ts.append(T)
        pos = torch.arange(T, device=dev).unsqueeze(0)
        cos, sin = rot(torch.empty(1, dtype=dt, device=dev), pos)
        q_post, k_post = apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
        ctrl.prefill_sequence(0, b, q_pre, q_post, k_pre, k_post, v, pos)
    ctrl.finish_prefill(0)
    a = ctrl.arenas[0]
    hot0 = [a.hot_pos[b].index_select(0, a.logical_order(b)).cpu().numpy() for b in range(n)]
    dq = torch.cat([t(inp["dq"]) for inp in seq_inputs], 1)  # (steps, n, Hq, D)
    dk = torch.cat([t(inp["dk"]) for inp in seq_inputs], 1)
    dv = torch.cat([t(inp["dv"]) for inp in seq_inputs], 1)
    outs, hot, held, launched = [], [], {}, set()
    for i in range(n_steps):
        pd = torch.tensor([T + i for T in Ts], device=dev, dtype=torch.long)
        c1, s1 = rot(torch.empty(1, dtype=dt, device=dev), pd[:, None])
        ready = ctrl.dbg["prefetch_ready"]
        n0 = ctrl.dbg["retrieval_launched"]
        o = ctrl.decode_layer(0, dq[i], dk[i], dv[i], c1.reshape(n, D), s1.reshape(n, D), pd)
        if ctrl.dbg["retrieval_launched"] != n0:
            launched.add(i + 1)
        outs.append(o.double().cpu().numpy())
        a = ctrl.arenas[0]
        hot.append([a.hot_pos[b].index_select(0, a.logical_order(b)).cpu().numpy() for b in range(n)])
        if ctrl.dbg["prefetch_ready"] != ready:
            R = a.r_max
            held[i + 1] = (a.held_pos[:, :R].cpu().numpy(), a.held_valid[:, :R].cpu().numpy().astype(bool),
                           a.held_k[:, :, :R].double().cpu().numpy())
    torch.cuda.synchronize(dev)
    return dict(outs=outs, hot=hot, held=held, hot0=hot0, launched=launched, ctrl=ctrl)


def ragged_seq(res, b):
    """Sequence b of a run_cuda_ragged result in run_cuda_layer's layout (batch of one)."""
    return dict(outs=np.stack([o[b:b + 1] for o in res["outs"]], 0), hot=[h[b][None] for h in res["hot"]],
                hot0=[res["hot0"][b][None]], launched=res["launched"],
                held={s: (p[b:b + 1], v[b:b + 1], k[b:b + 1]) for s, (p, v, k) in res["held"].items()})
