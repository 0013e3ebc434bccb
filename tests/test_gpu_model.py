"""The patched Llama forward on a random-init model: the reference's
tests/test_parity.py checks 1-5 (causality, prefill and teacher-forced decode
parity with compression off, zero counters, prefill independent of the budget)
and the logits of the reference's own patched forward on a 2-layer model
(golden vectors with compression and retrieval active)."""

import json

import numpy as np
import pytest
import torch

from golden_cases import load

pytestmark = pytest.mark.gpu

TOL_LOGIT = 0.5
TOL_DECODE_LOGIT = 1.0
MAX_TOP1_MISMATCH = 1


def _model(cfg: dict, seed: int, dtype=torch.float32):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    m = LlamaForCausalLM(LlamaConfig(**cfg)).eval()
    return m.to(device="cuda", dtype=dtype)


def _ctrl(budget=10 ** 9, **kw):
    from hotcold_kv_cache_b200 import KVController
    args = dict(max_capacity_prompt=budget, topk_ratio=0.15, recent_size=min(128, max(budget // 2, 1)),
                cpu_buffer_size=4096, faiss_dim=64, window_size=16, query_pool_size=4, lookahead_k=0,
                enable_asserts=True, profile_overlap=False)
    args.update(kw)
    return KVController(**args)


def decode_trace(model, ids, cache, n_steps, forced=None):
    out = model(input_ids=ids, use_cache=True, past_key_values=cache)
    prefill = out.logits[:, -1, :].float().cpu()
    past = out.past_key_values
    nxt = int(out.logits[0, -1].argmax())
    T = int(ids.shape[1])
    logits, fed = [], []
    for i in range(n_steps):
        tok = forced[i] if forced is not None else nxt
        fed.append(tok)
        cur = torch.tensor([[tok]], device=ids.device)
        cp = torch.tensor([T + i], device=ids.device)
        out = model(input_ids=cur, cache_position=cp, past_key_values=past, use_cache=True)
        lg = out.logits[:, -1, :].float()
        logits.append(lg.cpu())
        nxt = int(lg[0].argmax())
        past = out.past_key_values
    return prefill, logits, fed


SMALL = dict(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim=128, rope_theta=500000.0, max_position_embeddings=2048)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_reference_parity_checks(dtype):
    import hotcold_kv_cache_b200 as hc
    from transformers.cache_utils import DynamicCache
    model = _model(SMALL, 0, dtype)
    ids = torch.randint(0, SMALL["vocab_size"], (1, 300), generator=torch.Generator().manual_seed(5)).cuda()
    n_decode = 16
    with torch.inference_mode():
        ref_prefill, ref_logits, ref_fed = decode_trace(model, ids, DynamicCache(), n_decode)
    hc.set_active_rotary_emb(model.model.rotary_emb)
    hc.uninstall_monkeypatch()
    hc.install_monkeypatch(enable_debug=False)
    try:
        k = int(ids.shape[1]) // 2
        with torch.inference_mode():
            hc.set_active_kvctrl(_ctrl())
            full_k = model(input_ids=ids, use_cache=False).logits[0, k].float().cpu()
            hc.set_active_kvctrl(_ctrl())
            trunc_k = model(input_ids=ids[:, :k + 1], use_cache=False).logits[0, -1].float().cpu()
        assert (full_k - trunc_k).abs().max().item() < TOL_LOGIT, "1. prefill causality"
        kv = _ctrl()
        hc.set_active_kvctrl(kv)
        with torch.inference_mode():
            got_prefill, got_logits, _ = decode_trace(model, ids, hc.build_hotcold_cache(model, kv), n_decode,
                                                      forced=ref_fed)
        assert (ref_prefill - got_prefill).abs().max().item() < TOL_LOGIT, "2. prefill parity"
        d = max((a - b).abs().max().item() for a, b in zip(ref_logits, got_logits))
        agree = sum(int(a.argmax() == b.argmax()) for a, b in zip(ref_logits, got_logits))
        assert agree >= n_decode - MAX_TOP1_MISMATCH and d < TOL_DECODE_LOGIT, ("3. decode parity", d, agree)
        if dtype == torch.float32:
            assert d < 1e-3, d
        cold = sum(kv.cold_size(i) for i in range(SMALL["num_hidden_layers"]))
        assert cold == 0 and kv.dbg["evicted_tokens"] == 0 and kv.dbg["injection_used"] == 0, "4. compression off"
        assert kv.dbg["triton_decode_calls"] == n_decode * SMALL["num_hidden_layers"]
        small = max(8, int(ids.shape[1]) // 4)
        kv_c = _ctrl(budget=small)
        hc.set_active_kvctrl(kv_c)
        with torch.inference_mode():
            out = model(input_ids=ids, use_cache=True, past_key_values=hc.build_hotcold_cache(model, kv_c))
        comp = out.logits[:, -1, :].float().cpu()
        assert kv_c.dbg["evicted_tokens"] > 0
        assert (got_prefill - comp).abs().max().item() < TOL_LOGIT, "5. prefill vs budget"
    finally:
        hc.uninstall_monkeypatch()
        hc.set_active_kvctrl(None)


def test_tiny_model_golden():
    """Logits of every step against the reference's patched forward run on CPU (fp32, 2 layers,
    compression at prefill and during decode, retrieval every 4 steps, held)."""
    import hotcold_kv_cache_b200 as hc
    g = load("tiny_model")
    cfg, run = g["case"]["model"], g["case"]["run"]
    model = _model(cfg, run["model_seed"])
    ids = torch.from_numpy(g["ids"]).cuda()
    kv = hc.KVController(max_capacity_prompt=run["cap"], topk_ratio=run["topk_ratio"], recent_size=run["recent"],
                         cpu_buffer_size=run["ccap"], faiss_dim=run["faiss_dim"], window_size=run["window_size"],
                         query_pool_size=run["pool"], lookahead_k=run["R"], hold_retrieved=run["hold"],
                         retrieve_after_prefill=run["rap"], enable_asserts=True, profile_overlap=False)
    hc.uninstall_monkeypatch()
    hc.set_active_rotary_emb(model.model.rotary_emb)
    hc.install_monkeypatch(enable_debug=False)
    hc.set_active_kvctrl(kv)
    try:
        cache = hc.build_hotcold_cache(model, kv)
        T = run["T"]
        logits = []
        with torch.inference_mode():
            out = model(input_ids=ids[:, :T], use_cache=True, past_key_values=cache)
            logits.append(out.logits[0, -1].float().cpu().numpy())
            for i in range(run["steps"]):
                out = model(input_ids=ids[:, T + i:T + i + 1], cache_position=torch.tensor([T + i], device="cuda"),
                            past_key_values=cache, use_cache=True)
                logits.append(out.logits[0, -1].float().cpu().numpy())
    finally:
        hc.uninstall_monkeypatch()
        hc.set_active_kvctrl(None)
    got = np.stack(logits, 0)
    ref = g["logits"]
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 1e-4, err
    for k, v in g["dbg"].items():
        if k.startswith("triton") or k.startswith("prefetch_copy"):
            continue
        assert kv.dbg[k] == v, (k, kv.dbg[k], v)
    assert [kv.cold_size(i) for i in range(cfg["num_hidden_layers"])] == list(g["cold_sizes"])
    assert kv.device_status() == 0


def test_chunked_prompt_through_patched_forward():
    """A prompt sent in three forwards (the reference raises NotImplementedError on the second,
    patch.py:325-329): each chunk's tokens join the hot tier and the tier is compressed with the
    chunk's last recent_size queries as the observation window; decode then continues. Layer 0
    (its q/k/v recorded by hooks) against the oracle's chunked prefill at every step: hot sets
    after each chunk and each decode step, attention outputs, retrieved sets."""
    import hotcold_kv_cache_b200 as hc
    from golden_cases import oracle_kwargs
    from oracle import hotcold_oracle as O
    from oracle_follow import assert_same_run, run_following
    model = _model(SMALL, 3, torch.float32)
    Hq, Hk, D = SMALL["num_attention_heads"], SMALL["num_key_value_heads"], SMALL["head_dim"]
    bounds, steps = [0, 120, 250, 300], 12
    c = dict(B=1, Hq=Hq, Hk=Hk, D=D, T=bounds[-1], steps=steps, dtype="float32", policy="snapkv", cap=64, recent=16,
             topk_ratio=0.0, pool_kernel=7, ccap=1000, faiss_dim=128, window_size=4, pool=2, R=8, hold=True,
             rap=True, theta=SMALL["rope_theta"])
    kv = hc.KVController(max_capacity_prompt=c["cap"], topk_ratio=0.0, recent_size=c["recent"],
                         cpu_buffer_size=c["ccap"], faiss_dim=128, window_size=c["window_size"], query_pool_size=c["pool"],
                         lookahead_k=c["R"], hold_retrieved=True, retrieve_after_prefill=True, policy="snapkv",
                         profile_overlap=False)
    ids = torch.randint(0, SMALL["vocab_size"], (1, bounds[-1] + steps), generator=torch.Generator().manual_seed(8))
    ids = ids.cuda()
    att = model.model.layers[0].self_attn
    rec = {"q": [], "k": [], "v": [], "o": []}
    hooks = [att.q_proj.register_forward_hook(lambda m, i, o: rec["q"].append(o.detach().cpu())),
             att.k_proj.register_forward_hook(lambda m, i, o: rec["k"].append(o.detach().cpu())),
             att.v_proj.register_forward_hook(lambda m, i, o: rec["v"].append(o.detach().cpu())),
             att.o_proj.register_forward_pre_hook(lambda m, a: rec["o"].append(a[0].detach().cpu()))]
    hc.uninstall_monkeypatch()
    hc.set_active_rotary_emb(model.model.rotary_emb)
    hc.install_monkeypatch(enable_debug=False)
    hc.set_active_kvctrl(kv)
    res = dict(outs=[], hot=[], held={}, hot0=[], launched=set())
    try:
        cache = hc.build_hotcold_cache(model, kv)
        with torch.inference_mode():
            for c0, c1 in zip(bounds[:-1], bounds[1:]):
                model(input_ids=ids[:, c0:c1], cache_position=torch.arange(c0, c1, device="cuda"),
                      past_key_values=cache, use_cache=True, logits_to_keep=1)
                res["hot0"].append(kv.arenas[0].hot_positions().cpu().numpy())
            a = kv.arenas[0]
            for i in range(steps):
                T = bounds[-1]
                ready, launched = kv.dbg["prefetch_ready"], kv.dbg["retrieval_launched"]
                model(input_ids=ids[:, T + i:T + i + 1], cache_position=torch.tensor([T + i], device="cuda"),
                      past_key_values=cache, use_cache=True, logits_to_keep=1)
                res["outs"].append(rec["o"][-1].double().view(1, Hq, D).numpy())
                res["hot"].append(a.hot_positions().cpu().numpy())
                if kv.dbg["prefetch_ready"] != ready:
                    R = a.r_max
                    res["held"][i + 1] = (a.held_pos[:, :R].cpu().numpy(), a.held_valid[:, :R].cpu().numpy().astype(bool),
                                          a.held_k[:, :, :R].double().cpu().numpy())
                if kv.dbg["retrieval_launched"] != launched:
                    res["launched"].add(i + 1)
    finally:
        for h in hooks:
            h.remove()
        hc.uninstall_monkeypatch()
        hc.set_active_kvctrl(None)
    res["outs"] = np.stack(res["outs"], 0)
    f = lambda ts, H: np.concatenate([t.float().view(1, t.shape[1], H, D).transpose(1, 2).numpy() for t in ts], 2)
    n_chunks = len(bounds) - 1
    inp = dict(q_pre=f(rec["q"][:n_chunks], Hq), k_pre=f(rec["k"][:n_chunks], Hk), v=f(rec["v"][:n_chunks], Hk),
               dq=np.stack([f([t], Hq)[:, :, 0] for t in rec["q"][n_chunks:]], 0),
               dk=np.stack([f([t], Hk)[:, :, 0] for t in rec["k"][n_chunks:]], 0),
               dv=np.stack([f([t], Hk)[:, :, 0] for t in rec["v"][n_chunks:]], 0))
    kw = dict(oracle_kwargs(c), inv_freq=model.model.rotary_emb.inv_freq.float().cpu().numpy())
    layer, o_outs, o_hot, _ = run_following(O, inp, steps, res, chunks=bounds, **kw)
    assert assert_same_run(res, layer, o_outs, o_hot, "float32", steps, "layer 0") == steps
    assert kv.dbg["evicted_tokens"] > 0 and kv.device_status() == 0
