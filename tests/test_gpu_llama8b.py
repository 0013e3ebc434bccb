"""BASELINE configs 1 and 2 through the reference's own entry point: a random-init 32-layer
Llama-3.1-8B in fp16 (weights N(0, 0.02)), install_monkeypatch + build_hotcold_cache (the
reference's patch.py:122-348 / cache.py:170-173 API), the prompt forward and 63 teacher-forced
decode steps of uniform random tokens.

  config 1: 8192-token prompt, budget 512, top-64 retrieval every 16 steps, held;
  config 2: 16384-token prompt, budget 1024, a planted key in the first quarter of the prompt
            (synth.plant_key: 4 x the GQA-group mean of the final token's pre-RoPE queries),
            prompt-end retrieval of the top 128 from the last 8 queries, held.

Layer 0's attention, its q/k/v projections recorded by hooks, is compared with the oracle at
every step (hot sets, attention outputs, retrieved sets, re-rotated held keys). Config 2 also
checks the claim of the method: at decode step 1 the planted token is attended in every layer,
either kept in the hot tier by the eviction policy or, where the policy evicted it, brought back
by the prompt-end retrieval. (The policy keeps it in most layers: with RoPE theta 500000 the
lowest frequencies barely turn over 16k positions, so a key aligned with the final query before
RoPE keeps a large logit with it after RoPE, and the observation window holds that query.)"""

import numpy as np
import pytest
import torch

from golden_cases import oracle_kwargs
from oracle_follow import assert_same_run, run_following

pytestmark = pytest.mark.gpu

from oracle import hotcold_oracle as O  # noqa: E402

STEPS = 63


@pytest.fixture(scope="module")
def model():
    from hotcold_kv_cache_b200 import synth
    m = synth.llama8b_random("cuda", seed=0)
    yield m
    del m
    torch.cuda.empty_cache()


class _Recorder:
    """Layer li's pre-RoPE q/k/v projections and attention output (o_proj input)."""

    def __init__(self, att):
        self.q, self.k, self.v, self.o = [], [], [], []
        self.h = [att.q_proj.register_forward_hook(lambda m, i, o: self.q.append(o.detach().cpu())),
                  att.k_proj.register_forward_hook(lambda m, i, o: self.k.append(o.detach().cpu())),
                  att.v_proj.register_forward_hook(lambda m, i, o: self.v.append(o.detach().cpu())),
                  att.o_proj.register_forward_pre_hook(lambda m, a: self.o.append(a[0].detach().cpu()))]

    def remove(self):
        for h in self.h:
            h.remove()

    def inputs(self, Hq, Hk, D):
        """The layer's inputs in synth.layer_inputs layout (float32 holding fp16 values)."""
        f = lambda t, H: t.float().view(t.shape[0], t.shape[1], H, D).transpose(1, 2).numpy()
        dq = np.stack([f(t, Hq)[:, :, 0] for t in self.q[1:]], 0)
        dk = np.stack([f(t, Hk)[:, :, 0] for t in self.k[1:]], 0)
        dv = np.stack([f(t, Hk)[:, :, 0] for t in self.v[1:]], 0)
        return dict(q_pre=f(self.q[0], Hq), k_pre=f(self.k[0], Hk), v=f(self.v[0], Hk), dq=dq, dk=dk, dv=dv)


def _case(cfg):
    c = dict(B=1, Hq=32, Hk=8, D=128, dtype="float16", policy="snapkv", recent=32, topk_ratio=0.0, pool_kernel=7,
             faiss_dim=128, hold=True, theta=500000.0, steps=STEPS)
    if cfg == 1:
        c.update(T=8192, cap=512, ccap=32768, window_size=16, pool=4, R=64, rap=False)
    else:
        c.update(T=16384, cap=1024, ccap=16384, window_size=16, pool=8, R=128, rap=True)
    return c


def _run(model, c, seed, plant=None, record=0):
    """Prompt + STEPS decode steps through the patched forward. Returns (layer `record`'s run in
    cuda_runner's layout, its recorded inputs, the controller, per-layer prompt state, us/token)."""
    import hotcold_kv_cache_b200 as hc
    from cuda_runner import cold_positions
    ctrl = hc.KVController(max_capacity_prompt=c["cap"], topk_ratio=c["topk_ratio"], recent_size=c["recent"],
                           cpu_buffer_size=c["ccap"], faiss_dim=c["faiss_dim"], window_size=c["window_size"],
                           query_pool_size=c["pool"], lookahead_k=c["R"], hold_retrieved=c["hold"],
                           retrieve_after_prefill=c["rap"], policy=c["policy"], pool_kernel=c["pool_kernel"],
                           profile_overlap=False)
    T, n = c["T"], c["steps"]
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, model.config.vocab_size, (1, T + n), generator=g).cuda()
    hc.uninstall_monkeypatch()
    hc.set_active_rotary_emb(model.model.rotary_emb)
    hc.install_monkeypatch(enable_debug=False)
    hc.set_active_kvctrl(ctrl)
    handles = []
    try:
        cache = hc.build_hotcold_cache(model, ctrl)
        if plant is not None:
            from hotcold_kv_cache_b200 import synth
            handles = synth.plant_key(model, plant)
        rec = _Recorder(model.model.layers[record].self_attn)
        with torch.inference_mode():
            model(input_ids=ids[:, :T], use_cache=True, past_key_values=cache, logits_to_keep=1)
        for h in handles:
            h.remove()
        handles = []
        L = model.config.num_hidden_layers
        prompt_state = [(ctrl.arenas[li].hot_positions().cpu().numpy()[0], cold_positions(ctrl, li)[0])
                        for li in range(L)]
        a = ctrl.arenas[record]
        res = dict(outs=[], hot=[], held={}, hot0=[a.hot_positions().cpu().numpy()], launched=set(), ctrl=ctrl,
                   held_all={})
        times = []
        for i in range(n):
            ready, launched = ctrl.dbg["prefetch_ready"], ctrl.dbg["retrieval_launched"]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.inference_mode():
                e0.record()
                model(input_ids=ids[:, T + i:T + i + 1], cache_position=torch.tensor([T + i], device="cuda"),
                      past_key_values=cache, use_cache=True, logits_to_keep=1)
                e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
            res["outs"].append(rec.o[-1].float().view(1, c["Hq"], c["D"]).double().numpy())
            res["hot"].append(a.hot_positions().cpu().numpy())
            if ctrl.dbg["prefetch_ready"] != ready:
                R = a.r_max
                res["held"][i + 1] = (a.held_pos[:, :R].cpu().numpy(), a.held_valid[:, :R].cpu().numpy().astype(bool),
                                      a.held_k[:, :, :R].double().cpu().numpy())
                if i == 0:
                    res["held_all"] = {li: (ctrl.arenas[li].held_pos[0, :R].cpu().numpy(),
                                            ctrl.arenas[li].held_valid[0, :R].cpu().numpy().astype(bool))
                                       for li in range(L)}
            if ctrl.dbg["retrieval_launched"] != launched:
                res["launched"].add(i + 1)
        res["outs"] = np.concatenate(res["outs"], 0)[:, None]
        rec.remove()
        inp = rec.inputs(c["Hq"], c["Hk"], c["D"])
    finally:
        for h in handles:
            h.remove()
        hc.uninstall_monkeypatch()
        hc.set_active_kvctrl(None)
    return res, inp, ctrl, prompt_state, float(np.median(times))


def _check_layer(c, res, inp, model):
    # the oracle rotates with the model's own inverse frequencies (computed on the GPU, they can
    # differ from a CPU computation in the last place)
    kw = dict(oracle_kwargs(c), inv_freq=model.model.rotary_emb.inv_freq.float().cpu().numpy())
    layer, o_outs, o_hot, fc = run_following(O, inp, c["steps"], res, **kw)
    assert assert_same_run(res, layer, o_outs, o_hot, c["dtype"], c["steps"], "layer 0") == c["steps"]
    return layer, fc


def test_config1_llama8b_8k_budget512(model):
    c = _case(1)
    res, inp, ctrl, _, us = _run(model, c, seed=11)
    layer, _ = _check_layer(c, res, inp, model)
    assert [e["step"] for e in layer.events] == [15, 31, 47, 63]
    L = model.config.num_hidden_layers
    assert ctrl.dbg["retrieval_launched"] == 4 * L and ctrl.dbg["injection_used"] == (STEPS - 14) * L
    assert ctrl.device_status() == 0
    print(f"config 1: {us:.0f} us per decode token through the patched 32-layer forward")


def test_config2_llama8b_planted_key_is_retrieved(model):
    c = _case(2)
    rng = np.random.default_rng(2)
    p = int(rng.integers(0, c["T"] // 4))
    res, inp, ctrl, prompt_state, us = _run(model, c, seed=12, plant=p)
    L = model.config.num_hidden_layers
    assert 1 in res["held"] and res["held_all"]
    kept = evicted = 0
    for li, (hot, cold) in enumerate(prompt_state):
        in_hot, in_cold = p in set(hot.tolist()), p in set(cold.tolist())
        assert in_hot != in_cold, f"layer {li}: the planted token must be in exactly one tier"
        pos, valid = res["held_all"][li]
        if in_hot:
            kept += 1
        else:
            evicted += 1
            assert p in set(pos[valid].tolist()), f"layer {li} evicted the planted token and did not retrieve it"
    _check_layer(c, res, inp, model)
    assert ctrl.device_status() == 0
    print(f"config 2: planted token {p}: kept hot in {kept} layers, evicted and retrieved at step 1 in {evicted}; "
          f"{us:.0f} us per decode token")
