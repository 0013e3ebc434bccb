"""Seeded synthetic inputs for the hot/cold decode path.

The reference measures on LongBench prompts run through Llama-3.1-8B
(`benchmarks/run_baselines.py:66-96`). Neither the dataset nor the weights
exist here, so every workload is drawn from a seed with the shapes of those
runs: pre-RoPE queries, keys and values i.i.d. N(0, 1), 32 query heads,
8 KV heads, head_dim 128, RoPE theta 500000.

Draws use numpy's PCG64 generator, which gives the same numbers on every
machine, so the CPU checker and the GPU path see identical inputs.
"""

from __future__ import annotations

import numpy as np

LLAMA31_8B = dict(Hq=32, Hk=8, D=128, theta=500000.0)

_NP_DTYPES = {"float32": np.float32, "float16": np.float16}


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); float32 out."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    b = f.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def to_model_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round a float array to `dtype`. bfloat16 values are carried in float32."""
    if dtype == "bfloat16":
        return round_bf16(x)
    return np.asarray(x).astype(_NP_DTYPES[dtype])


def rope_inv_freq(D: int, theta: float) -> np.ndarray:
    """Default RoPE inverse frequencies, bit-identical to HF's
    `LlamaRotaryEmbedding.compute_default_rope_parameters` (torch float32 pow;
    numpy's float32 pow differs in the last place for some exponents)."""
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(dtype=torch.float) / D))
    return inv.numpy().astype(np.float32)


def layer_inputs(seed: int, B: int, Hq: int, Hk: int, D: int, T: int, n_steps: int,
                 dtype: str = "float32") -> dict:
    """One layer's prefill and decode inputs (pre-RoPE), drawn from `seed`.

    Returns a dict of numpy arrays in `dtype` (bfloat16 carried in float32):
      q_pre (B,Hq,T,D), k_pre (B,Hk,T,D), v (B,Hk,T,D) for the prompt and
      dq (n,B,Hq,D), dk (n,B,Hk,D), dv (n,B,Hk,D) for n decode steps.
    Positions are 0..T-1 for the prompt and T+i at decode step i.
    """
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in (("q_pre", (B, Hq, T, D)), ("k_pre", (B, Hk, T, D)), ("v", (B, Hk, T, D)),
                        ("dq", (n_steps, B, Hq, D)), ("dk", (n_steps, B, Hk, D)),
                        ("dv", (n_steps, B, Hk, D))):
        out[name] = to_model_dtype(rng.standard_normal(shape, dtype=np.float32), dtype)
    return out


def ragged_batch(seed: int, n_seq: int = 64, lo: int = 2048, hi: int = 32768,
                 budgets=(512, 1024, 2048)) -> list[tuple[int, int]]:
    """Sequence lengths uniform in [lo, hi] and budgets cycling over `budgets`
    (the ragged continuous batch of the multi-sequence configuration)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n_seq)
    return [(int(L), int(budgets[i % len(budgets)])) for i, L in enumerate(lens)]


def balanced_partition(items: list[tuple[int, int]], n_parts: int) -> list[list[int]]:
    """Longest-processing-time greedy: sort by load (length + budget) descending and
    give each sequence to the least-loaded part. Returns sequence ids per part,
    each list ascending."""
    order = sorted(range(len(items)), key=lambda i: (-(items[i][0] + items[i][1]), i))
    loads = [0] * n_parts
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        p = min(range(n_parts), key=lambda j: (loads[j], j))
        parts[p].append(i)
        loads[p] += items[i][0] + items[i][1]
    return [sorted(p) for p in parts]


def score_case_inputs(seed: int, Hq: int = 32, Hk: int = 8, D: int = 128, S: int = 700):
    """Inputs of the function-level eviction-score check: for float32 then float16,
    (q (1,Hq,S,D), k (1,Hk,S,D)) in that dtype (float16 as numpy float16)."""
    rng = np.random.default_rng(seed)
    out = {}
    for dt in ("float32", "float16"):
        q = to_model_dtype(rng.standard_normal((1, Hq, S, D), dtype=np.float32), dt)
        k = to_model_dtype(rng.standard_normal((1, Hk, S, D), dtype=np.float32), dt)
        out[dt] = (q, k)
    return out


def attention_case_inputs(seed: int, B: int = 2, Hq: int = 8, Hk: int = 2, S: int = 200, D: int = 128,
                          keep_frac: float = 0.8):
    """Inputs of the stand-alone decode-attention check (float32):
    q (B,Hq,1,D), k/v (B,Hk,S,D), mask (B,S) bool."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, Hq, 1, D), dtype=np.float32)
    k = rng.standard_normal((B, Hk, S, D), dtype=np.float32)
    v = rng.standard_normal((B, Hk, S, D), dtype=np.float32)
    m = rng.random((B, S)) < keep_frac
    return q, k, v, m


# the Llama-3.1-8B architecture with random weights (no checkpoint here)
LLAMA31_8B_MODEL = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                        num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=500000.0,
                        max_position_embeddings=131072, rms_norm_eps=1e-5, initializer_range=0.02)


def llama8b_random(device, seed: int, layers: int = 32, dtype=None):
    """A random-init Llama-3.1-8B (vocab 128256, hidden 4096, 32/8 heads, head_dim 128, RMSNorm,
    SwiGLU FFN 14336, RoPE theta 500000; linear and embedding weights N(0, 0.02)) built directly
    on `device` in `dtype` (fp16 by default), in eval mode."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(**dict(LLAMA31_8B_MODEL, num_hidden_layers=layers))
    with torch.device(device):
        model = LlamaForCausalLM._from_config(cfg, dtype=dtype or torch.float16)
    return model.eval().requires_grad_(False)


def plant_key(model, pos: int):
    """BASELINE config 2's planted key: in the prompt forward, every layer's pre-RoPE key at
    position `pos`, for each KV head, becomes 4 x the mean over that head's GQA group of the
    layer's final-token pre-RoPE query heads (forward hooks on q_proj and k_proj; one-token
    forwards are left alone). Returns the hook handles (call .remove() on each)."""
    handles = []
    for layer in model.model.layers:
        att = layer.self_attn
        Hq, Hk = att.config.num_attention_heads, att.config.num_key_value_heads
        D = att.head_dim
        stash = {}

        def qhook(mod, inp, out, stash=stash):
            stash["q"] = out

        def khook(mod, inp, out, stash=stash, Hq=Hq, Hk=Hk, D=D):
            if out.shape[1] <= pos:
                return out
            q = stash["q"][:, -1].float().view(out.shape[0], Hk, Hq // Hk, D).mean(2)  # (B, Hk, D)
            out = out.clone()
            out[:, pos] = (4.0 * q).reshape(out.shape[0], Hk * D).to(out.dtype)
            return out

        handles.append(att.q_proj.register_forward_hook(qhook))
        handles.append(att.k_proj.register_forward_hook(khook))
    return handles
