"""The patched LlamaAttention.forward (patch.py:13-350 of src/hotcold_kv).

Prompt forwards keep the reference's structure: projections, HF RoPE, stock
causal SDPA over the whole prompt, then the prompt goes into the hot tier
(compressed, evicted tokens into the cold ring) and the prompt-end retrieval
runs. A further multi-token forward on a non-empty cache (a prompt sent in
chunks, which the reference rejects) attends to the kept hot tokens and joins
them (KVController.prefill_chunk). A one-token decode forward runs the sm_100a
hot path of the layer: RoPE + append, the scheduled retrieval, compression,
attention over [held | hot] — without host synchronisation.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from transformers.cache_utils import Cache
from transformers.models.llama import modeling_llama

from .cache import HotColdLayer
from .datatypes import _canon_br_2d, _canon_kv_4d
from .kernels import triton_evict_attention_forward

ACTIVE_KVCTRL = None
ACTIVE_ROTARY_EMB = None  # set to model.model.rotary_emb


def set_active_kvctrl(kvctrl):
    global ACTIVE_KVCTRL
    ACTIVE_KVCTRL = kvctrl


def set_active_rotary_emb(rotary_emb_module):
    global ACTIVE_ROTARY_EMB
    ACTIVE_ROTARY_EMB = rotary_emb_module


def _rope_cos_sin_for_positions(pos_ids: torch.Tensor, dtype: torch.dtype, device: torch.device, head_dim: int):
    """cos/sin (B,R,D) of the active rotary module at arbitrary positions (patch.py:76-91)."""
    if ACTIVE_ROTARY_EMB is None:
        raise RuntimeError("ACTIVE_ROTARY_EMB is None. Call set_active_rotary_emb(model.model.rotary_emb).")
    pos_ids = _canon_br_2d(pos_ids, "pos_ids").to(device=device, dtype=torch.long)
    B, S = pos_ids.shape
    x = torch.empty((B, 1, S, head_dim), device=device, dtype=dtype)
    try:
        cos, sin = ACTIVE_ROTARY_EMB(x, pos_ids)
    except TypeError:
        cos, sin = ACTIVE_ROTARY_EMB(x, position_ids=pos_ids)
    return cos.reshape(B, S, head_dim), sin.reshape(B, S, head_dim)


def _rotate_k_with_pos(k_pre: torch.Tensor, pos_ids: torch.Tensor, head_dim: int):
    """Re-rotate pre-RoPE keys (B,Hk,R,D) to their positions (B,R) (patch.py:94-102).
    cos/sin are taken per sequence, so batches larger than one rotate correctly."""
    k_pre = _canon_kv_4d(k_pre, "k_pre")
    pos_ids = _canon_br_2d(pos_ids, "pos_ids")
    cos, sin = _rope_cos_sin_for_positions(pos_ids, k_pre.dtype, k_pre.device, head_dim)
    q_dummy = torch.zeros_like(k_pre)
    _, k_out = modeling_llama.apply_rotary_pos_emb(q_dummy, k_pre, cos, sin, unsqueeze_dim=1)
    return k_out


_ORIG = None


def uninstall_monkeypatch():
    global _ORIG
    if _ORIG is not None:
        modeling_llama.LlamaAttention.forward = _ORIG
        _ORIG = None


def install_monkeypatch(enable_debug: bool = True):
    global _ORIG
    if _ORIG is not None:
        return
    _ORIG = modeling_llama.LlamaAttention.forward

    def patched_forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor],
                        attention_mask: Optional[torch.Tensor] = None, past_key_values: Optional[Cache] = None,
                        cache_position: Optional[torch.LongTensor] = None, **kwargs):
        kvctrl = ACTIVE_KVCTRL
        if kvctrl is None:
            return _ORIG(self, hidden_states=hidden_states, position_embeddings=position_embeddings,
                         attention_mask=attention_mask, past_key_values=past_key_values,
                         cache_position=cache_position, **kwargs)
        num_heads = int(self.config.num_attention_heads)
        num_kv_heads = int(getattr(self.config, "num_key_value_heads", num_heads))
        head_dim = int(self.head_dim) if hasattr(self, "head_dim") else int(self.config.hidden_size // num_heads)
        bsz, q_len, _ = hidden_states.shape
        device = hidden_states.device

        q_pre = self.q_proj(hidden_states).view(bsz, q_len, num_heads, head_dim).transpose(1, 2)
        k_pre = self.k_proj(hidden_states).view(bsz, q_len, num_kv_heads, head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, q_len, num_kv_heads, head_dim).transpose(1, 2)
        kvctrl._lazy_init(k_pre, n_layers=int(self.config.num_hidden_layers))
        cos, sin = position_embeddings
        li = int(self.layer_idx)

        layer = None
        if past_key_values is not None and isinstance(past_key_values, Cache):
            layer = past_key_values.layers[li]
            if not isinstance(layer, HotColdLayer):
                layer = None
            elif layer.layer_idx is None:
                layer.layer_idx = li
        hot_prev_len = int(past_key_values.get_seq_length(li)) if past_key_values is not None else 0

        # absolute positions of this forward's tokens: cache_position, else the tokens this layer has
        # already seen (the hot tier's physical length is shorter once it has been compressed)
        if cache_position is not None and int(cache_position.numel()) == q_len:
            pos_new = cache_position.reshape(1, -1).expand(bsz, -1).to(device=device, dtype=torch.long)
        else:
            start = kvctrl.seen_tokens(li) if layer is not None else hot_prev_len
            pos_new = torch.arange(start, start + q_len, device=device, dtype=torch.long).unsqueeze(0).expand(bsz, -1)
        n_rep = num_heads // num_kv_heads

        if q_len == 1 and layer is not None:
            # decode: the sm_100a hot path of this layer. RoPE is applied at pos_new from the rotary
            # module's inv_freq inside the kernel, not from position_embeddings: transformers 5.x
            # derives a decode step's position ids from get_seq_length(), which is the compressed
            # (physical) hot length here, as in the reference, so its cos/sin belong to the wrong
            # position once the prompt has been compressed.
            attn = kvctrl.decode_layer(li, q_pre[:, :, 0], k_pre[:, :, 0], v[:, :, 0], None, None,
                                       pos_new[:, 0].contiguous())
            attn_out = attn.reshape(bsz, 1, num_heads * head_dim)
        elif q_len > 1 and layer is not None and kvctrl.seen_tokens(li) > 0:
            # a further chunk of a prompt (the reference raises here, patch.py:325-329): RoPE at the
            # chunk's absolute positions; its queries attend to the kept hot tokens and causally to
            # each other; then its tokens join the hot tier, which is compressed into the cold store
            cos_c, sin_c = _rope_cos_sin_for_positions(pos_new, q_pre.dtype, device, head_dim)
            q_post, k_post = modeling_llama.apply_rotary_pos_emb(q_pre, k_pre, cos_c, sin_c)
            a = kvctrl.arenas[li]
            hk, hv, _, _ = a.hot_dense()
            k_all, v_all = torch.cat([hk, k_post], 2), torch.cat([hv, v], 2)
            n_prev = int(hk.shape[2])
            mask = torch.ones((q_len, n_prev + q_len), dtype=torch.bool, device=device)
            mask[:, n_prev:] = torch.ones((q_len, q_len), dtype=torch.bool, device=device).tril()
            k_rep = modeling_llama.repeat_kv(k_all, n_rep) if n_rep > 1 else k_all
            v_rep = modeling_llama.repeat_kv(v_all, n_rep) if n_rep > 1 else v_all
            attn = F.scaled_dot_product_attention(q_post, k_rep, v_rep, attn_mask=mask[None, None], dropout_p=0.0)
            kvctrl.prefill_chunk(li, q_pre, q_post, k_pre, k_post, v, pos_new, last=True)
            attn_out = attn.transpose(1, 2).reshape(bsz, q_len, -1)
        else:
            q_post, k_post = modeling_llama.apply_rotary_pos_emb(q_pre, k_pre, cos, sin)
            if q_len > 1:
                k_rep = modeling_llama.repeat_kv(k_post, n_rep) if n_rep > 1 else k_post
                v_rep = modeling_llama.repeat_kv(v, n_rep) if n_rep > 1 else v
                attn = F.scaled_dot_product_attention(q_post, k_rep, v_rep, attn_mask=attention_mask, dropout_p=0.0,
                                                      is_causal=attention_mask is None)
                if layer is not None:
                    kvctrl.prefill_layer(li, q_pre, q_post, k_pre, k_post, v, pos_new)
                elif past_key_values is not None:
                    past_key_values.update(k_post, v, layer_idx=li, cache_kwargs={
                        "cache_position": cache_position, "pre_key_states": k_pre, "positions": pos_new})
            else:
                # one-token forward without a hot/cold layer: the stand-alone kernel
                if past_key_values is not None:
                    k_post, v = past_key_values.update(k_post, v, layer_idx=li, cache_kwargs={
                        "cache_position": cache_position, "pre_key_states": k_pre, "positions": pos_new})
                mask = torch.ones((bsz, k_post.shape[2]), dtype=torch.bool, device=device)
                out, _ = triton_evict_attention_forward(q_post, k_post, v, mask, n_rep, 1.0 / math.sqrt(head_dim))
                attn = out.transpose(1, 2)
            attn_out = attn.transpose(1, 2).reshape(bsz, q_len, -1)
        attn_out = self.o_proj(attn_out)

        if enable_debug and kvctrl._inited and li == 0 and kvctrl.step_count and kvctrl.step_count[0] % 50 == 0:
            ready_rate = kvctrl.dbg["prefetch_ready"] / max(1, kvctrl.dbg["prefetch_launched"])
            print("[DBG]", "step0", kvctrl.step_count[0], "hot0", hot_prev_len, "cold0", kvctrl.cold_size(0),
                  "ready_rate", round(ready_rate, 3))
        return attn_out, None

    modeling_llama.LlamaAttention.forward = patched_forward
