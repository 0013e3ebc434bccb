"""Stand-alone decode attention with the reference's kernel-wrapper signature.

`triton_evict_attention_forward` keeps the name, arguments, return values and
errors of the reference wrapper (kernels.py:77-137) and runs the sm_100a
split-K flash-decode kernel of this package. There is no Triton and no CPU
path: inputs must be CUDA tensors.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr, size

_counters: dict = {}
_scratch: dict = {}


def _buffers(device, n_counters: int, nbytes: int):
    key = (device.type, device.index)
    c = _counters.get(key)
    if c is None or c.numel() < n_counters:
        c = torch.zeros(max(n_counters, 1024), dtype=torch.int32, device=device)
        _counters[key] = c
    s = _scratch.get(key)
    if s is None or s.numel() < nbytes:
        s = torch.empty(int(nbytes * 1.25) + 4096, dtype=torch.uint8, device=device)
        _scratch[key] = s
    return c, s


def triton_evict_attention_forward(
    query: torch.Tensor,           # [B, Hq, 1, D]
    key: torch.Tensor,             # [B, Hk, S, D]
    value: torch.Tensor,           # [B, Hk, S, D]
    attention_mask: torch.Tensor,  # [B, S] bool, True = attend
    num_key_value_groups: int,
    scaling: float,
    dropout: float = 0.0,
    block_s: int = 64,
    overflow_nan: bool = True,
):
    """Returns (attn_out [B,1,Hq,D] contiguous, evict_idx [B] int64) like the reference:
    attention over keys where the mask is True, and the argmin over tokens of the
    head-mean softmax probability times mean |v| (kernels.py:134-137). `block_s` is
    accepted for signature compatibility; the kernel picks its own chunking."""
    assert query.is_cuda and key.is_cuda and value.is_cuda and attention_mask.is_cuda
    if dropout != 0.0:
        raise ValueError("dropout must be 0.0 , because we are not in training")
    query = query.contiguous()
    key = key.contiguous()
    value = value.contiguous()
    attention_mask = attention_mask.contiguous()
    B, Hq, _, D = query.shape
    _, Hk, S, _ = key.shape
    if Hq // num_key_value_groups != Hk:
        raise ValueError(f"Hq({Hq})//N_REP({num_key_value_groups}) must equal Hk({Hk})")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise TypeError("query, key and value must share a dtype")
    mask = attention_mask.to(torch.uint8) if attention_mask.dtype != torch.uint8 else attention_mask
    out = torch.empty((B, Hq, D), dtype=query.dtype, device=query.device)
    evict_idx = torch.empty((B,), dtype=torch.int64, device=query.device)
    nbytes = size("hc_attention_dense_scratch_bytes", B, Hq, Hk, S, D)
    counters, scratch = _buffers(query.device, B * Hk, nbytes)
    with torch.cuda.device(query.device):
        call("hc_attention_dense", ptr(query), ptr(key), ptr(value), ptr(mask), ptr(out), ptr(evict_idx), B, Hq, Hk, S,
             D, _lib.dtype_code(query.dtype), float(scaling), 1 if overflow_nan else 0, ptr(counters), ptr(scratch),
             scratch.numel(), _lib.stream_of(query.device))
    return out.view(B, 1, Hq, D), evict_idx
