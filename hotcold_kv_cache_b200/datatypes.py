"""Transfer objects and shape canonicalisers of the hot/cold path, with the
reference's names and fields (datatypes.py:8-63 of src/hotcold_kv)."""

from dataclasses import dataclass

import torch


def _canon_kv_4d(x: torch.Tensor, name: str) -> torch.Tensor:
    """Squeeze extra singleton dims (never the batch dim) down to (B,Hk,R,D);
    RuntimeError otherwise (datatypes.py:8-27)."""
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a Tensor")
    while x.dim() > 4:
        for d in range(1, x.dim()):
            if x.shape[d] == 1:
                x = x.squeeze(d)
                break
        else:
            break
    if x.dim() != 4:
        raise RuntimeError(f"{name} must be 4D (B,Hk,R,D); got {tuple(x.shape)}")
    return x


def _canon_br_2d(x: torch.Tensor, name: str) -> torch.Tensor:
    """Squeeze extra singleton dims down to (B,R) (datatypes.py:29-44)."""
    if not isinstance(x, torch.Tensor):
        raise RuntimeError(f"{name} must be a Tensor")
    while x.dim() > 2:
        for d in range(1, x.dim()):
            if x.shape[d] == 1:
                x = x.squeeze(d)
                break
        else:
            break
    if x.dim() != 2:
        raise RuntimeError(f"{name} must be 2D (B,R); got {tuple(x.shape)}")
    return x


@dataclass
class RetrievedKV:
    """A retrieved set (datatypes.py:50-56). Here the tensors are device views of
    the held segment: k_pre (B,Hk,R,D) pre-RoPE keys gathered from the cold ring,
    v (B,Hk,R,D), pos (B,R) int64, valid (B,R) bool."""
    k_pre: torch.Tensor
    v: torch.Tensor
    pos: torch.Tensor
    valid: torch.Tensor
    ready: bool = False


@dataclass
class EvictedKV:
    """Evicted tokens handed to the cold store (datatypes.py:58-63): k_pre/v
    (B,Hk,Te,D), pos (B,Te) int64, evicted_idx (B,Te) int64 padded with -1.
    The reference stages them in pinned host memory; here they may live on the
    host or the device."""
    k_pre_cpu: torch.Tensor
    v_cpu: torch.Tensor
    pos_cpu: torch.Tensor
    evicted_idx: torch.Tensor
