"""HotColdLayer: the HuggingFace cache layer of the hot tier (cache.py:12-173 of
src/hotcold_kv). The hot tokens live in the layer's HBM slab owned by the
KVController; `keys`, `values`, `pre_keys` and `positions` are materialised in
logical order on access (they are not on the decode path)."""

from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from .controller import KVController


class HotColdLayer(CacheLayerMixin):
    is_compileable = False

    def __init__(self, kvctrl: KVController, layer_idx: Optional[int] = None):
        super().__init__()
        self.kvctrl = kvctrl
        self.layer_idx = layer_idx
        self.is_initialized = False
        self._last_q_post: Optional[torch.Tensor] = None

    # the reference stores tensors in these attributes; here they are views of the slab
    def _arena(self):
        c = self.kvctrl
        if self.layer_idx is None or not c._inited or c.arenas[self.layer_idx] is None:
            return None
        return c.arenas[self.layer_idx]

    @property
    def keys(self):
        a = self._arena()
        return None if a is None else a.hot_view("k")

    @keys.setter
    def keys(self, _):
        pass

    @property
    def values(self):
        a = self._arena()
        return None if a is None else a.hot_view("v")

    @values.setter
    def values(self, _):
        pass

    @property
    def pre_keys(self):
        a = self._arena()
        return None if a is None else a.hot_view("kpre")

    @property
    def positions(self):
        a = self._arena()
        return None if a is None else a.hot_positions()

    def set_last_query_post(self, q_post: torch.Tensor):
        """cache.py:25-26: post-RoPE queries that score the next compression."""
        self._last_q_post = q_post

    def lazy_initialization(self, key_states: torch.Tensor, value_states: Optional[torch.Tensor] = None):
        self.is_initialized = True

    def update(self, layer_idx: int, key_states: torch.Tensor, value_states: torch.Tensor,
               cache_kwargs: Optional[dict[str, Any]] = None):
        """cache.py:130-151: append post-RoPE keys, values, pre-RoPE keys and positions,
        compress when over budget, return (keys, values) in logical order. A multi-token
        call on an empty layer stores a prompt; a one-token call appends."""
        if self.layer_idx is None:
            self.layer_idx = int(layer_idx)
        if not self.is_initialized:
            self.lazy_initialization(key_states)
        c = self.kvctrl
        B, Hk, T, D = key_states.shape
        if not c._inited:
            c._lazy_init(key_states, n_layers=max(int(layer_idx) + 1, 1))
        pre_k = pos = None
        if cache_kwargs is not None:
            pre_k = cache_kwargs.get("pre_key_states")
            pos = cache_kwargs.get("positions")
        if pre_k is None or pos is None:
            pre_k = torch.zeros_like(key_states)
            pos = torch.zeros((B, T), device=key_states.device, dtype=torch.long)
        q = self._last_q_post
        a = c.arena(layer_idx, q.shape[1] if q is not None else Hk, key_states.dtype, key_states.device)
        if a.n_hot.max() == 0:
            if q is None:
                q = torch.zeros((B, Hk, 1, D), dtype=key_states.dtype, device=key_states.device)
            r = c.recent_size
            q_obs = q if q.shape[2] <= r else q[:, :, -r:, :]
            c._count_eviction(a.compress_prompt(q_obs, key_states, value_states, pre_k, pos.to(torch.long)))
        else:
            for t in range(T):
                a.append_rotated(key_states[:, :, t], pre_k[:, :, t], value_states[:, :, t],
                                 pos[:, t].to(torch.long).contiguous())
                if q is not None:
                    c._count_eviction(a.compress_decode(q[:, :, -1:, :] if q.shape[2] > 1 else q))
        return self.keys, self.values

    def get_mask_sizes(self, cache_position) -> Tuple[int, int]:
        """Accepts the query length as an int (transformers 5.x) or a cache_position
        tensor (transformers 4.x, cache.py:153-156)."""
        q = cache_position if isinstance(cache_position, int) else int(cache_position.shape[0])
        return int(self.get_seq_length() + q), 0

    def get_seq_length(self) -> int:
        a = self._arena()
        return 0 if a is None else int(a.n_hot.max())

    def get_max_cache_shape(self) -> int:
        return int(self.kvctrl.max_capacity_prompt)


def build_hotcold_cache(model, kvctrl: KVController) -> Cache:
    """cache.py:170-173: one HotColdLayer per decoder layer."""
    n_layers = int(model.config.num_hidden_layers)
    return Cache(layers=[HotColdLayer(kvctrl, layer_idx=i) for i in range(n_layers)])
