"""B200-native (sm_100a) hot/cold KV decode path.

Drop-in for the public API of tarun931/hotcold-kv-cache (`hotcold_kv`,
__init__.py:4-26): the same names, with the per-decode-step hot path (attention
over the hot cache and the held retrieved set, compression with eviction into
an HBM cold store, exact inner-product retrieval, re-RoPE splice) running as
hand-written CUDA kernels through the C ABI in include/hotcold_b200.h.

Importing the package does not load the CUDA library; the first op does, and
raises if it is missing.
"""

from .datatypes import EvictedKV, RetrievedKV

__all__ = [
    "RetrievedKV",
    "EvictedKV",
    "triton_evict_attention_forward",
    "KVController",
    "HotColdLayer",
    "build_hotcold_cache",
    "set_active_kvctrl",
    "set_active_rotary_emb",
    "install_monkeypatch",
    "uninstall_monkeypatch",
]


def __getattr__(name):
    if name == "triton_evict_attention_forward":
        from .kernels import triton_evict_attention_forward
        return triton_evict_attention_forward
    if name == "KVController":
        from .controller import KVController
        return KVController
    if name in ("HotColdLayer", "build_hotcold_cache"):
        from . import cache
        return getattr(cache, name)
    if name in ("set_active_kvctrl", "set_active_rotary_emb", "install_monkeypatch", "uninstall_monkeypatch"):
        from . import patch
        return getattr(patch, name)
    raise AttributeError(name)
