"""ctypes binding of the sm_100a library (include/hotcold_b200.h).

The library is built in-tree by `hotcold_kv_cache_b200.build` into
`_lib/libhotcold_b200.so`. There is no fallback: if the library is missing or
the device is not CUDA, every op raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, byref, c_double, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p,
                    c_char_p)

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libhotcold_b200.so")

HC_F32, HC_F16, HC_BF16 = 0, 1, 2
HC_POLICY_HOTCOLD, HC_POLICY_SNAPKV = 0, 1
HC_POOL_MAX, HC_POOL_AVG = 0, 1
HC_DEV_CAPACITY, HC_DEV_TIMEOUT, HC_DEV_INDEX = 1, 2, 4


class HcSeqState(Structure):
    _fields_ = [("n_hot", c_int32), ("n_free", c_int32), ("cold_head", c_int32), ("cold_count", c_int32),
                ("held_len", c_int32), ("n_hits", c_int32), ("qwin_head", c_int32), ("n_evict", c_int32),
                ("status", c_int32), ("pad", c_int32 * 7)]


class HcSeqDesc(Structure):
    _fields_ = [("hot_k", c_void_p), ("hot_v", c_void_p), ("hot_kpre", c_void_p), ("hot_pos", c_void_p),
                ("hot_ord", c_void_p), ("hot_free", c_void_p), ("held_k", c_void_p), ("held_v", c_void_p),
                ("held_pos", c_void_p), ("held_valid", c_void_p), ("held_src", c_void_p), ("cold_vec", c_void_p),
                ("cold_kpre", c_void_p), ("cold_v", c_void_p), ("cold_pos", c_void_p), ("qwin", c_void_p),
                ("st", c_void_p), ("cap", c_int32), ("budget", c_int32), ("r_max", c_int32), ("ccap", c_int32),
                ("p_max", c_int32), ("pad", c_int32 * 1)]


class HcLayer(Structure):
    _fields_ = [("desc", c_void_p), ("inv_freq", c_void_p), ("counters", c_void_p), ("topk_ratio", c_double),
                ("n_seq", c_int32), ("Hq", c_int32), ("Hk", c_int32), ("D", c_int32), ("F", c_int32),
                ("dtype", c_int32), ("policy", c_int32), ("recent", c_int32), ("pool_kernel", c_int32),
                ("pooling", c_int32), ("normalize", c_int32), ("max_cap", c_int32), ("max_r", c_int32),
                ("max_ccap", c_int32), ("scale", c_float), ("rope_scaling", c_float), ("kmaps", c_void_p)]


assert ctypes.sizeof(HcSeqState) == 64
assert ctypes.sizeof(HcSeqDesc) == 160
assert ctypes.sizeof(HcLayer) == 104

_P = c_void_p
_I64 = c_int64
# name -> (restype, argtypes); mirrors include/hotcold_b200.h
SIGNATURES = {
    "hc_version": (c_char_p, []),
    "hc_host_device_pointer": (c_int, [_P, POINTER(c_void_p)]),
    "hc_last_error": (c_char_p, []),
    "hc_attention_dense_scratch_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "hc_attention_dense": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                   _P, _P, c_size_t, _P]),
    "hc_attention_dense_noalloc": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int,
                                           c_float, c_int, _P]),
    "hc_append": (c_int, [_P, _P, _I64, _P, _P, _I64, _P, _P, _P, _P, _P]),
    "hc_append_rotated": (c_int, [_P, _P, _P, _P, _I64, _P, _P]),
    "hc_cold_append": (c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _P, c_int, _P]),
    "hc_compress_scratch_bytes": (c_size_t, [_P, c_int, c_int]),
    "hc_compress": (c_int, [_P, _P, _I64, _I64, _I64, c_int, c_int, _P, _P, _P, _I64, _I64, _I64, _P, _P, c_size_t,
                            _P]),
    "hc_compress_ex": (c_int, [_P, _P, _I64, _I64, _I64, c_int, c_int, _P, _P, _P, _I64, _I64, _I64, _P, _P,
                               c_size_t, c_int, _P]),
    "hc_store_prompt": (c_int, [_P, c_int, _P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "hc_retrieve_scratch_bytes": (c_size_t, [_P]),
    "hc_retrieve": (c_int, [_P, _P, _I64, _I64, _I64, c_int, c_int, _P, c_int, _P, c_size_t, _P]),
    "hc_retrieve_ex": (c_int, [_P, _P, _I64, _I64, _I64, c_int, c_int, _P, c_int, _P, _P, c_size_t, c_int, _P]),
    "hc_prompt_query_sum_scratch_bytes": (c_size_t, [_P]),
    "hc_prompt_query_sum": (c_int, [_P, _P, _I64, _I64, _I64, c_int, _P, _P, c_size_t, _P]),
    "hc_attend_scratch_bytes": (c_size_t, [_P]),
    "hc_attend": (c_int, [_P, _P, _P, c_int, _P, c_int, _P, c_size_t, _P]),
    "hc_shard_merge": (c_int, [_P, _P, c_int, c_int, _P, _P, _P]),
    "hc_cold_topk_scratch_bytes": (c_size_t, [c_int64, c_int]),
    "hc_cold_topk": (c_int, [_P, c_int64, c_int, c_int64, _P, c_int, _P, _P, _P, c_size_t, _P]),
    "hc_splice_hits": (c_int, [_P, _P, c_int, _P]),
    "hc_retrieve_query": (c_int, [_P, _P, c_int64, c_int64, c_int64, c_int, c_int, _P, c_int, _P, _P]),
    "hc_step_check": (c_int, [_P, c_int]),
    "hc_retrieve_decode": (c_int, [_P, _P, _I64, c_int, _P, c_size_t, _P]),
    "hc_encode_kmap": (c_int, [_P, _P, c_int, _I64, c_int, c_int]),
    "hc_step": (c_int, [_P, _P, _I64, _P, _P, _I64, _P, _P, _P, c_int, _P, c_int, c_int, _P]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the library (once) and attach the prototypes. Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"hotcold_b200 CUDA library not built: {path} is missing "
                           "(run `python -m hotcold_kv_cache_b200.build`)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call an hc_* entry point; raise RuntimeError with hc_last_error() on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.hc_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (code {rc}): {msg}")


def size(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))


def ptr(t) -> int | None:
    """Device address of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


_RAW_STREAM = []  # torch's raw current-stream getter, looked up once (None when absent)


def stream_of(device) -> int:
    """The raw handle of the current CUDA stream of `device`."""
    import torch
    if not _RAW_STREAM:
        _RAW_STREAM.append(getattr(torch._C, "_cuda_getCurrentRawStream", None))
    idx = getattr(device, "index", None)
    if idx is None:
        idx = torch.cuda.current_device()
    raw = _RAW_STREAM[0]
    if raw is not None:
        return raw(idx)
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype) -> int:
    import torch
    codes = {torch.float32: HC_F32, torch.float16: HC_F16, torch.bfloat16: HC_BF16}
    if dtype not in codes:
        raise TypeError(f"unsupported dtype {dtype}; float32, float16 or bfloat16")
    return codes[dtype]


__all__ = ["load", "call", "size", "ptr", "stream_of", "dtype_code", "HcLayer", "HcSeqDesc", "HcSeqState", "byref",
           "SIGNATURES", "LIB_PATH", "POINTER"]
