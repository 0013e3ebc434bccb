"""CPU checks of the C ABI: the library loads without a GPU, exports every
entry point include/hotcold_b200.h declares, the ctypes prototypes cover them,
and the struct sizes agree with the header; nothing falls back to the host."""

import ctypes
import os
import re

import pytest

from hotcold_kv_cache_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hotcold_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^HC_API\s+[\w\s\*]+?\b(hc_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "hc_attend" in names and "hc_compress" in names and "hc_retrieve" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.hc_version().startswith(b"hotcold_b200")


def test_prototypes_cover_header():
    assert set(declared()) == set(_lib.SIGNATURES)


def test_struct_sizes_match_header_comments():
    src = open(HEADER).read()
    for cname, pyt in (("hc_seq_state", _lib.HcSeqState), ("hc_seq_desc", _lib.HcSeqDesc),
                       ("hc_layer", _lib.HcLayer)):
        m = re.search(r"\}\s*" + cname + r";\s*/\*\s*(\d+) bytes", src)
        assert m, cname
        assert ctypes.sizeof(pyt) == int(m.group(1)), cname


def test_scratch_queries_run_without_gpu():
    n = _lib.size("hc_attention_dense_scratch_bytes", 1, 32, 8, 577, 128)
    assert n > 0
    L = _lib.HcLayer()
    L.n_seq, L.Hq, L.Hk, L.D, L.F, L.max_cap, L.max_r, L.max_ccap = 1, 32, 8, 128, 128, 513, 64, 32768
    assert _lib.size("hc_attend_scratch_bytes", ctypes.byref(L)) > 0
    assert _lib.size("hc_retrieve_scratch_bytes", ctypes.byref(L)) >= 32768 * 5
    assert _lib.size("hc_compress_scratch_bytes", ctypes.byref(L), 8192, 32) > 8 * 32 * 8192 * 4


def test_argument_errors_are_reported_not_launched():
    lib = _lib.load()
    rc = lib.hc_attend(None, None, None, 0, None, 1, None, 0, None)
    assert rc != 0 and b"NULL" in lib.hc_last_error()
    L = _lib.HcLayer()
    L.desc = 1
    L.n_seq, L.Hq, L.Hk, L.D = 1, 30, 8, 128
    rc = lib.hc_append(ctypes.byref(L), None, 0, None, None, 0, None, None, None, None, None)
    assert rc != 0 and b"multiple" in lib.hc_last_error()
    L.Hq, L.D = 32, 96
    rc = lib.hc_append(ctypes.byref(L), None, 0, None, None, 0, None, None, None, None, None)
    assert rc == 3 and b"head_dim" in lib.hc_last_error()
    rc = lib.hc_shard_merge(None, None, 8, 1024, None, None, None)
    assert rc != 0


def test_no_fallback_when_the_library_is_missing():
    """The product path has no CPU or eager fallback: loading a library that is not there
    raises, naming the build command."""
    import subprocess
    import sys
    code = ("from hotcold_kv_cache_b200 import _lib\n"
            "try:\n"
            "    _lib.load('/nonexistent/libhotcold_b200.so')\n"
            "except RuntimeError as e:\n"
            "    print('raised:', e)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "raised:" in r.stdout and "hotcold_kv_cache_b200.build" in r.stdout


def test_drop_in_attention_refuses_cpu_tensors():
    """triton_evict_attention_forward runs on CUDA tensors only, as the reference's asserts
    require (kernels.py:87): CPU inputs are refused, never computed on the host."""
    import torch
    from hotcold_kv_cache_b200 import triton_evict_attention_forward
    q = torch.zeros(1, 8, 1, 64, dtype=torch.float16)
    k = torch.zeros(1, 2, 16, 64, dtype=torch.float16)
    m = torch.ones(1, 16, dtype=torch.bool)
    with pytest.raises(AssertionError):
        triton_evict_attention_forward(q, k, k, m, 4, 0.125)
