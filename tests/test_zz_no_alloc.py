"""The allocation-free attention entry point, for callers that cannot allocate
device memory (a host that binds the library over FFI with only its own input
and output buffers, or a process whose device memory belongs to its own pool).

It is called through the C ABI and must give the same output as
hc_attention_dense with a caller-provided workspace, on two calls in a row
(the static scratch keeps the first call's contents; the second call must not
depend on them). This file is collected last, so a failure here comes after
every other test has run; it also passes alone in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL = {torch.float32: 1e-5, torch.float16: 2e-3}


def _close(a, b, dt):
    a, b = a.double().cpu().numpy(), b.double().cpu().numpy()
    rel = REL[dt]
    err = (np.abs(a - b) - rel * np.abs(b)).max() / max(np.abs(b).max(), 1e-30)
    assert err <= rel, err


def _reference_call(lib, q, k, v, m, out, idx, B, Hq, Hk, S, D, dt_code, stream):
    """The existing entry point with its own workspace."""
    n = lib.hc_attention_dense_scratch_bytes(B, Hq, Hk, S, D)
    scratch = torch.empty(n, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(B * Hk, dtype=torch.int32, device="cuda")
    rc = lib.hc_attention_dense(q.data_ptr(), k.data_ptr(), v.data_ptr(), m.data_ptr(), out.data_ptr(),
                                idx.data_ptr(), B, Hq, Hk, S, D, dt_code, 1.0 / math.sqrt(D), 1,
                                counters.data_ptr(), scratch.data_ptr(), n, stream)
    assert rc == 0, lib.hc_last_error()


@pytest.mark.parametrize("dtype,code", [(torch.float32, 0), (torch.float16, 1)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, code):
    from hotcold_kv_cache_b200 import _lib
    lib = _lib.load()
    torch.cuda.init()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (B, Hq, Hk, S) in enumerate([(2, 32, 8, 577), (1, 8, 2, 1100)]):
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        D = 128
        q = torch.randn((B, Hq, 1, D), generator=g, device="cuda").to(dtype)
        k = torch.randn((B, Hk, S, D), generator=g, device="cuda").to(dtype)
        v = torch.randn((B, Hk, S, D), generator=g, device="cuda").to(dtype)
        m = (torch.rand((B, S), generator=g, device="cuda") < 0.9).to(torch.uint8)
        m[:, 0] = 1
        want = torch.empty((B, Hq, D), dtype=dtype, device="cuda")
        want_idx = torch.empty(B, dtype=torch.int64, device="cuda")
        _reference_call(lib, q, k, v, m, want, want_idx, B, Hq, Hk, S, D, code, stream)
        got = torch.full((B, Hq, D), float("nan"), dtype=dtype, device="cuda")
        got_idx = torch.full((B,), -1, dtype=torch.int64, device="cuda")
        rc = lib.hc_attention_dense_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), m.data_ptr(), got.data_ptr(),
                                            got_idx.data_ptr(), B, Hq, Hk, S, D, code, 1.0 / math.sqrt(D), 1,
                                            stream)
        assert rc == 0, lib.hc_last_error()
        torch.cuda.synchronize()
        _close(got, want, dtype)
        assert torch.equal(got_idx, want_idx)


def test_noalloc_rejects_shapes_beyond_its_static_area():
    from hotcold_kv_cache_b200 import _lib
    lib = _lib.load()
    # 64 sequences x 8 KV heads x 130 chunks of 32 rows of partials needs more than the 8 MiB area
    rc = lib.hc_attention_dense_noalloc(1, 1, 1, 1, 1, None, 64, 32, 8, 4100, 128, 1, 0.1, 1, None)
    assert rc == 3 and b"scratch" in lib.hc_last_error()
    # one row past the largest 16-sequence shape that fits
    assert lib.hc_attention_dense_scratch_bytes(16, 32, 8, 961, 128) > 8 << 20
    rc = lib.hc_attention_dense_noalloc(1, 1, 1, 1, 1, None, 16, 32, 8, 961, 128, 1, 0.1, 1, None)
    assert rc == 3 and b"scratch" in lib.hc_last_error()


def test_noalloc_accepts_the_largest_shape_that_fits():
    """16 sequences x 960 rows: the split-K partials fill the static area to within 1 %."""
    from hotcold_kv_cache_b200 import _lib
    lib = _lib.load()
    B, Hq, Hk, S, D = 16, 32, 8, 960, 128
    need = lib.hc_attention_dense_scratch_bytes(B, Hq, Hk, S, D)
    assert 0.99 * (8 << 20) <= need <= 8 << 20
    torch.cuda.init()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn((B, Hq, 1, D), generator=g, device="cuda").half()
    k = torch.randn((B, Hk, S, D), generator=g, device="cuda").half()
    v = torch.randn((B, Hk, S, D), generator=g, device="cuda").half()
    m = torch.ones((B, S), dtype=torch.uint8, device="cuda")
    want = torch.empty((B, Hq, D), dtype=torch.float16, device="cuda")
    want_idx = torch.empty(B, dtype=torch.int64, device="cuda")
    _reference_call(lib, q, k, v, m, want, want_idx, B, Hq, Hk, S, D, 1, stream)
    got = torch.empty_like(want)
    got_idx = torch.empty_like(want_idx)
    rc = lib.hc_attention_dense_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), m.data_ptr(), got.data_ptr(),
                                        got_idx.data_ptr(), B, Hq, Hk, S, D, 1, 1.0 / math.sqrt(D), 1, stream)
    assert rc == 0, lib.hc_last_error()
    torch.cuda.synchronize()
    _close(got, want, torch.float16)
    assert torch.equal(got_idx, want_idx)
