"""The stand-alone decode attention (drop-in for triton_evict_attention_forward)
against the reference kernel's golden output and the oracle, plus edge cases."""

import math

import numpy as np
import pytest
import torch

from golden_cases import assert_close, load

pytestmark = pytest.mark.gpu

from oracle import hotcold_oracle as O  # noqa: E402

DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _fwd(q, k, v, m, **kw):
    from hotcold_kv_cache_b200 import triton_evict_attention_forward
    dev = torch.device("cuda:0")
    return triton_evict_attention_forward(q.to(dev), k.to(dev), v.to(dev), m.to(dev),
                                          q.shape[1] // k.shape[1], 1.0 / math.sqrt(q.shape[-1]), **kw)


def test_reference_kernel_golden():
    from hotcold_kv_cache_b200 import synth
    g = load("triton_kernel")
    q, k, v, m = (torch.from_numpy(x) for x in synth.attention_case_inputs(7))
    out, idx = _fwd(q, k, v, m)
    assert out.shape == (2, 1, 8, 128) and out.is_contiguous()
    assert_close(out.cpu().numpy(), g["out"], "float32", "attention vs reference kernel")
    assert np.array_equal(idx.cpu().numpy(), g["evict_idx"])


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("B,Hq,Hk,S,D", [(1, 32, 8, 577, 128), (3, 8, 2, 1, 128), (2, 4, 4, 65, 64),
                                         (2, 16, 2, 200, 128), (1, 32, 8, 4100, 128), (4, 8, 1, 33, 64)])
def test_vs_oracle(dtype, B, Hq, Hk, S, D):
    rng = np.random.default_rng(S * 7 + B)
    from hotcold_kv_cache_b200 import synth
    q = synth.to_model_dtype(rng.standard_normal((B, Hq, 1, D), dtype=np.float32), dtype)
    k = synth.to_model_dtype(rng.standard_normal((B, Hk, S, D), dtype=np.float32), dtype)
    v = synth.to_model_dtype(rng.standard_normal((B, Hk, S, D), dtype=np.float32), dtype)
    m = rng.random((B, S)) < 0.85
    m[:, 0] = True
    ref = O.decode_attention(q[:, :, 0].astype(np.float64), k, v, m, 1.0 / math.sqrt(D), dtype)
    tq, tk, tv = (torch.from_numpy(np.asarray(x, np.float32)).to(DT[dtype]) for x in (q, k, v))
    out, idx = _fwd(tq, tk, tv, torch.from_numpy(m))
    assert_close(out[:, 0].float().cpu().numpy(), ref, dtype, "attention")
    if dtype == "float32":
        ri = O.evict_loss_argmin(q[:, :, 0], k, v, m, 1.0 / math.sqrt(D), dtype)
        assert np.array_equal(idx.cpu().numpy(), ri)


def test_all_masked_and_overflow_give_nan():
    rng = np.random.default_rng(1)
    q = torch.from_numpy(rng.standard_normal((2, 4, 1, 128), dtype=np.float32))
    k = torch.from_numpy(rng.standard_normal((2, 1, 100, 128), dtype=np.float32))
    v = torch.from_numpy(rng.standard_normal((2, 1, 100, 128), dtype=np.float32))
    m = torch.ones(2, 100, dtype=torch.bool)
    m[1] = False                      # sequence 1 attends to nothing: 0/0
    k[0, 0, 37] = q[0, 0, 0] * 50.0   # head 0 of sequence 0: logit far above ln(FLT_MAX)
    out, _ = _fwd(q, k, v, m)
    o = out[:, 0].cpu()
    assert torch.isnan(o[1]).all()
    assert torch.isnan(o[0, 0]).all()
    assert torch.isfinite(o[0, 1:]).all()
    out2, _ = _fwd(q, k, v, m, overflow_nan=False)
    assert torch.isfinite(out2[0, 0, 0]).all()


def test_errors_match_reference():
    from hotcold_kv_cache_b200 import triton_evict_attention_forward as f
    q = torch.zeros(1, 8, 1, 128, device="cuda")
    k = torch.zeros(1, 2, 10, 128, device="cuda")
    m = torch.ones(1, 10, dtype=torch.bool, device="cuda")
    with pytest.raises(ValueError):
        f(q, k, k, m, 4, 0.1, dropout=0.1)
    with pytest.raises(ValueError):
        f(q, k, k, m, 2, 0.1)
    with pytest.raises(AssertionError):
        f(q.cpu(), k, k, m, 4, 0.1)
