"""GPU parity of the QuantLinear path against the oracle: quantizeInt8/Int4
(bit-exact codes and scales), dequantize (bit-exact), the synthetic-input
generator, and QuantLinear.forward (within the north-star tolerance)."""
import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import TOL

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("shape", [(64, 2048), (3, 32), (130, 96)])
def test_quantize_bit_exact(bits, shape):
    torch = _torch()
    w = O.randn(21, bits, shape, 0.02)
    w[0, :32] = 0.0                      # all-zero group -> 1e-8 floor
    if shape[1] >= 64:
        w[0, 32:64] = 1e-9                # below the floor
    w[-1, -32:] = np.linspace(-1, 1, 32, dtype=np.float32)  # exact .5 ties
    q_ref, s_ref = O.quantize(w, bits)
    q, s32, s16 = qgmoe.quantize_device(torch.from_numpy(w).cuda(), bits)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s32.cpu().numpy(), s_ref)
    assert np.array_equal(s16.cpu().numpy().view(np.uint16), O.f16_bits(s_ref))


@pytest.mark.parametrize("bits", [8, 4, 32])
def test_dequantize_bit_exact(bits):
    torch = _torch()
    w = O.randn(22, 0, (96, 256), 0.05)
    if bits == 32:
        ql = qgmoe.QuantLinear(32, 96, 256, w)
        assert np.array_equal(ql.dequantize().cpu().numpy(), w)
        return
    q, s = O.quantize(w, bits)
    s16 = O.f16_bits(s)
    ql = qgmoe.QuantLinear(bits, 96, 256, q, s16, scale_dtype=qgmoe.SCALE_F16)
    got = ql.dequantize().cpu().numpy()
    ref = O.dequantize(bits, q, O.f16_round(s), 256)
    assert np.array_equal(got, ref)
    # f32 host scales are rounded to fp16 by the library
    ql32 = qgmoe.QuantLinear(bits, 96, 256, q, s, scale_dtype=qgmoe.SCALE_F32)
    assert np.array_equal(ql32.dequantize().cpu().numpy(), ref)
    del torch


def test_randn_matches_oracle_generator():
    torch = _torch()
    n = 1 << 20
    t = torch.empty(n, dtype=torch.float32, device="cuda")
    qgmoe.randn_device(t, 9, 4, 0.5, offset=12345)
    got = t.cpu().numpy()
    ref = O.randn(9, 4, (n,), 0.5, offset=12345)
    ulps = np.abs(got.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert ulps.max() <= 1
    assert (ulps == 0).mean() > 0.999


@pytest.mark.parametrize("bits", [32, 8, 4])
@pytest.mark.parametrize("T", [1, 5, 64])
@pytest.mark.parametrize("shape", [(300, 96), (1024, 2048)])
def test_quantlinear_forward(bits, T, shape):
    Od, Id = shape
    w = O.randn(23, 1, (Od, Id), 0.02)
    x = O.randn(23, 2, (T, Id))
    if bits == 32:
        ql = qgmoe.QuantLinear(32, Od, Id, w)
        ref = O.linear_rows(32, w, None, None, x, Od)
    else:
        q, s = O.quantize(w, bits)
        ql = qgmoe.QuantLinear(bits, Od, Id, q, O.f16_bits(s))
        ref = O.linear_rows(bits, None, q, O.f16_round(s), x, Od)
    y = ql.forward(x)
    tol = TOL[bits]
    assert np.all(np.abs(y - ref) <= tol + tol * np.abs(ref)), np.abs(y - ref).max()
    # one token through the [in] signature (quantLinear.forward)
    assert np.array_equal(ql.forward(x[0]), y[0])


def test_quantlinear_T0_is_noop():
    w = O.randn(1, 1, (32, 64))
    ql = qgmoe.QuantLinear(32, 32, 64, w)
    assert qgmoe.lib().qgql_forward(ql.h, None, 0, None) == 0
