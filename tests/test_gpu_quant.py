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


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("T", [1, 16, 100, 300])
@pytest.mark.parametrize("shape", [(256, 384), (1024, 2048)])
def test_quantlinear_tensor_path(bits, T, shape):
    """The opt-in tensor-core QuantLinear (fp16 x, fp16 dequantised weights,
    f32 accumulation and output) against the oracle, at 16-, 64- and
    128-token tiles.  Its bound is the fp16 rounding of both operands: each
    product is off by at most ~2^-10 of |w_k x_k| (the f32 accumulation adds
    far less), so |y - ref| <= 2^-10 * sum_k |w_k x_k| per output.  Also
    deterministic from call to call."""
    Od, Id = shape
    w = O.randn(31, 1, (Od, Id), 0.02)
    x = O.randn(31, 2 + T, (T, Id))
    q, s = O.quantize(w, bits)
    ql = qgmoe.QuantLinear(bits, Od, Id, q, O.f16_bits(s))
    ql.set_path(qgmoe.PATH_TENSOR)
    y = ql.forward(x)
    ref = O.linear_rows(bits, None, q, O.f16_round(s), x, Od)
    wd = np.abs(O.dequantize(bits, q, O.f16_round(s), Id)).astype(np.float64)
    bound = 1.25 * 2.0 ** -10 * (np.abs(x).astype(np.float64) @ wd.T) + 1e-6
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= bound), (err / bound).max()
    # and at the level of fp16 rounding on average, not merely inside the bound
    assert np.sqrt(np.mean(err ** 2)) <= 1e-3 * np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert np.array_equal(ql.forward(x), y)


def test_quantlinear_tensor_path_on_device_buffers():
    torch = _torch()
    Od, Id, T = 512, 1024, 200
    w = O.randn(33, 1, (Od, Id), 0.02)
    q, s = O.quantize(w, 8)
    ql = qgmoe.QuantLinear(8, Od, Id, q, O.f16_bits(s))
    x = O.randn(33, 2, (T, Id))
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((T, Od), dtype=torch.float32, device="cuda")
    ql.set_path(qgmoe.PATH_TENSOR)
    ql.forward_device(xd, yd)
    ql.sync()
    assert np.array_equal(yd.cpu().numpy(), ql.forward(x))


def test_quantlinear_tensor_path_shape_and_range_checks():
    w = O.randn(34, 1, (300, 96), 0.02)
    q, s = O.quantize(w, 8)
    ql = qgmoe.QuantLinear(8, 300, 96, q, O.f16_bits(s))
    with pytest.raises(qgmoe.QgmoeError):
        ql.set_path(qgmoe.PATH_TENSOR)  # out_features not a multiple of 128
    w = O.randn(34, 2, (128, 128), 0.02)
    q, s = O.quantize(w, 8)
    ql = qgmoe.QuantLinear(8, 128, 128, q, O.f16_bits(s))
    ql.set_path(qgmoe.PATH_TENSOR)
    x = O.randn(34, 3, (20, 128))
    x[3, 7] = 1e6  # finite, beyond fp16: flagged, not turned into infinities
    with pytest.raises(qgmoe.QgmoeError):
        ql.forward(x)
    x[3, 7] = 1.0
    ref = O.linear_rows(8, None, q, O.f16_round(s), x, 128)
    y = ql.forward(x)  # the flag was cleared
    wd = np.abs(O.dequantize(8, q, O.f16_round(s), 128)).astype(np.float64)
    assert np.all(np.abs(y - ref) <= 1.25 * 2.0 ** -10 * (np.abs(x) @ wd.T) + 1e-6)


def test_quantlinear_T0_is_noop():
    w = O.randn(1, 1, (32, 64))
    ql = qgmoe.QuantLinear(32, 32, 64, w)
    assert qgmoe.lib().qgql_forward(ql.h, None, 0, None) == 0
