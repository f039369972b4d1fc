"""CPU tests of the oracle (oracle/qg_oracle.c).

The reference is pure Go and cannot run here, so the oracle is pinned by
(1) the reference's own MoE/quant test fixtures, (2) known answers derived by
hand from the Go source, and (3) an independent numpy restatement written
directly from model/moe.go and model/tensors.go.
"""
import numpy as np
import pytest

import qg_oracle as O

# --------------------------------------------------------------------------
# Independent numpy restatement (pure float32 element ops, serial order)
# --------------------------------------------------------------------------


def np_matvec(x, W):
    """matmulVec (model/tensors.go:77-89): s += x[k]*w[o,k], k ascending."""
    x = x.astype(np.float32)
    W = W.astype(np.float32)
    s = np.zeros(W.shape[0], np.float32)
    for k in range(W.shape[1]):
        s = (s + (x[k] * W[:, k]).astype(np.float32)).astype(np.float32)
    return s


def np_softmax(v):
    v = v.astype(np.float32).copy()
    mx = np.float32(v.max())
    e = np.exp((v - mx).astype(np.float64)).astype(np.float32)
    s = np.float32(0)
    for val in e:
        s = np.float32(s + val)
    return (e / s).astype(np.float32)


def np_silu(g):
    return (g / (np.float32(1) + np.exp(-g.astype(np.float64)).astype(np.float32))).astype(np.float32)


def np_route(logits, k, mode):
    p = np_softmax(logits)
    idx = list(range(len(p)))
    lim = k if mode == O.ROUTER_PREFIX else len(p)
    for i in range(1, min(lim, len(p))):
        j = i
        while j > 0 and p[idx[j]] > p[idx[j - 1]]:
            idx[j], idx[j - 1] = idx[j - 1], idx[j]
            j -= 1
    wsum = np.float32(0)
    for i in range(k):
        wsum = np.float32(wsum + p[idx[i]])
    den = np.float32(wsum + np.float32(1e-9))
    return np.array(idx[:k], np.int32), np.array([p[i] / den for i in idx[:k]], np.float32)


def np_dequant(bits, q, s, in_dim):
    O_ = q.shape[0]
    w = np.zeros((O_, in_dim), np.float32)
    if bits == 8:
        codes = q.view(np.int8).astype(np.float32)
    else:
        hi = ((q >> 4) & 0xF).astype(np.float32) - 8
        lo = (q & 0xF).astype(np.float32) - 8
        codes = np.stack([hi, lo], axis=-1).reshape(O_, in_dim)
    for c in range(in_dim):
        w[:, c] = (codes[:, c] * s[:, c // 32]).astype(np.float32)
    return w


def np_moe_token(m, x, mode):
    logits = np_matvec(x, m.router)
    idx, w = np_route(logits, m.k, mode)
    H, I = m.H, m.I
    out = np.zeros(H, np.float32)

    def lin(name, row0, rows, in_dim, v):
        if m.bits == 16:  # bf16matvec: the bf16 bits widened (<< 16), then the f32 dot
            h = m.q[name].reshape(-1, in_dim)[row0:row0 + rows]
            W = (h.astype(np.uint32) << 16).view(np.float32)
        elif m.bits == 32:
            W = getattr(m, name).reshape(-1, in_dim)[row0:row0 + rows]
        else:
            q = m.q[name][row0:row0 + rows]
            W = np_dequant(m.bits, q, m.s[name][row0:row0 + rows], in_dim)
        return np_matvec(v, W)

    for r in range(m.k):
        e = int(idx[r])
        gu = lin("gate_up", e * 2 * I, 2 * I, H, x)
        g = np_silu(gu[:I])
        g = (g * gu[I:]).astype(np.float32)
        d = lin("down", e * H, H, I, g)
        out = (out + (w[r] * d).astype(np.float32)).astype(np.float32)
    if m.Is > 0:
        g = lin("sh_gate", 0, m.Is, H, x)
        u = lin("sh_up", 0, m.Is, H, x)
        g = (np_silu(g) * u).astype(np.float32)
        s = lin("sh_down", 0, H, m.Is, g)
        gd = np.float32(0)
        for i in range(H):
            gd = np.float32(gd + np.float32(x[i] * m.shared_gate[i]))
        sg = np.float32(1) / (np.float32(1) + np.float32(np.exp(-np.float64(gd))))
        out = (out + (sg * s).astype(np.float32)).astype(np.float32)
    return out, idx, w


# --------------------------------------------------------------------------
# Reference fixtures
# --------------------------------------------------------------------------


def test_reference_TestMoERouting_fixture():
    """model/model_test.go:182-201: E=4, k=2, H=8, I=16, router row 0 =
    [1,2,3,4,0,0,0,0] (the test's gate.w sliced to len 4 but read through its
    capacity), every other weight zero, x = 0.1..0.8.  The reference asserts
    len(out) == 8 and finite; with all expert/shared weights zero the output
    is exactly zero, and routing picks expert 0 then expert 1."""
    H, E, k, I, Is = 8, 4, 2, 16, 4
    m = O.MoeWeights(H=H, E=E, k=k, I=I, Is=Is, bits=32,
                     router=np.zeros((E, H), np.float32))
    m.router[0, :4] = [1, 2, 3, 4]
    m.shared_gate = np.zeros(H, np.float32)
    m.gate_up = np.zeros((E, 2 * I, H), np.float32)
    m.down = np.zeros((E, H, I), np.float32)
    m.sh_gate = np.zeros((Is, H), np.float32)
    m.sh_up = np.zeros((Is, H), np.float32)
    m.sh_down = np.zeros((H, Is), np.float32)
    x = np.array([0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8], np.float32)[None]
    for mode in (O.ROUTER_PREFIX, O.ROUTER_TOPK):
        out, idx, w, sg, _ = O.moe_forward(m, x, mode)
        assert out.shape == (1, 8)
        assert np.all(np.isfinite(out)) and np.all(out == 0)
        assert idx.tolist() == [[0, 1]]
        assert sg[0] == np.float32(0.5)
        # logit0 = .1+.4+.9+1.6 = 3 (f32 serial), others 0
        p0 = np.float32(np.exp(np.float64(0)))
        e3 = np.float32(np.exp(np.float64(np.float32(0) - np.float32(3.0000002))))
        assert w[0, 0] > 0.9 and w[0, 1] < 0.1
        assert abs(float(w[0].sum()) - 1.0) < 1e-6
        del p0, e3


def test_reference_TestQuantRoundTrip_property():
    """model/model_test.go:130-147: int8 quantize->dequant of a 16x64 N(0, 0.1)
    matrix stays within 0.02 of the input (the Go test's math/rand stream is
    not reproducible without Go; the property is checked on our generator)
    and, per its comment, int4 within ~2 scale steps."""
    w = O.randn(7, 0, (16, 64), 0.1)
    q, s = O.quantize(w, 8)
    dq = O.dequantize(8, q, s, 64)
    assert np.max(np.abs(w - dq)) <= 0.02
    q4, s4 = O.quantize(w, 4)
    dq4 = O.dequantize(4, q4, s4, 64)
    steps = np.abs(w - dq4) / np.repeat(s4, 32, axis=1)
    assert steps.max() <= 2.0


# --------------------------------------------------------------------------
# Hand-derived known answers from model/moe.go
# --------------------------------------------------------------------------


def test_quantize_int8_known_answer():
    # group amax = 1.27 -> s = 1.27/127 = 0.01 (f32); w/s rounds half away.
    row = np.zeros(32, np.float32)
    row[:6] = [1.27, -1.27, 0.005, -0.005, 0.015, 0.63]
    q, s = O.quantize(row[None], 8)
    s_exp = np.float32(np.float32(1.27) / np.float32(127))
    assert s[0, 0] == s_exp
    codes = q.view(np.int8)[0]
    expect = [int(np.round(np.float64(np.float32(v) / s_exp))) for v in row[:6]]
    # math.Round: half away from zero
    expect = [int(np.sign(np.float32(v) / s_exp) * np.floor(abs(np.float32(v) / s_exp) + 0.5))
              for v in row[:6]]
    assert codes[:6].tolist() == expect
    assert codes[0] == 127 and codes[1] == -127
    assert np.all(codes[6:] == 0)


def test_quantize_int4_nibble_order_known_answer():
    # amax 0.7 -> s = 0.1; values -> clamp(round(w/s), -7, 7) + 8;
    # element 0 goes to the HIGH nibble of byte 0 (moe.go:208-212).
    row = np.zeros(32, np.float32)
    row[0], row[1], row[2], row[3] = 0.7, -0.7, 0.3, 0.0
    q, s = O.quantize(row[None], 4)
    assert s[0, 0] == np.float32(np.float32(0.7) / np.float32(7))
    assert q[0, 0] == (15 << 4) | 1   # +7+8=15 high, -7+8=1 low
    assert q[0, 1] == (11 << 4) | 8   # round(3)+8=11 high, 0+8 low
    assert np.all(q[0, 2:] == 0x88)


def test_quantize_all_zero_group_floor():
    q, s = O.quantize(np.zeros((2, 32), np.float32), 8)
    assert np.all(s == np.float32(1e-8)) and np.all(q == 0)
    q4, s4 = O.quantize(np.zeros((2, 32), np.float32), 4)
    assert np.all(s4 == np.float32(1e-8)) and np.all(q4 == 0x88)


def test_prefix_router_is_degenerate():
    """moe.go:49 bounds the insertion sort by topK, so PREFIX always picks
    experts {0..k-1} ordered by probability."""
    rng = np.random.default_rng(0)
    for _ in range(50):
        logits = rng.normal(size=16).astype(np.float32)
        idx, _ = O.route_token(logits, 4, O.ROUTER_PREFIX)
        assert sorted(idx.tolist()) == [0, 1, 2, 3]
        p = np_softmax(logits)
        assert all(p[idx[i]] >= p[idx[i + 1]] for i in range(3))
        idx2, _ = O.route_token(logits, 4, O.ROUTER_TOPK)
        assert idx2.tolist() == np.argsort(-p, kind="stable")[:4].tolist()


def test_route_ties_keep_lower_index():
    logits = np.zeros(8, np.float32)
    idx, w = O.route_token(logits, 3, O.ROUTER_TOPK)
    assert idx.tolist() == [0, 1, 2]
    assert np.allclose(w, 1 / 3, atol=1e-6)


def test_f16_encode_matches_numpy():
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.normal(0, 1e-3, 20000), rng.normal(0, 1, 20000), rng.uniform(-7e4, 7e4, 2000),
        np.array([0.0, -0.0, 1e-8, 6e-8, 2.98e-8, 3e-8, 65504, 65519, 65520, 1e-5, 6.1e-5,
                  np.inf, -np.inf])]).astype(np.float32)
    got = O.f16_bits(vals)
    want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_f16_decode_restates_safetensors():
    h = np.arange(0, 65536, dtype=np.uint16)
    h = h[(h & 0x7C00) != 0x7C00]  # finite values
    out = np.empty(h.shape, np.float32)
    O.lib().qgo_f16_decode(h.ctypes.data_as(O._u16p), h.size, out.ctypes.data_as(O._f32p))
    assert np.array_equal(out, h.view(np.float16).astype(np.float32))


def test_randn_counter_based_and_moments():
    a = O.randn(3, 5, (1000,))
    b = O.randn(3, 5, (600,), offset=400)
    assert np.array_equal(a[400:], b)
    assert not np.array_equal(a, O.randn(3, 6, (1000,)))
    z = O.randn(0, 0, (200000,))
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01


# --------------------------------------------------------------------------
# Oracle == independent numpy restatement (bit-exact)
# --------------------------------------------------------------------------


@pytest.mark.parametrize("bits", [32, 16, 8, 4])
@pytest.mark.parametrize("mode", [O.ROUTER_TOPK, O.ROUTER_PREFIX])
@pytest.mark.parametrize("Is", [0, 64])
def test_oracle_matches_numpy_restatement(bits, mode, Is):
    H, E, k, I = 64, 8, 3, 32
    m = O.make_moe(H, E, k, I, Is, bits, seed=11)
    x = O.randn(11, 100, (3, H))
    out, idx, w, _, _ = O.moe_forward(m, x, mode)
    for t in range(3):
        o2, i2, w2 = np_moe_token(m, x[t], mode)
        assert idx[t].tolist() == i2.tolist()
        assert np.array_equal(w[t], w2)
        assert np.array_equal(out[t], o2), np.max(np.abs(out[t] - o2))


@pytest.mark.parametrize("bits", [8, 4])
def test_dequantize_matches_numpy(bits):
    w = O.randn(5, 1, (24, 96), 0.05)
    q, s = O.quantize(w, bits)
    assert np.array_equal(O.dequantize(bits, q, s, 96), np_dequant(bits, q, s, 96))


def test_token_parallel_equals_serial():
    m = O.make_moe(64, 8, 2, 32, 32, 8, seed=2)
    x = O.randn(2, 100, (13, 64))
    out, *_ = O.moe_forward(m, x)
    assert np.array_equal(O.moe_forward_mt(m, x, 4), out)


def test_bf16_rounding_known_answers():
    """float32 -> bf16 (round to nearest even on the dropped 16 bits) and the
    reference's widening bf16f32 (model/model.go:113-115)."""
    vals = np.array([1.0, 1.00390625, 1.01171875, 1.0078125, -2.5, 3.0e38, 1e-40, 0.0, -0.0,
                     np.inf, -np.inf], np.float32)
    bits = O.bf16_bits(vals)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 ties up to 1 + 2^-6; 1 + 2^-7 exact
    assert bits.tolist()[:5] == [0x3F80, 0x3F80, 0x3F82, 0x3F81, 0xC020]
    assert bits[5] == 0x7F62  # 3e38 rounds to 0x7F62 (3.0e38 ~ 0x7F61B1E6)
    assert bits[7] == 0x0000 and bits[8] == 0x8000 and bits[9] == 0x7F80 and bits[10] == 0xFF80
    w = O.bf16_widen(bits)
    assert w[0] == 1.0 and w[2] == np.float32(1.015625) and w[4] == -2.5
    nan = O.bf16_bits(np.array([np.nan], np.float32))
    assert np.isnan(O.bf16_widen(nan)[0])
    # widening is exact: every bf16 value survives a round trip
    h = np.arange(0, 1 << 16, 97, dtype=np.uint32).astype(np.uint16)
    finite = np.isfinite(O.bf16_widen(h))
    assert np.array_equal(O.bf16_bits(O.bf16_widen(h))[finite], h[finite])


def test_oracle_reproduces_committed_golden_vectors():
    """tests/golden/moe_small.npz (written by tests/golden/make_golden.py):
    16 small layers (bits 32/16/8/4, both router modes, with and without the
    shared expert) must come out bit for bit as committed."""
    import importlib.util
    import os
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    g = np.load(os.path.join(here, "moe_small.npz"))
    assert [tuple(c) for c in g["cases"]] == [tuple(c) for c in mg.CASES]
    for i, (bits, mode, Is) in enumerate(mg.CASES):
        m, x = mg.case_arrays(i, bits, mode, Is)
        y, idx, w, _, _ = O.moe_forward(m, x, mode)
        assert np.array_equal(y, g[f"c{i}_out"]), i
        assert np.array_equal(idx, g[f"c{i}_idx"]) and np.array_equal(w, g[f"c{i}_w"]), i
