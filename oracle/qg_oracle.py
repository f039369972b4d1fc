"""ctypes binding of the CPU oracle (oracle/qg_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker.  The product library
(qwen-go_b200/) never imports this module.

Parity status: unpinned at the value level -- the reference is pure Go and no
Go toolchain exists on the build or GPU machines.  The restatement is checked
against the reference's own test fixtures (TestMoERouting, TestQuantRoundTrip
in model/model_test.go) and hand-derived known answers (tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libqg_oracle.so")

ROUTER_TOPK = 0
ROUTER_PREFIX = 1

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i32p = C.POINTER(C.c_int32)
_u16p = C.POINTER(C.c_uint16)


class _Lin(C.Structure):
    _fields_ = [("w", _f32p), ("q", _u8p), ("scale", _f32p)]


class _Moe(C.Structure):
    _fields_ = [
        ("n_embed", C.c_int), ("n_experts", C.c_int), ("top_k", C.c_int),
        ("n_moe_mlp", C.c_int), ("n_shared_mlp", C.c_int), ("bits", C.c_int),
        ("router_mode", C.c_int),
        ("router", _f32p), ("shared_gate", _f32p),
        ("gate_up", _Lin), ("down", _Lin), ("sh_gate", _Lin), ("sh_up", _Lin), ("sh_down", _Lin),
        ("shared_bits", C.c_int), ("router_bits", C.c_int), ("router_q", _Lin),
    ]


def build() -> str:
    """Compiles the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "qg_oracle.c")):
            build()
        L = C.CDLL(LIB_PATH)
        L.qgo_randn.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_int64, C.c_float, _f32p]
        L.qgo_quantize_int8.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _f32p]
        L.qgo_quantize_int4.argtypes = [_f32p, C.c_int, C.c_int, _u8p, _f32p]
        L.qgo_dequantize.argtypes = [C.c_int, C.c_int, C.c_int, _u8p, _f32p, _f32p]
        L.qgo_matmul_vec.argtypes = [_f32p, _f32p, C.c_int, C.c_int, _f32p]
        L.qgo_softmax.argtypes = [_f32p, C.c_int]
        L.qgo_route_token.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _i32p, _f32p]
        L.qgo_moe_forward.argtypes = [C.POINTER(_Moe), _f32p, C.c_int, _f32p, _i32p, _f32p,
                                      _f32p, _f32p]
        L.qgo_moe_forward_mt.argtypes = [C.POINTER(_Moe), _f32p, C.c_int, _f32p, _i32p, _f32p,
                                         _f32p, _f32p, C.c_int]
        L.qgo_moe_forward_mt.restype = C.c_int
        L.qgo_f16_encode.argtypes = [_f32p, C.c_int64, _u16p]
        L.qgo_f16_decode.argtypes = [_u16p, C.c_int64, _f32p]
        L.qgo_linear_forward_rows.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _u8p, _f32p,
                                              _f32p, C.c_int, _f32p]
        _lib = L
    return _lib


def _p(a: np.ndarray | None, ty):
    if a is None:
        return C.cast(None, ty)
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ty)


def randn(seed: int, stream: int, shape, std: float = 1.0, offset: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    lib().qgo_randn(seed, stream, offset, n, std, _p(out, _f32p))
    return out.reshape(shape)


def quantize(w: np.ndarray, bits: int):
    """quantizeInt8 / quantizeInt4 (model/moe.go:165-217): codes, f32 scales."""
    w = np.ascontiguousarray(w, np.float32)
    O, I = w.shape
    q = np.zeros((O, I if bits == 8 else I // 2), np.uint8)
    s = np.zeros((O, I // 32), np.float32)
    fn = lib().qgo_quantize_int8 if bits == 8 else lib().qgo_quantize_int4
    fn(_p(w, _f32p), O, I, _p(q, _u8p), _p(s, _f32p))
    return q, s


def dequantize(bits: int, q: np.ndarray, s: np.ndarray, in_dim: int) -> np.ndarray:
    O = q.shape[0]
    w = np.empty((O, in_dim), np.float32)
    lib().qgo_dequantize(bits, O, in_dim, _p(np.ascontiguousarray(q), _u8p),
                         _p(np.ascontiguousarray(s, np.float32), _f32p), _p(w, _f32p))
    return w


def f16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest fp16 (RNE) and back."""
    a = np.ascontiguousarray(a, np.float32)
    h = np.empty(a.shape, np.uint16)
    lib().qgo_f16_encode(_p(a, _f32p), a.size, _p(h, _u16p))
    out = np.empty(a.shape, np.float32)
    lib().qgo_f16_decode(_p(h, _u16p), a.size, _p(out, _f32p))
    return out


def f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    h = np.empty(a.shape, np.uint16)
    lib().qgo_f16_encode(_p(a, _f32p), a.size, _p(h, _u16p))
    return h


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN stays a
    quiet NaN).  The reference reads bf16 weights as the high half of a
    float32 (bf16f32, model/model.go:113-115); HF checkpoints store them so."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(a, np.float32))
    out = (r & 0xFFFF).astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_widen(h: np.ndarray) -> np.ndarray:
    """bf16f32 (model/model.go:113-115): the bits as the high half of a float32."""
    return (np.ascontiguousarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def softmax(v: np.ndarray) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    lib().qgo_softmax(_p(v, _f32p), v.size)
    return v


def route_token(logits: np.ndarray, k: int, mode: int):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.zeros(k, np.int32)
    w = np.zeros(k, np.float32)
    lib().qgo_route_token(_p(logits, _f32p), logits.size, k, mode, _p(idx, _i32p), _p(w, _f32p))
    return idx, w


def linear_rows(bits, w32, q, s, x, out_dim):
    x = np.ascontiguousarray(x, np.float32)
    T, in_dim = x.shape
    y = np.zeros((T, out_dim), np.float32)
    lib().qgo_linear_forward_rows(bits, out_dim, in_dim, _p(w32, _f32p), _p(q, _u8p),
                                  _p(s, _f32p), _p(x, _f32p), T, _p(y, _f32p))
    return y


@dataclass
class MoeWeights:
    """Weights of one moeMLP in the reference layout (model/moe.go:10-25).

    bits 32: gate_up [E,2I,H], down [E,H,I], sh_gate/sh_up [Is,H], sh_down [H,Is].
    bits 16: raw bf16 experts (gateUpRaw / downRaw, model/moe.go:14-15, 64-81):
             q holds the bf16 bit patterns and the float32 fields their exact
             widening; bf16matvec (model/moe.go:102-113) and the raw linear
             (matvecRange, model/model.go:167-176) are the serial float32 dot of
             matmulVec (model/tensors.go:77-89) over those widened values, so
             the oracle runs the bits-32 arithmetic on them.
    bits 8/4: the same tensors as quantLinear codes + f32 scale arrays; the
    scale arrays here are what the dequantiser multiplies by (rounded to
    fp16: the library stores expert and shared-expert scales as fp16).
    shared_bits (0 = bits): the shared expert's own format.  router_bits:
    32 = float32 rows in `router`; 16 = bf16 bits in q["router"] (router
    holds their widening); 8 / 4 = routerQuant (model/moe.go:16) codes in
    q["router"] with scales s["router"] as dequantised (router holds the
    dequantised rows), s16 / s32 the fp16 bits / raw f32 scales handed to
    the library.
    """
    H: int
    E: int
    k: int
    I: int
    Is: int
    bits: int
    router: np.ndarray
    shared_gate: np.ndarray | None = None
    gate_up: np.ndarray | None = None
    down: np.ndarray | None = None
    sh_gate: np.ndarray | None = None
    sh_up: np.ndarray | None = None
    sh_down: np.ndarray | None = None
    q: dict = field(default_factory=dict)   # name -> codes
    s: dict = field(default_factory=dict)   # name -> f32 scales (as dequantised)
    s16: dict = field(default_factory=dict)  # name -> fp16 bits of the scales
    s32: dict = field(default_factory=dict)  # name -> raw f32 scales (router, f32 format)
    shared_bits: int = 0
    router_bits: int = 32


def make_moe(H, E, k, I, Is, bits, seed, std=0.02, shared_bits=0, router_bits=32,
             router_scale_f32=False) -> MoeWeights:
    """Synthetic layer: draws router, gate_up, down, shared_gate, shared
    gate/up/down from streams 0..6 of `seed` (N(0, std)), then puts each
    group in its format: the routed experts in `bits`, the shared expert in
    `shared_bits` (0 = bits), the router in `router_bits` (32 = f32 rows;
    with router_scale_f32 a quantised router keeps its f32 scales, as
    cmd/qwen-quant writes them)."""
    m = MoeWeights(H=H, E=E, k=k, I=I, Is=Is, bits=bits,
                   router=randn(seed, 0, (E, H), std), shared_bits=shared_bits,
                   router_bits=router_bits)
    gate_up = randn(seed, 1, (E, 2 * I, H), std)
    down = randn(seed, 2, (E, H, I), std)
    mats = {"gate_up": (gate_up, bits), "down": (down, bits)}
    if Is > 0:
        m.shared_gate = randn(seed, 3, (H,), std)
        sb = shared_bits or bits
        mats.update(sh_gate=(randn(seed, 4, (Is, H), std), sb),
                    sh_up=(randn(seed, 5, (Is, H), std), sb),
                    sh_down=(randn(seed, 6, (H, Is), std), sb))
    for name, (w, b) in mats.items():
        if b == 32:
            setattr(m, name, w)
        elif b == 16:
            m.q[name] = bf16_bits(w)
            setattr(m, name, bf16_widen(m.q[name]))
        else:
            q, s = quantize(w.reshape(-1, w.shape[-1]), b)
            m.q[name] = q
            m.s16[name] = f16_bits(s)
            m.s[name] = f16_round(s)
    if router_bits == 16:
        m.q["router"] = bf16_bits(m.router)
        m.router = bf16_widen(m.q["router"])
    elif router_bits in (8, 4):
        q, s = quantize(m.router, router_bits)
        m.q["router"] = q
        m.s16["router"] = f16_bits(s)
        m.s32["router"] = s
        m.s["router"] = s if router_scale_f32 else f16_round(s)
        m.router = dequantize(router_bits, q, m.s["router"], H)
    return m


def _none_lin() -> _Lin:
    return _Lin(C.cast(None, _f32p), C.cast(None, _u8p), C.cast(None, _f32p))


def _lin(m: MoeWeights, name: str, bits: int) -> _Lin:
    if bits in (32, 16):
        w = getattr(m, name)
        return _none_lin() if w is None else _Lin(_p(w, _f32p), C.cast(None, _u8p),
                                                  C.cast(None, _f32p))
    if name not in m.q:
        return _none_lin()
    return _Lin(C.cast(None, _f32p), _p(m.q[name], _u8p), _p(m.s[name], _f32p))


def _struct(m: MoeWeights, mode: int) -> _Moe:
    """bf16 groups run as float32 on their exact widening (bf16matvec and the
    raw linear are matmulVec over bf16f32 values)."""
    st = _Moe()
    sb = m.shared_bits or m.bits
    st.n_embed, st.n_experts, st.top_k, st.n_moe_mlp = m.H, m.E, m.k, m.I
    st.n_shared_mlp, st.router_mode = m.Is, mode
    st.bits = 32 if m.bits == 16 else m.bits
    st.shared_bits = 32 if sb == 16 else sb
    st.router = _p(m.router, _f32p)
    st.shared_gate = _p(m.shared_gate, _f32p)
    for name in ("gate_up", "down"):
        setattr(st, name, _lin(m, name, m.bits))
    for name in ("sh_gate", "sh_up", "sh_down"):
        setattr(st, name, _lin(m, name, sb))
    if m.router_bits in (8, 4):
        st.router_bits = m.router_bits
        st.router_q = _lin(m, "router", m.router_bits)
    else:
        st.router_bits = 32
        st.router_q = _none_lin()
    return st


def moe_forward(m: MoeWeights, x: np.ndarray, mode: int = ROUTER_TOPK, want_probs=False):
    """moeMLP.forward token by token.  Returns out [T,H], idx [T,k], w [T,k],
    shared gate [T] and (optionally) softmax probabilities [T,E]."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.zeros((T, m.H), np.float32)
    idx = np.zeros((T, m.k), np.int32)
    w = np.zeros((T, m.k), np.float32)
    sg = np.zeros(T, np.float32)
    probs = np.zeros((T, m.E), np.float32) if want_probs else None
    st = _struct(m, mode)
    lib().qgo_moe_forward(C.byref(st), _p(x, _f32p), T, _p(out, _f32p), _p(idx, _i32p),
                          _p(w, _f32p), _p(sg, _f32p), _p(probs, _f32p))
    return out, idx, w, sg, probs


def moe_forward_mt(m: MoeWeights, x: np.ndarray, threads: int, mode: int = ROUTER_TOPK,
                   want_routing: bool = False):
    """moe_forward over tokens split across `threads` host threads (the same
    per-token arithmetic, bit-identical results).  Returns out, or (out, idx,
    w, shared gate, probs) with want_routing."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.zeros((T, m.H), np.float32)
    idx = w = sg = probs = None
    if want_routing:
        idx = np.zeros((T, m.k), np.int32)
        w = np.zeros((T, m.k), np.float32)
        sg = np.zeros(T, np.float32)
        probs = np.zeros((T, m.E), np.float32)
    st = _struct(m, mode)
    lib().qgo_moe_forward_mt(C.byref(st), _p(x, _f32p), T, _p(out, _f32p), _p(idx, _i32p),
                             _p(w, _f32p), _p(sg, _f32p), _p(probs, _f32p), threads)
    return (out, idx, w, sg, probs) if want_routing else out
