"""Host-side mirror of qwen-go's MoE / QuantLinear API over libqgmoe.so.

The reference's seam is the Go `mixer` interface (`forward(x []float32)
[]float32`, model/model.go:373-375) implemented by `moeMLP`
(model/moe.go:10-99), and `quantLinear` (model/moe.go:126-162) with the
quantisers `QuantizeInt8` / `QuantizeInt4` (model/moe.go:233-239).  This
module exposes the same objects over the C ABI in include/qgmoe.h:

    MoeMLP(desc...).forward(x)          x [H]      -> out [H]      (T = 1)
    MoeMLP.forward_batch(x)             x [T, H]   -> out [T, H]   (batched)
    MoeMLP.forward_device(x, out, ...)  torch CUDA tensors, async on a stream
    QuantLinear(bits, q, scale).forward(x) / .dequantize()
    QuantLinear.set_path(PATH_TENSOR)   prefill-sized projections on the tensor cores
    quantize_int8(w) / quantize_int4(w) -> (codes, scales)  on the GPU
    MoeMLP.from_file(path, prefix, top_k)  a layer from a safetensors file
    LayerFile(path).tensor(name) / .layer_desc(prefix, top_k)   the mapped file
    qgmoe.checkpoint.save_layer / save_layer_raw, python -m qgmoe.quantize_layer

Every call goes to the CUDA library; there is no CPU fallback.  A failing
status raises QgmoeError with the library's message.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .build import LIB, build as _build

ROUTER_TOPK = 0
ROUTER_PREFIX = 1
SCALE_F16 = 0
SCALE_F32 = 1
PATH_AUTO = 0
PATH_CUDA_CORE = 1
PATH_TENSOR = 2

# status codes (include/qgmoe.h)
ERR_INVALID_ARG, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_DEVICE_FLAG, ERR_UNSUPPORTED, ERR_NO_DEVICE = (
    -1, -2, -3, -4, -5, -6, -7)

_vp = C.c_void_p


class QgmoeError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: {status_text(status)} ({status}): {last_error()}")
        self.status = status


class _Desc(C.Structure):
    _fields_ = [
        ("n_embed", C.c_int32), ("n_experts", C.c_int32), ("top_k", C.c_int32),
        ("n_moe_mlp", C.c_int32), ("n_shared_mlp", C.c_int32), ("bits", C.c_int32),
        ("router_mode", C.c_int32), ("scale_dtype", C.c_int32),
        ("weights_on_device", C.c_int32), ("device", C.c_int32),
        ("router", _vp), ("shared_gate", _vp),
        ("gate_up", _vp), ("down", _vp),
        ("shared_gate_proj", _vp), ("shared_up_proj", _vp), ("shared_down_proj", _vp),
        ("gate_up_q", _vp), ("gate_up_scale", _vp),
        ("down_q", _vp), ("down_scale", _vp),
        ("shared_gate_q", _vp), ("shared_gate_scale", _vp),
        ("shared_up_q", _vp), ("shared_up_scale", _vp),
        ("shared_down_q", _vp), ("shared_down_scale", _vp),
        ("ep_world", C.c_int32), ("ep_rank", C.c_int32),
        ("ep_slot", _vp),
        ("router_bits", C.c_int32), ("router_q", _vp), ("router_scale", _vp),
        ("shared_bits", C.c_int32),
    ]


# Every symbol include/qgmoe.h declares, with its ctypes signature.
SIGNATURES = {
    "qgmoe_create": ([C.POINTER(_Desc), C.POINTER(_vp)], C.c_int),
    "qgmoe_destroy": ([_vp], C.c_int),
    "qgmoe_forward": ([_vp, _vp, C.c_int32, _vp, _vp, _vp], C.c_int),
    "qgmoe_forward_device": ([_vp, _vp, C.c_int32, _vp, _vp, _vp, _vp], C.c_int),
    "qgmoe_sync": ([_vp, _vp], C.c_int),
    "qgmoe_ep_dispatch": ([_vp, _vp, C.c_int32, _vp, _vp], C.c_int),
    "qgmoe_ep_send_counts": ([_vp, C.POINTER(C.c_int32), _vp], C.c_int),
    "qgmoe_ep_experts": ([_vp, _vp, C.c_int32, C.POINTER(C.c_int32), _vp, _vp], C.c_int),
    "qgmoe_ep_combine": ([_vp, _vp, C.c_int32, _vp, _vp, _vp, _vp], C.c_int),
    "qgmoe_ep_px_setup": ([_vp, C.c_int32, _vp], C.c_int),
    "qgmoe_ep_px_connect": ([_vp, _vp], C.c_int),
    "qgmoe_ep_px_forward": ([_vp, _vp, C.c_int32, _vp, _vp], C.c_int),
    "qgmoe_last_launch_count": ([_vp], C.c_int),
    "qgmoe_set_path": ([_vp, C.c_int32], C.c_int),
    "qgmoe_set_decode_speculation": ([_vp, C.c_int32], C.c_int),
    "qgmoe_set_wait_limit": ([_vp, C.c_int64], C.c_int),
    "qgmoe_set_graphs": ([_vp, C.c_int32], C.c_int),
    "qgmoe_set_timing": ([_vp, C.c_int32], C.c_int),
    "qgmoe_read_timing": ([_vp, C.POINTER(C.c_float), C.c_int32, C.POINTER(C.c_int32)], C.c_int),
    "qgmoe_stage_name": ([_vp, C.c_int32], C.c_char_p),
    "qgql_create": ([C.c_int32, C.c_int32, C.c_int32, _vp, _vp, C.c_int32, C.c_int32, C.c_int32,
                     C.POINTER(_vp)], C.c_int),
    "qgql_destroy": ([_vp], C.c_int),
    "qgql_forward": ([_vp, _vp, C.c_int32, _vp], C.c_int),
    "qgql_forward_device": ([_vp, _vp, C.c_int32, _vp, _vp], C.c_int),
    "qgql_set_path": ([_vp, C.c_int32], C.c_int),
    "qgql_sync": ([_vp, _vp], C.c_int),
    "qgmoe_file_open": ([C.c_char_p, C.POINTER(_vp)], C.c_int),
    "qgmoe_file_close": ([_vp], C.c_int),
    "qgmoe_file_tensor": ([_vp, C.c_char_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                           C.POINTER(C.c_int64), C.POINTER(_vp), C.POINTER(C.c_int64)], C.c_int),
    "qgmoe_file_layer_desc": ([_vp, C.c_char_p, C.c_int32, C.c_int32, C.c_int32,
                               C.POINTER(_Desc)], C.c_int),
    "qgql_dequantize_device": ([_vp, _vp, _vp], C.c_int),
    "qgql_quantize_device": ([C.c_int32, C.c_int32, C.c_int32, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "qg_randn_device": ([C.c_uint64, C.c_uint64, C.c_uint64, C.c_int64, C.c_float, _vp, _vp],
                        C.c_int),
    "qgmoe_route_static": ([_vp, _vp, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                            _vp, _vp, _vp, _vp], C.c_int),
    "qgmoe_strerror": ([C.c_int], C.c_char_p),
    "qgmoe_last_error": ([], C.c_char_p),
    "qgmoe_device_ok": ([C.c_int32], C.c_int),
}

_lib = None


def lib(build_if_missing: bool = True):
    """Loads libqgmoe.so (building it in-tree first when it is absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            if not build_if_missing:
                raise QgmoeError(-6, f"{LIB} not built")
            _build()
        L = C.CDLL(LIB)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def status_text(status: int) -> str:
    return lib().qgmoe_strerror(status).decode()


def last_error() -> str:
    return lib().qgmoe_last_error().decode()


def _check(status: int, what: str):
    if status != 0:
        raise QgmoeError(status, what)


def _ptr(a) -> int | None:
    """Address of a numpy array or torch tensor (None passes NULL)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
        return a.ctypes.data
    assert a.is_contiguous(), "tensors must be contiguous"
    return a.data_ptr()


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)


def _is_dev(a) -> bool:
    return a is not None and not isinstance(a, np.ndarray) and a.is_cuda


class MoeMLP:
    """moeMLP (model/moe.go:10-99) on one B200.

    Weight arguments follow the reference layouts ((out, in) rows):
      router [E,H] f32, shared_gate [H] f32 (when Is > 0),
      bits 32: gate_up [E,2I,H], down [E,H,I], shared_{gate,up}_proj [Is,H],
               shared_down_proj [H,Is] float32;
      bits 8/4: the same tensors as quantLinear codes (uint8) with group-32
               scales (fp16 bits as uint16, or float32 with scale_dtype=F32).
    bits 16: raw bf16 experts (gateUpRaw / downRaw) as uint16 bit patterns in
               the *_q arguments, no scales.
    shared_bits (0 = bits) gives the shared expert its own format (the
    shared_* arguments in that format); router_bits 16 / 8 / 4 takes the
    router as bf16 bits or quantLinear codes in router_q (+ router_scale)
    instead of float32 rows (routerQuant, model/moe.go:16).
    Arrays may be numpy (host) or torch CUDA tensors (device); create()
    copies them.
    """

    def __init__(self, *, n_embed, n_experts, top_k, n_moe_mlp, n_shared_mlp=0, bits=32,
                 router_mode=ROUTER_TOPK, scale_dtype=SCALE_F16, device=0, ep_world=1, ep_rank=0,
                 ep_slot=None, router=None, shared_gate=None, router_bits=0, router_q=None,
                 router_scale=None, shared_bits=0,
                 gate_up=None, down=None, shared_gate_proj=None, shared_up_proj=None,
                 shared_down_proj=None, gate_up_q=None, gate_up_scale=None, down_q=None,
                 down_scale=None, shared_gate_q=None, shared_gate_scale=None, shared_up_q=None,
                 shared_up_scale=None, shared_down_q=None, shared_down_scale=None):
        arrays = dict(router=router, router_q=router_q, router_scale=router_scale,
                      shared_gate=shared_gate, gate_up=gate_up, down=down,
                      shared_gate_proj=shared_gate_proj, shared_up_proj=shared_up_proj,
                      shared_down_proj=shared_down_proj, gate_up_q=gate_up_q,
                      gate_up_scale=gate_up_scale, down_q=down_q, down_scale=down_scale,
                      shared_gate_q=shared_gate_q, shared_gate_scale=shared_gate_scale,
                      shared_up_q=shared_up_q, shared_up_scale=shared_up_scale,
                      shared_down_q=shared_down_q, shared_down_scale=shared_down_scale)
        present = [v for v in arrays.values() if v is not None]
        on_dev = _is_dev(present[0]) if present else False
        if any(_is_dev(v) != on_dev for v in present):
            raise ValueError("weights must be all host arrays or all device tensors")
        d = _Desc()
        d.n_embed, d.n_experts, d.top_k, d.n_moe_mlp = n_embed, n_experts, top_k, n_moe_mlp
        d.n_shared_mlp, d.bits, d.router_mode, d.scale_dtype = n_shared_mlp, bits, router_mode, \
            scale_dtype
        d.weights_on_device, d.device = int(on_dev), device
        d.ep_world, d.ep_rank = ep_world, ep_rank
        d.router_bits, d.shared_bits = router_bits, shared_bits
        slot = None
        if ep_slot is not None:
            slot = np.ascontiguousarray(ep_slot, np.int32)
            d.ep_slot = slot.ctypes.data_as(_vp)
        for name, v in arrays.items():
            setattr(d, name, _ptr(v))
        self._keep = (arrays, slot)  # alive until create() has copied them
        h = _vp()
        _check(lib().qgmoe_create(C.byref(d), C.byref(h)), "qgmoe_create")
        self._keep = None
        self.h = h
        self.n_embed, self.top_k, self.n_experts = n_embed, top_k, n_experts
        self.device = device
        self.ep_world, self.ep_rank = ep_world, ep_rank

    @classmethod
    def from_file(cls, path: str, prefix: str, top_k: int, router_mode: int = ROUTER_TOPK,
                  device: int = 0) -> "MoeMLP":
        """The quantised layer stored under `prefix` in a safetensors file
        (qgmoe_file_layer_desc): the tensors are mapped, not read, and
        create() copies them from the mapping to the device."""
        f = LayerFile(path)
        try:
            d = f.layer_desc(prefix, top_k, router_mode, device)
            h = _vp()
            _check(lib().qgmoe_create(C.byref(d), C.byref(h)), "qgmoe_create")
        finally:
            f.close()
        self = cls.__new__(cls)
        self._keep = None
        self.h = h
        self.n_embed, self.top_k, self.n_experts = d.n_embed, top_k, d.n_experts
        self.device = device
        self.ep_world, self.ep_rank = 1, 0
        return self

    def close(self):
        if getattr(self, "h", None):
            lib().qgmoe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x: np.ndarray) -> np.ndarray:
        """mixer.forward: one token x [H] -> out [H]."""
        return self.forward_batch(np.asarray(x, np.float32).reshape(1, -1))[0]

    def forward_batch(self, x: np.ndarray, return_routing: bool = False):
        """T tokens from host memory (blocking).  With return_routing, also
        the selected experts [T,k] (routing order) and their weights [T,k]."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        out = np.empty((T, self.n_embed), np.float32)
        idx = np.empty((T, self.top_k), np.int32) if return_routing else None
        w = np.empty((T, self.top_k), np.float32) if return_routing else None
        _check(lib().qgmoe_forward(self.h, _ptr(x), T, _ptr(out), _ptr(idx), _ptr(w)),
               "qgmoe_forward")
        return (out, idx, w) if return_routing else out

    def forward_device(self, x, out, sel_idx=None, sel_w=None, stream=None):
        """Enqueue on device tensors (torch CUDA); call sync() to wait."""
        T = x.shape[0]
        _check(lib().qgmoe_forward_device(self.h, _ptr(x), T, _ptr(out), _ptr(sel_idx),
                                          _ptr(sel_w), _stream_ptr(stream)),
               "qgmoe_forward_device")

    def sync(self, stream=None):
        _check(lib().qgmoe_sync(self.h, _stream_ptr(stream)), "qgmoe_sync")

    def last_launch_count(self) -> int:
        return lib().qgmoe_last_launch_count(self.h)

    def set_path(self, mode: int):
        """PATH_AUTO, PATH_CUDA_CORE or PATH_TENSOR (see include/qgmoe.h)."""
        _check(lib().qgmoe_set_path(self.h, mode), "qgmoe_set_path")

    def set_decode_speculation(self, enable: bool = True):
        """Stream the approximate top-k's experts while the exact router
        logits are summed (default on); results are the same either way."""
        _check(lib().qgmoe_set_decode_speculation(self.h, int(enable)),
               "qgmoe_set_decode_speculation")

    def set_wait_limit(self, microseconds: int = 0):
        """Limit of the device waits on other CTAs / ranks (0: defaults)."""
        _check(lib().qgmoe_set_wait_limit(self.h, int(microseconds)), "qgmoe_set_wait_limit")

    def set_graphs(self, enable: bool = True):
        """CUDA-graph replay of repeated identical forwards (default on)."""
        _check(lib().qgmoe_set_graphs(self.h, int(enable)), "qgmoe_set_graphs")

    def set_timing(self, enable: bool = True):
        _check(lib().qgmoe_set_timing(self.h, int(enable)), "qgmoe_set_timing")

    def read_timing(self):
        """(per-stage ms summed over the timed forwards since the last read,
        number of those forwards), stages in launch order."""
        buf = (C.c_float * 16)()
        nf = C.c_int32(0)
        n = lib().qgmoe_read_timing(self.h, buf, 16, C.byref(nf))
        if n < 0:
            raise QgmoeError(n, "qgmoe_read_timing")
        return {lib().qgmoe_stage_name(self.h, i).decode(): buf[i] for i in range(n)}, nf.value


class QuantLinear:
    """quantLinear (model/moe.go:126-162): group-32 int8/int4 weights with
    fp16 scales (or bits=32 for a plain float32 linear)."""

    def __init__(self, bits, out_features, in_features, qweight, scale=None,
                 scale_dtype=SCALE_F16, device=0):
        on_dev = _is_dev(qweight)
        h = _vp()
        _check(lib().qgql_create(bits, out_features, in_features, _ptr(qweight), _ptr(scale),
                                 scale_dtype, int(on_dev), device, C.byref(h)), "qgql_create")
        self.h = h
        self.bits, self.out_features, self.in_features = bits, out_features, in_features
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            lib().qgql_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x: np.ndarray) -> np.ndarray:
        """y = x W^T for x [in] or [T, in] (host arrays, blocking)."""
        x = np.ascontiguousarray(x, np.float32)
        x2 = x.reshape(-1, self.in_features)
        y = np.empty((x2.shape[0], self.out_features), np.float32)
        _check(lib().qgql_forward(self.h, _ptr(x2), x2.shape[0], _ptr(y)), "qgql_forward")
        return y.reshape(x.shape[:-1] + (self.out_features,))

    def forward_device(self, x, y, stream=None):
        _check(lib().qgql_forward_device(self.h, _ptr(x), x.shape[0], _ptr(y),
                                         _stream_ptr(stream)), "qgql_forward_device")

    def set_path(self, mode: int):
        """PATH_AUTO, PATH_CUDA_CORE or PATH_TENSOR (qgql_set_path)."""
        _check(lib().qgql_set_path(self.h, mode), "qgql_set_path")

    def sync(self, stream=None):
        """Waits for the stream; raises on a device error flag (qgql_sync)."""
        _check(lib().qgql_sync(self.h, _stream_ptr(stream)), "qgql_sync")

    def dequantize(self):
        """quantLinear.dequantize: the [out, in] float32 matrix (torch CUDA)."""
        import torch
        w = torch.empty((self.out_features, self.in_features), dtype=torch.float32,
                        device=f"cuda:{self.device}")
        _check(lib().qgql_dequantize_device(self.h, _ptr(w), None), "qgql_dequantize_device")
        torch.cuda.synchronize(self.device)
        return w


def quantize_device(w, bits: int, stream=None):
    """quantizeInt8/Int4 on the GPU: w [O, I] float32 CUDA tensor ->
    (codes uint8, scales float32, scales fp16 as int16 bits)."""
    import torch
    O, I = w.shape
    q = torch.empty((O, I if bits == 8 else I // 2), dtype=torch.uint8, device=w.device)
    s32 = torch.empty((O, I // 32), dtype=torch.float32, device=w.device)
    s16 = torch.empty((O, I // 32), dtype=torch.int16, device=w.device)
    _check(lib().qgql_quantize_device(bits, O, I, _ptr(w.contiguous()), _ptr(q), _ptr(s32),
                                      _ptr(s16), _stream_ptr(stream)), "qgql_quantize_device")
    return q, s32, s16


def quantize_int8(w):
    return quantize_device(w, 8)


def quantize_int4(w):
    return quantize_device(w, 4)


def randn_device(out, seed: int, stream_id: int, std: float = 1.0, offset: int = 0,
                 cuda_stream=None):
    """Fill a float32 CUDA tensor from the counter-based generator."""
    _check(lib().qg_randn_device(seed, stream_id, offset, out.numel(), std, _ptr(out),
                                 _stream_ptr(cuda_stream)), "qg_randn_device")
    return out


DT_F32, DT_F16, DT_BF16, DT_I8, DT_U8, DT_I32, DT_OTHER = range(7)


class LayerFile:
    """A safetensors file mapped by the library (qgmoe_file_open): tensor
    lookup and the qgmoe_desc of one quantised MoE layer (host only)."""

    def __init__(self, path: str):
        h = _vp()
        _check(lib().qgmoe_file_open(os.fsencode(path), C.byref(h)), "qgmoe_file_open")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().qgmoe_file_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def tensor(self, name: str):
        """(dtype code, shape tuple, address inside the mapping, bytes)."""
        dt, rank = C.c_int32(), C.c_int32()
        shape = (C.c_int64 * 8)()
        data, nbytes = _vp(), C.c_int64()
        _check(lib().qgmoe_file_tensor(self.h, name.encode(), C.byref(dt), C.byref(rank), shape,
                                       C.byref(data), C.byref(nbytes)), "qgmoe_file_tensor")
        return dt.value, tuple(shape[i] for i in range(rank.value)), data.value or 0, nbytes.value

    def layer_desc(self, prefix: str, top_k: int, router_mode: int = ROUTER_TOPK,
                   device: int = 0) -> _Desc:
        d = _Desc()
        _check(lib().qgmoe_file_layer_desc(self.h, prefix.encode(), top_k, router_mode, device,
                                           C.byref(d)), "qgmoe_file_layer_desc")
        return d
