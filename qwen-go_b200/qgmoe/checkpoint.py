"""Quantised MoE layers on disk: the writer for the layout qgmoe_file_*
reads (include/qgmoe.h).

qwen-go stores quantised linears as <name>.qweight / <name>.scale tensor
pairs in safetensors shards listed by quant.json ({"bits": ..., "quantized":
[...]}, model/load.go:478-582, written by cmd/qwen-quant); its MoE loader
takes the stacked expert tensors only as float blobs (model/load.go:
415-456).  save_layer writes one MoE layer with the stacked expert codes
and fp16 (or f32) group scales under the same mlp.* names:

    <prefix>gate.weight                      F32 [E, H]
    <prefix>experts.gate_up_proj.qweight     I8 [E, 2I, H] (int8) / U8 [E, 2I, H/2] (int4)
    <prefix>experts.gate_up_proj.scale       F16 or F32 [E, 2I, H/32]
    <prefix>experts.down_proj.qweight/.scale [E, H, I] ... / [E, H, I/32]
    <prefix>shared_expert.{gate,up,down}_proj.qweight/.scale   (optional)
    <prefix>shared_expert_gate.weight        F32 [1, H]        (with the shared expert)

save_layer_raw writes a layer with raw stacked experts instead, as the
reference reads them from bf16 checkpoints (<prefix>experts.gate_up_proj.weight
BF16 [E, 2I, H], .down_proj.weight BF16 [E, H, I], shared_expert.*.weight);
qgmoe_file_layer_desc takes either form (bits 16 for BF16, 32 for F32).
save_layer_groups writes each group (router, routed experts, shared expert)
in its own format, as the reference's checkpoints mix them: cmd/qwen-quant
quantises an MoE model's shared-expert projections and leaves the router and
the stacked experts raw (cmd/qwen-quant/main.go:61-65), and a quantised
router (mlp.gate.qweight / .scale) loads as routerQuant (model/load.go:651).

Tensor data starts on 64-byte boundaries (the header is space-padded), so
the mapped tensors are aligned for any element type.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

_DTYPES = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int8): "I8",
           np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32"}
_ALIGN = 64


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None,
                      bf16: set | None = None) -> None:
    """tensors: name -> numpy array (float32/float16/int8/uint8/int32), in
    the order given; uint16 arrays are fp16 bit patterns, or bf16 bit
    patterns for the names in `bf16`."""
    header = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs, off = [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        dt = None
        if a.dtype == np.uint16:
            if bf16 and name in bf16:
                dt = "BF16"
            else:  # fp16 bit patterns
                a = a.view(np.float16)
        if dt is None and a.dtype not in _DTYPES:
            raise TypeError(f"{name}: unsupported dtype {a.dtype}")
        pad = (-off) % _ALIGN
        if pad:
            blobs.append(b"\0" * pad)
            off += pad
        raw = a.tobytes()
        header[name] = {"dtype": dt or _DTYPES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((-(8 + len(hj))) % _ALIGN)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def read_header(path: str) -> dict:
    """The JSON header of a safetensors file (independent of the library)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        return json.loads(f.read(n))


def save_layer(path: str, prefix: str, *, router, gate_up_q, gate_up_scale, down_q, down_scale,
               bits: int, shared_gate=None, shared_gate_q=None, shared_gate_scale=None,
               shared_up_q=None, shared_up_scale=None, shared_down_q=None,
               shared_down_scale=None, quant_json: str | None = None, append: dict | None = None):
    """Writes one quantised MoE layer (the arrays qgmoe.MoeMLP takes for bits
    8/4, with E, 2I, H / E, H, I leading shapes) to `path`; `append` adds
    more tensors to the same file (other layers).  With quant_json, also
    writes the reference's manifest listing the quantised tensors."""
    if bits not in (8, 4):
        raise ValueError("bits must be 8 or 4")
    router = np.asarray(router, np.float32)
    E, H = router.shape
    t = dict(append or {})
    t[prefix + "gate.weight"] = router

    def codes(q, lead_shape):
        q = np.asarray(q)
        q = q.view(np.int8) if bits == 8 else q.view(np.uint8)
        return q.reshape(lead_shape + (-1,))

    def scales(s, lead_shape):
        s = np.asarray(s)
        if s.dtype not in (np.float32, np.float16, np.uint16):
            raise TypeError("scales: float32, float16 or fp16 bits (uint16)")
        return s.reshape(lead_shape + (-1,))

    gu_rows = np.asarray(gate_up_scale).size // (E * (H // 32))
    I = gu_rows // 2
    t[prefix + "experts.gate_up_proj.qweight"] = codes(gate_up_q, (E, 2 * I))
    t[prefix + "experts.gate_up_proj.scale"] = scales(gate_up_scale, (E, 2 * I))
    t[prefix + "experts.down_proj.qweight"] = codes(down_q, (E, H))
    t[prefix + "experts.down_proj.scale"] = scales(down_scale, (E, H))
    names = [prefix + "experts.gate_up_proj.weight", prefix + "experts.down_proj.weight"]
    if shared_gate_q is not None:
        Is = np.asarray(shared_gate_scale).size // (H // 32)
        for base, q, s, rows in (("shared_expert.gate_proj", shared_gate_q, shared_gate_scale, Is),
                                 ("shared_expert.up_proj", shared_up_q, shared_up_scale, Is),
                                 ("shared_expert.down_proj", shared_down_q, shared_down_scale, H)):
            t[prefix + base + ".qweight"] = codes(q, (rows,))
            t[prefix + base + ".scale"] = scales(s, (rows,))
            names.append(prefix + base + ".weight")
        t[prefix + "shared_expert_gate.weight"] = np.asarray(shared_gate, np.float32).reshape(1, H)
    write_safetensors(path, t, {"format": "pt", "qgmoe_bits": bits})
    if quant_json:
        man = {"bits": bits, "quantized": names}
        if os.path.exists(quant_json):
            with open(quant_json) as f:
                old = json.load(f)
            if old.get("bits") != bits:
                raise ValueError("quant.json already lists another bit width")
            man["quantized"] = list(dict.fromkeys(old.get("quantized", []) + names))
        with open(quant_json, "w") as f:
            json.dump(man, f, indent=1)


def save_layer_raw(path: str, prefix: str, *, router, gate_up, down, shared_gate=None,
                   shared_gate_proj=None, shared_up_proj=None, shared_down_proj=None,
                   bf16: bool = True, append: dict | None = None,
                   append_bf16: set | None = None):
    """One MoE layer with raw (unquantised) stacked experts, as the reference's
    loader reads them (model/load.go:419-449): <prefix>experts.gate_up_proj.weight
    [E, 2I, H] and .down_proj.weight [E, H, I] in BF16 (uint16 bit patterns,
    e.g. from qg_oracle.bf16_bits) or F32, the shared expert's .weight
    tensors likewise, the router and shared-expert gate in F32 (or BF16 bits
    when given as uint16).  `append` adds other tensors to the file, those
    named in `append_bf16` being bf16 bit patterns."""
    t = dict(append or {})
    names16 = set(append_bf16 or ())

    def put(name, a):
        a = np.asarray(a)
        if bf16 or a.dtype == np.uint16:
            if a.dtype != np.uint16:
                raise TypeError(f"{name}: bf16 bit patterns (uint16) expected")
            names16.add(name)
        elif a.dtype != np.float32:
            raise TypeError(f"{name}: float32 expected")
        t[name] = a

    r = np.asarray(router)
    t[prefix + "gate.weight"] = r
    if r.dtype == np.uint16:
        names16.add(prefix + "gate.weight")
    E, H = r.shape
    put(prefix + "experts.gate_up_proj.weight", np.asarray(gate_up).reshape(E, -1, H))
    put(prefix + "experts.down_proj.weight", np.asarray(down).reshape(E, H, -1))
    if shared_gate_proj is not None:
        put(prefix + "shared_expert.gate_proj.weight", shared_gate_proj)
        put(prefix + "shared_expert.up_proj.weight", shared_up_proj)
        put(prefix + "shared_expert.down_proj.weight", shared_down_proj)
        g = np.asarray(shared_gate).reshape(1, H)
        t[prefix + "shared_expert_gate.weight"] = g
        if g.dtype == np.uint16:
            names16.add(prefix + "shared_expert_gate.weight")
    write_safetensors(path, t, {"format": "pt"}, bf16=names16)


def save_layer_groups(path: str, prefix: str, *, router, experts, shared=None, shared_gate=None,
                      append: dict | None = None, quant_json: str | None = None):
    """One MoE layer, each group in its own format.  A weight is given as a
    float32 array (F32 <name>.weight), a uint16 array of bf16 bit patterns
    (BF16 <name>.weight) or a (codes, scales) pair of a quantised linear
    (<name>.qweight I8 [.., K] for int8 or U8 [.., K/2] for int4, <name>.scale
    F32, F16 or fp16 bits as uint16, [.., K/32]).
      router      [E, H]
      experts     (gate_up [E, 2I, H], down [E, H, I])
      shared      (gate_proj [Is, H], up_proj [Is, H], down_proj [H, Is]) or None
      shared_gate [H] float32 (with the shared expert)
    With quant_json, also writes the reference's manifest of the quantised
    tensors (one bit width per manifest, as the reference's)."""
    t = dict(append or {})
    names16, quantised, widths = set(), [], set()

    def put(base, w, lead):
        if isinstance(w, tuple):
            q, s = (np.asarray(a) for a in w)
            s = s.reshape(lead + (-1,))
            K = s.shape[-1] * 32
            q = q.reshape(lead + (-1,))
            bits = 8 if q.shape[-1] == K else 4
            if bits == 4 and 2 * q.shape[-1] != K:
                raise ValueError(f"{base}: codes of width {q.shape[-1]} do not fit {K} inputs")
            t[prefix + base + ".qweight"] = q.view(np.int8) if bits == 8 else q.view(np.uint8)
            if s.dtype not in (np.float32, np.float16, np.uint16):
                raise TypeError(f"{base}: scales must be float32, float16 or fp16 bits")
            t[prefix + base + ".scale"] = s
            quantised.append(prefix + base + ".weight")
            widths.add(bits)
            return
        a = np.asarray(w)
        if a.dtype == np.uint16:
            names16.add(prefix + base + ".weight")
        elif a.dtype != np.float32:
            raise TypeError(f"{base}: float32, bf16 bits (uint16) or (codes, scales) expected")
        t[prefix + base + ".weight"] = a.reshape(lead + (-1,))

    def rows_cols(w):  # (rows, inputs) of a weight in any of the three forms
        if isinstance(w, tuple):
            s = np.asarray(w[1])
            K = s.shape[-1] * 32
            return s.size // s.shape[-1], K
        a = np.asarray(w)
        return a.size // a.shape[-1], a.shape[-1]

    E, H = rows_cols(router)
    gu, dn = experts
    put("gate", router, (E,))
    put("experts.gate_up_proj", gu, (E, rows_cols(gu)[0] // E))
    put("experts.down_proj", dn, (E, H))
    if shared is not None:
        sg, su, sd = shared
        Is = rows_cols(sg)[0]
        put("shared_expert.gate_proj", sg, (Is,))
        put("shared_expert.up_proj", su, (Is,))
        put("shared_expert.down_proj", sd, (H,))
        t[prefix + "shared_expert_gate.weight"] = np.asarray(shared_gate, np.float32).reshape(1, H)
    write_safetensors(path, t, {"format": "pt"}, bf16=names16)
    if quant_json and quantised:
        if len(widths) != 1:
            raise ValueError("quant.json holds one bit width; the layer mixes int8 and int4")
        with open(quant_json, "w") as f:
            json.dump({"bits": widths.pop(), "quantized": quantised}, f, indent=1)
