"""On-disk quantised MoE layers (qgmoe_file_*, qgmoe.checkpoint): the writer's
safetensors layout, the library's header parser and tensor lookup, and the
qgmoe_desc it builds, checked byte for byte against the arrays written.
Host only (no CUDA call); the device side is qgmoe_create, tested elsewhere."""
import ctypes as C
import json
import struct

import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from qgmoe import checkpoint as ck


def _layer(bits, Is, seed=5):
    return O.make_moe(H=128, E=4, k=2, I=64, Is=Is, bits=bits, seed=seed)


def _save(tmp_path, m, prefix="model.layers.0.mlp.", scale="f16", **kw):
    sc = (lambda n: m.s16[n]) if scale == "f16" else (lambda n: m.s[n].astype(np.float32))
    args = dict(router=m.router, gate_up_q=m.q["gate_up"], gate_up_scale=sc("gate_up"),
                down_q=m.q["down"], down_scale=sc("down"), bits=m.bits)
    if m.Is:
        args.update(shared_gate=m.shared_gate, shared_gate_q=m.q["sh_gate"],
                    shared_gate_scale=sc("sh_gate"), shared_up_q=m.q["sh_up"],
                    shared_up_scale=sc("sh_up"), shared_down_q=m.q["sh_down"],
                    shared_down_scale=sc("sh_down"))
    args.update(kw)
    path = str(tmp_path / "layer.safetensors")
    ck.save_layer(path, prefix, **args)
    return path


def _bytes(addr, a):
    a = np.ascontiguousarray(a)
    return C.string_at(addr, a.nbytes) == a.tobytes()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("Is", [0, 128])
@pytest.mark.parametrize("scale", ["f16", "f32"])
def test_layer_desc_points_at_the_written_arrays(tmp_path, bits, Is, scale):
    m = _layer(bits, Is)
    qj = str(tmp_path / "quant.json")
    path = _save(tmp_path, m, scale=scale, quant_json=qj)
    with qgmoe.LayerFile(path) as f:
        d = f.layer_desc("model.layers.0.mlp.", top_k=2, router_mode=qgmoe.ROUTER_PREFIX, device=3)
        assert (d.n_embed, d.n_experts, d.top_k, d.n_moe_mlp, d.n_shared_mlp) == (128, 4, 2, 64, Is)
        assert (d.bits, d.router_mode, d.device, d.weights_on_device) == (bits, 1, 3, 0)
        assert d.scale_dtype == (qgmoe.SCALE_F16 if scale == "f16" else qgmoe.SCALE_F32)
        assert d.ep_world == 0 and not d.ep_slot and not d.gate_up and not d.down
        assert _bytes(d.router, m.router)
        pairs = [("gate_up", d.gate_up_q, d.gate_up_scale), ("down", d.down_q, d.down_scale)]
        if Is:
            pairs += [("sh_gate", d.shared_gate_q, d.shared_gate_scale),
                      ("sh_up", d.shared_up_q, d.shared_up_scale),
                      ("sh_down", d.shared_down_q, d.shared_down_scale)]
            assert _bytes(d.shared_gate, m.shared_gate)
        else:
            assert not d.shared_gate_q and not d.shared_gate
        for name, q, s in pairs:
            assert _bytes(q, m.q[name]), name
            want = m.s16[name] if scale == "f16" else m.s[name].astype(np.float32)
            assert _bytes(s, want), name
            assert q % 64 == 0 and s % 64 == 0  # aligned for any element type
    man = json.load(open(qj))
    assert man["bits"] == bits
    assert "model.layers.0.mlp.experts.gate_up_proj.weight" in man["quantized"]
    assert ("model.layers.0.mlp.shared_expert.down_proj.weight" in man["quantized"]) == bool(Is)


def test_tensor_lookup_matches_an_independent_header_parse(tmp_path):
    m = _layer(4, 128)
    path = _save(tmp_path, m)
    hdr = ck.read_header(path)
    codes = {"F32": qgmoe.DT_F32, "F16": qgmoe.DT_F16, "I8": qgmoe.DT_I8, "U8": qgmoe.DT_U8}
    with open(path, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        raw = fh.read()
    data = raw[n:]
    with qgmoe.LayerFile(path) as f:
        for name, t in hdr.items():
            if name == "__metadata__":
                continue
            dt, shape, addr, nbytes = f.tensor(name)
            assert dt == codes[t["dtype"]] and list(shape) == t["shape"], name
            b0, b1 = t["data_offsets"]
            assert nbytes == b1 - b0
            assert C.string_at(addr, nbytes) == data[b0:b1]
        with pytest.raises(qgmoe.QgmoeError):
            f.tensor("model.layers.0.mlp.no_such.weight")
    assert hdr["__metadata__"]["qgmoe_bits"] == "4"
    assert hdr["model.layers.0.mlp.experts.gate_up_proj.qweight"]["shape"] == [4, 128, 64]


def test_two_layers_in_one_file(tmp_path):
    a, b = _layer(8, 0, seed=7), _layer(8, 0, seed=8)
    first = {}
    pa = _save(tmp_path, a, prefix="model.layers.1.mlp.")
    hdr = ck.read_header(pa)
    with open(pa, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        data = fh.read()[n:]
    for name, t in hdr.items():
        if name != "__metadata__":
            dt = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8}[t["dtype"]]
            b0, b1 = t["data_offsets"]
            first[name] = np.frombuffer(data[b0:b1], dt).reshape(t["shape"])
    path = _save(tmp_path, b, prefix="model.layers.2.mlp.", append=first)
    with qgmoe.LayerFile(path) as f:
        d1 = f.layer_desc("model.layers.1.mlp.", 2)
        d2 = f.layer_desc("model.layers.2.mlp.", 2)
        assert _bytes(d1.gate_up_q, a.q["gate_up"]) and _bytes(d2.gate_up_q, b.q["gate_up"])
        assert _bytes(d1.router, a.router) and _bytes(d2.router, b.router)
        with pytest.raises(qgmoe.QgmoeError):
            f.layer_desc("model.layers.3.mlp.", 2)


def _write_raw(path, header: dict, data: bytes = b"", pad=True):
    hj = json.dumps(header).encode()
    if pad:
        hj += b" " * ((-(8 + len(hj))) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj + data)


def test_malformed_files_are_rejected(tmp_path):
    p = str(tmp_path / "bad.safetensors")
    for content in (b"", b"\x01\x02", struct.pack("<Q", 1 << 40) + b"{}", struct.pack("<Q", 3) + b"{x}",
                    struct.pack("<Q", 2) + b"[]"):
        with open(p, "wb") as f:
            f.write(content)
        with pytest.raises(qgmoe.QgmoeError):
            qgmoe.LayerFile(p)
    # data beyond the file, byte count not matching the shape, missing keys,
    # a byte count that overflows
    for hdr, data in (({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8),
                      ({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}}, b"\0" * 16),
                      ({"a": {"dtype": "F32", "shape": [4]}}, b"\0" * 16),
                      ({"a": {"dtype": "F32", "shape": [-4], "data_offsets": [0, 16]}}, b"\0" * 16),
                      # 2^62 float32s: the byte count wraps to 0 in 64 bits
                      ({"a": {"dtype": "F32", "shape": [1 << 62], "data_offsets": [0, 0]}}, b"")):
        _write_raw(p, hdr, data)
        with pytest.raises(qgmoe.QgmoeError):
            qgmoe.LayerFile(p)
    # a well-formed file with escapes, metadata and an unknown dtype opens
    # (json.dumps writes the non-ASCII key as a \u escape)
    _write_raw(p, {"__metadata__": {"k": "v\"\u00e9"},
                   "n\u00e9": {"dtype": "F8_E4M3", "shape": [2], "data_offsets": [0, 2]}}, b"\0\0")
    with qgmoe.LayerFile(p) as f:
        dt, shape, _, nbytes = f.tensor("né")
        assert dt == qgmoe.DT_OTHER and shape == (2,) and nbytes == 2


def test_layer_desc_rejects_inconsistent_layers(tmp_path):
    m = _layer(8, 0)
    p = _save(tmp_path, m)
    hdr = ck.read_header(p)
    with open(p, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        data = fh.read()[n:]
    arrays = {}
    for name, t in hdr.items():
        if name != "__metadata__":
            dt = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8}[t["dtype"]]
            b0, b1 = t["data_offsets"]
            arrays[name] = np.frombuffer(data[b0:b1], dt).reshape(t["shape"])
    pre = "model.layers.0.mlp."
    cases = [
        # router in fp16
        {pre + "gate.weight": arrays[pre + "gate.weight"].astype(np.float16)},
        # down stack with the wrong number of experts
        {pre + "experts.down_proj.qweight": arrays[pre + "experts.down_proj.qweight"][:3],
         pre + "experts.down_proj.scale": arrays[pre + "experts.down_proj.scale"][:3]},
        # gate_up scales for a different input width
        {pre + "experts.gate_up_proj.scale": arrays[pre + "experts.gate_up_proj.scale"][:, :, :2]},
        # int4-width codes stored as I8
        {pre + "experts.gate_up_proj.qweight": arrays[pre + "experts.gate_up_proj.qweight"][:, :, :64]},
        # mixed scale dtypes
        {pre + "experts.down_proj.scale":
            arrays[pre + "experts.down_proj.scale"].astype(np.float32)},
        # a shared expert with only one projection
        {pre + "shared_expert.gate_proj.qweight": np.zeros((128, 128), np.int8),
         pre + "shared_expert.gate_proj.scale": np.zeros((128, 4), np.float16)},
    ]
    q = str(tmp_path / "bad_layer.safetensors")
    for change in cases:
        t = dict(arrays)
        t.update(change)
        ck.write_safetensors(q, t)
        with qgmoe.LayerFile(q) as f:
            with pytest.raises(qgmoe.QgmoeError):
                f.layer_desc(pre, 2)
    # and the unchanged set is accepted
    ck.write_safetensors(q, arrays)
    with qgmoe.LayerFile(q) as f:
        assert f.layer_desc(pre, 2).n_experts == 4


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [8, 4])
def test_layer_from_file_matches_layer_from_arrays(tmp_path, bits):
    """qgmoe_create from the mapped file and from the same arrays gives
    bit-identical forwards (the desc differs only in where the bytes live)."""
    from moe_cases import make_gpu_moe
    m = _layer(bits, 128, seed=11)
    path = _save(tmp_path, m)
    a = make_gpu_moe(m, O.ROUTER_TOPK)
    b = qgmoe.MoeMLP.from_file(path, "model.layers.0.mlp.", top_k=2)
    x = O.randn(11, 9, (24, 128))
    assert np.array_equal(a.forward_batch(x), b.forward_batch(x))


@pytest.mark.parametrize("raw", ["bf16", "f32"])
@pytest.mark.parametrize("Is", [0, 128])
def test_raw_layers_bf16_and_f32(tmp_path, raw, Is):
    """Raw stacked experts as the reference reads them (experts.*.weight in
    BF16 or F32): bits 16 / 32 descriptors pointing into the mapping; a BF16
    router / shared gate is widened once into a buffer the handle owns."""
    m = O.make_moe(H=128, E=4, k=2, I=64, Is=Is, bits=16 if raw == "bf16" else 32, seed=6)
    pre = "model.layers.5.mlp."
    path = str(tmp_path / "raw.safetensors")
    if raw == "bf16":
        router = O.bf16_bits(m.router)  # the router in bf16 too, as in bf16 checkpoints
        args = dict(router=router, gate_up=m.q["gate_up"], down=m.q["down"])
        if Is:
            args.update(shared_gate=O.bf16_bits(m.shared_gate), shared_gate_proj=m.q["sh_gate"],
                        shared_up_proj=m.q["sh_up"], shared_down_proj=m.q["sh_down"])
        ck.save_layer_raw(path, pre, bf16=True, **args)
    else:
        args = dict(router=m.router, gate_up=m.gate_up, down=m.down)
        if Is:
            args.update(shared_gate=m.shared_gate, shared_gate_proj=m.sh_gate,
                        shared_up_proj=m.sh_up, shared_down_proj=m.sh_down)
        ck.save_layer_raw(path, pre, bf16=False, **args)
    hdr = ck.read_header(path)
    assert hdr[pre + "experts.gate_up_proj.weight"]["dtype"] == ("BF16" if raw == "bf16" else "F32")
    assert hdr[pre + "experts.gate_up_proj.weight"]["shape"] == [4, 128, 128]
    with qgmoe.LayerFile(path) as f:
        d = f.layer_desc(pre, 2)
        assert (d.n_embed, d.n_experts, d.n_moe_mlp, d.n_shared_mlp) == (128, 4, 64, Is)
        if raw == "bf16":
            assert d.bits == 16 and not d.gate_up and not d.down
            assert _bytes(d.gate_up_q, m.q["gate_up"]) and _bytes(d.down_q, m.q["down"])
            assert not d.gate_up_scale and not d.down_scale
            assert _bytes(d.router, O.bf16_widen(O.bf16_bits(m.router)))
            if Is:
                assert _bytes(d.shared_gate_q, m.q["sh_gate"])
                assert _bytes(d.shared_down_q, m.q["sh_down"])
                assert _bytes(d.shared_gate, O.bf16_widen(O.bf16_bits(m.shared_gate)))
        else:
            assert d.bits == 32 and not d.gate_up_q
            assert _bytes(d.gate_up, m.gate_up) and _bytes(d.down, m.down)
            assert _bytes(d.router, m.router)
            if Is:
                assert _bytes(d.shared_up_proj, m.sh_up) and _bytes(d.shared_gate, m.shared_gate)
        # the descriptor is stable across calls (the widened copies are reused)
        d2 = f.layer_desc(pre, 2)
        assert d2.router == d.router and d2.gate_up_q == d.gate_up_q


def test_raw_and_quantised_stacks_do_not_mix(tmp_path):
    m8 = _layer(8, 0)
    p = _save(tmp_path, m8)
    hdr = ck.read_header(p)
    with open(p, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        data = fh.read()[n:]
    arrays = {}
    for name, t in hdr.items():
        if name != "__metadata__":
            dt = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8}[t["dtype"]]
            b0, b1 = t["data_offsets"]
            arrays[name] = np.frombuffer(data[b0:b1], dt).reshape(t["shape"])
    pre = "model.layers.0.mlp."
    # down as raw bf16 next to int8 gate_up codes
    del arrays[pre + "experts.down_proj.qweight"], arrays[pre + "experts.down_proj.scale"]
    arrays[pre + "experts.down_proj.weight"] = np.zeros((4, 128, 64), np.uint16)
    q = str(tmp_path / "mixed.safetensors")
    ck.write_safetensors(q, arrays, bf16={pre + "experts.down_proj.weight"})
    with qgmoe.LayerFile(q) as f:
        with pytest.raises(qgmoe.QgmoeError):
            f.layer_desc(pre, 2)


@pytest.mark.gpu
def test_bf16_layer_from_file_matches_layer_from_arrays(tmp_path):
    m = O.make_moe(H=128, E=4, k=2, I=64, Is=128, bits=16, seed=12)
    path = str(tmp_path / "raw.safetensors")
    ck.save_layer_raw(path, "mlp.", router=m.router, gate_up=m.q["gate_up"], down=m.q["down"],
                      shared_gate=m.shared_gate, shared_gate_proj=m.q["sh_gate"],
                      shared_up_proj=m.q["sh_up"], shared_down_proj=m.q["sh_down"])
    a = qgmoe.MoeMLP(n_embed=128, n_experts=4, top_k=2, n_moe_mlp=64, n_shared_mlp=128, bits=16,
                     router=m.router, shared_gate=m.shared_gate, gate_up_q=m.q["gate_up"],
                     down_q=m.q["down"], shared_gate_q=m.q["sh_gate"], shared_up_q=m.q["sh_up"],
                     shared_down_q=m.q["sh_down"])
    b = qgmoe.MoeMLP.from_file(path, "mlp.", top_k=2)
    x = O.randn(12, 9, (16, 128))
    assert np.array_equal(a.forward_batch(x), b.forward_batch(x))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("Is", [0, 128])
def test_quantize_layer_tool(tmp_path, bits, Is):
    """qgmoe.quantize_layer: raw bf16 layer in, quantised layer out, codes and
    scales exactly those of quantizeInt8/Int4 on the widened weights (the
    quantiser is the oracle's here; the library's GPU quantiser is bit-checked
    against it in tests/test_gpu_quant.py)."""
    from qgmoe.quantize_layer import quantize_layer
    m = O.make_moe(H=128, E=4, k=2, I=64, Is=Is, bits=16, seed=21)
    pre = "model.layers.2.mlp."
    src, dst = str(tmp_path / "raw.safetensors"), str(tmp_path / "q.safetensors")
    args = dict(router=m.router, gate_up=m.q["gate_up"], down=m.q["down"])
    if Is:
        args.update(shared_gate=m.shared_gate, shared_gate_proj=m.q["sh_gate"],
                    shared_up_proj=m.q["sh_up"], shared_down_proj=m.q["sh_down"])
    ck.save_layer_raw(src, pre, **args)

    def oracle_quantize(w, b):
        q, s = O.quantize(np.ascontiguousarray(w, np.float32), b)
        return q, O.f16_bits(s)

    qj = str(tmp_path / "quant.json")
    quantize_layer(src, dst, pre, bits, quant_json=qj, quantize=oracle_quantize)
    with qgmoe.LayerFile(dst) as f:
        d = f.layer_desc(pre, 2)
        assert d.bits == bits and d.n_shared_mlp == Is and d.scale_dtype == qgmoe.SCALE_F16
        q_gu, s_gu = oracle_quantize(O.bf16_widen(m.q["gate_up"]).reshape(-1, 128), bits)
        assert _bytes(d.gate_up_q, q_gu) and _bytes(d.gate_up_scale, s_gu)
        q_dn, s_dn = oracle_quantize(O.bf16_widen(m.q["down"]).reshape(4 * 128, -1), bits)
        assert _bytes(d.down_q, q_dn) and _bytes(d.down_scale, s_dn)
        assert _bytes(d.router, m.router)
        if Is:
            q_sd, s_sd = oracle_quantize(O.bf16_widen(m.q["sh_down"]), bits)
            assert _bytes(d.shared_down_q, q_sd) and _bytes(d.shared_down_scale, s_sd)
    assert json.load(open(qj))["bits"] == bits


@pytest.mark.parametrize("sdt", ["f16", "f32"])
def test_mixed_layer_desc(tmp_path, sdt):
    """A layer whose groups have their own formats (bf16 routed experts, an
    int8 shared expert, an int8 router) gives a descriptor with each group's
    format and pointers into the mapping at the written bytes, and the
    reference's quant.json lists the quantised linears; a layer whose
    quantised groups mix F16 and F32 scales is rejected."""
    m = O.make_moe(H=128, E=4, k=2, I=64, Is=64, bits=16, seed=31, shared_bits=8, router_bits=8)
    sc = (lambda s16, s32: s16) if sdt == "f16" else (lambda s16, s32: s32)
    s32 = {k: m.s[k] for k in ("sh_gate", "sh_up", "sh_down")}
    s32["router"] = m.s32["router"]
    p = str(tmp_path / "mixed.safetensors")
    qj = str(tmp_path / "quant.json")
    ck.save_layer_groups(
        p, "L.", router=(m.q["router"], sc(m.s16["router"], s32["router"])),
        experts=(m.q["gate_up"], m.q["down"]),
        shared=tuple((m.q[k], sc(m.s16[k], s32[k])) for k in ("sh_gate", "sh_up", "sh_down")),
        shared_gate=m.shared_gate, quant_json=qj)
    with qgmoe.LayerFile(p) as f:
        d = f.layer_desc("L.", top_k=2)
        assert (d.n_embed, d.n_experts, d.n_moe_mlp, d.n_shared_mlp) == (128, 4, 64, 64)
        assert (d.bits, d.shared_bits, d.router_bits) == (16, 8, 8)
        assert d.scale_dtype == (qgmoe.SCALE_F16 if sdt == "f16" else qgmoe.SCALE_F32)
        assert not d.router
        _, _, rq, nb = f.tensor("L.gate.qweight")
        assert d.router_q == rq and nb == m.q["router"].nbytes
        assert bytes(C.string_at(d.router_q, nb)) == m.q["router"].tobytes()
        assert bytes(C.string_at(d.gate_up_q, m.q["gate_up"].nbytes)) == m.q["gate_up"].tobytes()
        assert bytes(C.string_at(d.shared_up_q, m.q["sh_up"].nbytes)) == m.q["sh_up"].tobytes()
    with open(qj) as fh:
        man = json.load(fh)
    assert man == {"bits": 8, "quantized": ["L.gate.weight"] + [
        f"L.shared_expert.{n}_proj.weight" for n in ("gate", "up", "down")]}
    # mixed scale dtypes across groups
    bad = str(tmp_path / "bad.safetensors")
    ck.save_layer_groups(
        bad, "L.", router=(m.q["router"], m.s16["router"]), experts=(m.q["gate_up"], m.q["down"]),
        shared=tuple((m.q[k], s32[k]) for k in ("sh_gate", "sh_up", "sh_down")),
        shared_gate=m.shared_gate)
    with qgmoe.LayerFile(bad) as f:
        with pytest.raises(qgmoe.QgmoeError):
            f.layer_desc("L.", top_k=2)
