"""CPU tests of the C-ABI boundary: the library builds for sm_100a, loads,
exports every function include/qgmoe.h declares, and rejects bad arguments
before touching a device.  No compute runs here."""
import ctypes as C
import os
import re

import pytest

import qgmoe
from qgmoe.build import LIB, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "qgmoe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qg\w+)\s*\(", src)))


def test_library_builds_and_loads():
    path = build()
    assert path == LIB and os.path.exists(LIB)
    assert qgmoe.lib() is not None


def test_exports_every_declared_symbol():
    names = header_functions()
    assert len(names) >= 16
    L = C.CDLL(LIB)
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(qgmoe.SIGNATURES), set(names) ^ set(qgmoe.SIGNATURES)


def test_descriptor_layout_matches_the_c_struct(tmp_path):
    """The ctypes mirror of qgmoe_desc (qgmoe/__init__.py) has the C struct's
    size and field offsets, compiled from include/qgmoe.h with gcc."""
    import subprocess
    fields = [f for f, _ in qgmoe._Desc._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"qgmoe.h\"\n"
                   "int main(void) {\n  printf(\"%zu\\n\", sizeof(qgmoe_desc));\n" +
                   "".join(f'  printf("%zu\\n", offsetof(qgmoe_desc, {f}));\n' for f in fields) +
                   "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-I", os.path.join(REPO, "include"), str(src), "-o",
                    str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert got[0] == C.sizeof(qgmoe._Desc)
    assert got[1:] == [getattr(qgmoe._Desc, f).offset for f in fields]


def test_status_strings():
    assert qgmoe.status_text(0) == "ok"
    assert "invalid" in qgmoe.status_text(-1)
    assert qgmoe.status_text(12345) == "unknown status"


def test_create_rejects_bad_shapes_without_device():
    d = qgmoe._Desc()
    h = C.c_void_p()
    d.n_embed, d.n_experts, d.top_k, d.n_moe_mlp, d.bits = 30, 4, 2, 32, 32  # H % 32 != 0
    assert qgmoe.lib().qgmoe_create(C.byref(d), C.byref(h)) == -1
    assert "bad shape" in qgmoe.last_error()
    d.n_embed, d.top_k = 64, 5  # k > E
    assert qgmoe.lib().qgmoe_create(C.byref(d), C.byref(h)) == -1
    d.top_k, d.bits = 2, 6
    assert qgmoe.lib().qgmoe_create(C.byref(d), C.byref(h)) == -1
    assert "bits" in qgmoe.last_error()
    assert qgmoe.lib().qgmoe_create(None, C.byref(h)) == -1


def test_quantlinear_rejects_bad_arguments_without_device():
    h = C.c_void_p()
    assert qgmoe.lib().qgql_create(5, 4, 64, None, None, 0, 0, 0, C.byref(h)) == -1
    assert qgmoe.lib().qgql_create(8, 4, 48, None, None, 0, 0, 0, C.byref(h)) == -1
    assert qgmoe.lib().qgql_quantize_device(3, 4, 64, None, None, None, None, None) == -1


def test_null_handles_are_errors_not_crashes():
    L = qgmoe.lib()
    assert L.qgmoe_forward(None, None, 1, None, None, None) == -1
    assert L.qgmoe_destroy(None) == 0
    assert L.qgql_forward(None, None, 1, None) == -1
    assert L.qgmoe_last_launch_count(None) == 0


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES", None) == "", reason="n/a")
def test_device_ok_is_false_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert qgmoe.lib().qgmoe_device_ok(0) == 0


def test_plain_c_host_uses_the_abi(tmp_path):
    """include/qgmoe.h compiles as C99 (what cgo sees) and a C host can map a
    layer file and build its descriptor through the library; create() then
    answers without a GPU (no sm_100 device) or with one."""
    import shutil
    import subprocess

    import numpy as np
    import qg_oracle as O
    from qgmoe import checkpoint as ck

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    build()
    exe = str(tmp_path / "abi_host")
    src = os.path.join(REPO, "tests", "c", "abi_host.c")
    libdir = os.path.dirname(LIB)
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-pedantic", "-I",
                    os.path.join(REPO, "include"), src, "-o", exe, "-L", libdir, "-lqgmoe",
                    "-Wl,-rpath," + libdir], check=True)
    m = O.make_moe(H=128, E=4, k=2, I=64, Is=0, bits=4, seed=3)
    path = str(tmp_path / "l.safetensors")
    ck.save_layer(path, "model.layers.7.mlp.", router=m.router, gate_up_q=m.q["gate_up"],
                  gate_up_scale=m.s16["gate_up"], down_q=m.q["down"],
                  down_scale=m.s16["down"], bits=4)
    out = subprocess.run([exe, path, "model.layers.7.mlp.", "2"], capture_output=True, text=True,
                         check=True).stdout
    assert "router rc=0 dtype=0 rank=2 shape=4,128 bytes=2048" in out
    assert "desc rc=0 H=128 E=4 k=2 I=64 Is=0 bits=4 scale=0" in out
    rc = int(out.split("create rc=")[1].split()[0])
    assert rc in (0, -7), out  # OK on a B200, QGMOE_ERR_NO_DEVICE without one
