"""The plain-C host (tests/c/stack_host.c) on a GPU: the way a cgo shim
drives the library, with no Python between the host program and the C ABI.

check: a layer written to a safetensors file, created by the C host from the
mapping and run once through qgmoe_forward (host pointers), against the
oracle.  bench: a small stack of layers generated on the GPU, a prefill and a
few decode steps layer after layer (the residual kept on the host as
decodeLayers keeps it, model/model.go:473-526), finite all the way."""
import json
import subprocess

import numpy as np
import pytest

import qg_oracle as O
from moe_cases import check_outputs
from qgmoe import checkpoint as ck
from qgmoe.build import build_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,Is,T", [(8, 128, 5), (4, 0, 40)])
def test_c_host_forward_matches_oracle(tmp_path, bits, Is, T):
    exe = build_host("stack_host")
    m = O.make_moe(H=256, E=16, k=4, I=128, Is=Is, bits=bits, seed=300 + T)
    p = str(tmp_path / "layer.safetensors")
    sh = {}
    if Is:
        sh = dict(shared_gate=m.shared_gate, shared_gate_q=m.q["sh_gate"],
                  shared_gate_scale=m.s16["sh_gate"], shared_up_q=m.q["sh_up"],
                  shared_up_scale=m.s16["sh_up"], shared_down_q=m.q["sh_down"],
                  shared_down_scale=m.s16["sh_down"])
    ck.save_layer(p, "model.layers.0.mlp.", router=m.router, gate_up_q=m.q["gate_up"],
                  gate_up_scale=m.s16["gate_up"], down_q=m.q["down"],
                  down_scale=m.s16["down"], bits=bits, **sh)
    x = O.randn(300, T, (T, 256))
    xf, of, jf = (str(tmp_path / n) for n in ("x.f32", "out.f32", "idx.i32"))
    x.tofile(xf)
    r = subprocess.run([exe, "check", p, "model.layers.0.mlp.", "4", xf, str(T), of, jf],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    out = np.fromfile(of, np.float32).reshape(T, 256)
    idx = np.fromfile(jf, np.int32).reshape(T, 4)
    ref, ridx, _rw, _, _ = O.moe_forward(m, x)
    assert np.array_equal(idx, ridx)
    check_outputs(out, ref, bits)


def test_c_host_stack_prefill_and_decode():
    exe = build_host("stack_host")
    r = subprocess.run([exe, "bench", "4", "512", "16", "4", "256", "8", "64", "8", "7"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["finite"] and res["layers"] == 4
    assert res["prefill_moe_tokens_per_s"] > 0 and res["decode_moe_tokens_per_s"] > 0
