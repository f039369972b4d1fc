"""Mixed-format MoE layers, as the reference holds and loads them.

moeMLP (model/moe.go:10-25) keeps one format per weight group: the router is
float32 or bf16 rows (linear) or a quantLinear (routerQuant, installed by
model/load.go:651-652); the routed experts are float32 or raw bf16 stacks;
the shared expert's projections are float32, bf16 or quantLinears of their
own (model/load.go:653-658).  cmd/qwen-quant quantises exactly the
shared-expert projections of an MoE model and writes f32 scales
(cmd/qwen-quant/main.go:61-65, 209).  Every combination below runs against
the oracle with the same per-group formats: routing exact, outputs within
1e-3 (2e-3 when a group is int4), created from arrays and from layer files.
"""
import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import check_outputs, check_routing, make_gpu_moe
from qgmoe import checkpoint as ck

pytestmark = pytest.mark.gpu

# (label, routed bits, shared bits, router bits, shared width)
CASES = [
    ("bf16-experts_int8-shared", 16, 8, 32, 256),
    ("bf16-experts_int4-shared_bf16-router", 16, 4, 16, 128),
    ("f32-experts_int8-shared_int8-router", 32, 8, 8, 128),
    ("int8-experts_int8-router", 8, 0, 8, 0),
    ("int4-experts_int4-router_int8-shared", 4, 8, 4, 128),
    ("int8-experts_bf16-shared", 8, 16, 32, 128),
    ("int8-experts_f32-shared_int8-router", 8, 32, 8, 128),
    ("int8-experts_int8-shared-96", 8, 8, 32, 96),
]


def tol_bits(bits, sb):
    return 4 if 4 in (bits, sb) else 8


def compare(m, x, mode, g):
    out, idx, w = g.forward_batch(x, return_routing=True)
    ref, ridx, rw, _, probs = O.moe_forward(m, x, mode, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, tol_bits(m.bits, m.shared_bits or m.bits))
    return out


@pytest.mark.parametrize("T", [1, 5, 40, 300])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_mixed_layer_matches_oracle(case, T):
    _, bits, sb, rb, Is = case
    m = O.make_moe(H=256, E=8, k=2, I=128, Is=Is, bits=bits, seed=200 + T, shared_bits=sb,
                   router_bits=rb)
    x = O.randn(200, T, (T, 256))
    compare(m, x, O.ROUTER_TOPK, make_gpu_moe(m, O.ROUTER_TOPK))


@pytest.mark.parametrize("path", [qgmoe.PATH_CUDA_CORE, qgmoe.PATH_TENSOR])
def test_mixed_layer_on_each_path(path):
    """int8 experts with a bf16 shared expert and an int8 router, forced onto
    each expert path: on CUDA cores the two formats take separate GEMV
    launches, on the tensor path the shared expert runs on the GEMV beside
    the tensor-core experts."""
    m = O.make_moe(H=256, E=8, k=2, I=128, Is=128, bits=8, seed=230, shared_bits=16,
                   router_bits=8)
    x = O.randn(230, 1, (24, 256))
    g = make_gpu_moe(m, O.ROUTER_PREFIX)
    g.set_path(path)
    compare(m, x, O.ROUTER_PREFIX, g)


def test_f32_scales_as_qwen_quant_writes_them():
    """cmd/qwen-quant writes f32 scales and the loader keeps them: the
    quantised router is dequantised with them unrounded (routing stays
    exact); the shared expert stores them as fp16."""
    m = O.make_moe(H=256, E=16, k=4, I=128, Is=128, bits=16, seed=240, shared_bits=8,
                   router_bits=8, router_scale_f32=True)
    x = O.randn(240, 1, (33, 256))
    compare(m, x, O.ROUTER_TOPK, make_gpu_moe(m, O.ROUTER_TOPK, scale_f32=True))


def _groups(m):
    """The layer's groups in save_layer_groups form."""
    def w(key, b):
        if b == 32:
            return np.ascontiguousarray(getattr(m, key), np.float32)
        if b == 16:
            return m.q[key]
        return (m.q[key], m.s16[key])
    sb = m.shared_bits or m.bits
    router = m.router if m.router_bits == 32 else (
        m.q["router"] if m.router_bits == 16 else (m.q["router"], m.s16["router"]))
    shared = None
    if m.Is:
        shared = (w("sh_gate", sb), w("sh_up", sb), w("sh_down", sb))
    return dict(router=router, experts=(w("gate_up", m.bits), w("down", m.bits)),
                shared=shared, shared_gate=m.shared_gate)


@pytest.mark.parametrize("case", [CASES[0], CASES[3], CASES[4]], ids=lambda c: c[0])
def test_mixed_layer_from_file_equals_from_arrays(case, tmp_path):
    _, bits, sb, rb, Is = case
    m = O.make_moe(H=256, E=8, k=2, I=128, Is=Is, bits=bits, seed=250, shared_bits=sb,
                   router_bits=rb)
    p = str(tmp_path / "layer.safetensors")
    ck.save_layer_groups(p, "model.layers.0.mlp.", **_groups(m))
    x = O.randn(250, 1, (40, 256))
    a = make_gpu_moe(m, O.ROUTER_TOPK).forward_batch(x)
    g = qgmoe.MoeMLP.from_file(p, "model.layers.0.mlp.", top_k=2)
    assert np.array_equal(g.forward_batch(x), a)
    compare(m, x, O.ROUTER_TOPK, g)
