"""The decode path (qg_decode.cu): batches of up to 8 tokens in four kernels
-- router logits in the reference's serial order; routing of the batch;
gate_up + SwiGLU; down + rank-order combine -- taken by AUTO whenever the
batch fits.

Its row arithmetic and its combine are the CUDA-core path's, so the two give
bit-identical outputs and routing; both meet the oracle bar (routing and
weights bit-exact, outputs within 1e-3, 2e-3 for int4)."""
import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import CONFIGS, check_outputs, check_routing, device_case, host_case, make_gpu_moe

pytestmark = pytest.mark.gpu


def both_paths(m, x, mode):
    g = make_gpu_moe(m, mode)
    out, idx, w = g.forward_batch(x, return_routing=True)
    launches = g.last_launch_count()
    g.set_path(qgmoe.PATH_CUDA_CORE)
    ref_out, ref_idx, ref_w = g.forward_batch(x, return_routing=True)
    return (out, idx, w, launches), (ref_out, ref_idx, ref_w)


@pytest.mark.parametrize("bits", [32, 16, 8, 4])
@pytest.mark.parametrize("Is", [0, 128])
@pytest.mark.parametrize("mode", [O.ROUTER_TOPK, O.ROUTER_PREFIX])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_decode_path_equals_cuda_core_path_and_oracle(bits, Is, mode, T):
    m = host_case(H=256, E=16, k=4, I=128, Is=Is, bits=bits, seed=400 + T + Is)
    x = O.randn(400, T, (T, 256))
    (out, idx, w, launches), (r_out, r_idx, r_w) = both_paths(m, x, mode)
    assert launches == 4
    assert np.array_equal(idx, r_idx) and np.array_equal(w, r_w)
    assert np.array_equal(out, r_out)
    ref, ridx, rw, _, probs = O.moe_forward(m, x, mode, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, 32 if bits == 16 else bits)


@pytest.mark.parametrize("name,Ts", [("c1", (1, 2, 8)), ("c2", (1, 4))])
def test_decode_path_at_benchmark_shapes(name, Ts):
    c = CONFIGS[name]
    m, dev = device_case(**c)
    g = make_gpu_moe(m, O.ROUTER_TOPK, dev)
    for T in Ts:
        x = O.randn(c["seed"], 100 + T, (T, c["H"]))
        out, idx, w = g.forward_batch(x, return_routing=True)
        assert g.last_launch_count() == 4
        ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
        assert not check_routing(idx, w, ridx, rw, probs)
        check_outputs(out, ref, c["bits"])


def test_decode_path_graph_replay_and_nan():
    """Repeated identical calls replay a captured graph of the four kernels;
    a NaN activation routes like the reference (experts 0..k-1, NaN out)."""
    m = host_case(H=256, E=16, k=4, I=128, Is=128, bits=8, seed=410)
    g = make_gpu_moe(m, O.ROUTER_TOPK)
    x = O.randn(410, 1, (5, 256))
    x[2, 7] = np.nan
    first = g.forward_batch(x)
    for _ in range(3):
        assert np.array_equal(g.forward_batch(x), first, equal_nan=True)
    ref, ridx, *_ = O.moe_forward(m, x)
    check_outputs(first, ref, 8)
    assert np.all(np.isnan(first[2])) and not np.isnan(first[[0, 1, 3, 4]]).any()


def test_decode_path_falls_back_when_the_batch_does_not_fit():
    """Config 2 at 8 tokens: the h rows of 64 (token, rank) pairs exceed the
    down kernel's shared memory, so the general path runs (more launches)."""
    c = CONFIGS["c2"]
    m, dev = device_case(**c)
    g = make_gpu_moe(m, O.ROUTER_TOPK, dev)
    x = O.randn(c["seed"], 108, (8, c["H"]))
    out, idx, w = g.forward_batch(x, return_routing=True)
    assert g.last_launch_count() > 4
    ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, c["bits"])
