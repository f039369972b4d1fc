"""The decode kernel (qg_decode.cu): batches of up to 8 tokens in ONE
persistent launch -- serial-order router logits on one warp per CTA while
the other warps stream the experts of an approximate top-k, then the exact
routing, the experts it picked that the approximation missed, and the
rank-order combine -- taken by AUTO whenever the batch fits.

Routing and weights are the reference's bit for bit (identical to the
CUDA-core path's); int8/int4 expert products run on the tensor cores with
fp16 operands (the prefill tensor path's arithmetic), f32/bf16 experts keep
the CUDA-core arithmetic and equal that path bit for bit.  Outputs meet the
oracle bar: within 1e-3, 2e-3 for int4.  Speculation on or off gives the
same bits."""
import re

import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import CONFIGS, check_outputs, check_routing, device_case, host_case, make_gpu_moe

pytestmark = pytest.mark.gpu


def run(m, x, mode, speculate=True):
    g = make_gpu_moe(m, mode)
    g.set_decode_speculation(speculate)
    out, idx, w = g.forward_batch(x, return_routing=True)
    return g, out, idx, w, g.last_launch_count()


@pytest.mark.parametrize("bits", [32, 16, 8, 4])
@pytest.mark.parametrize("Is", [0, 256])
@pytest.mark.parametrize("mode", [O.ROUTER_TOPK, O.ROUTER_PREFIX])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_decode_kernel_matches_oracle_and_cuda_core_routing(bits, Is, mode, T):
    m = host_case(H=256, E=16, k=4, I=256, Is=Is, bits=bits, seed=400 + T + Is)
    x = O.randn(400, T, (T, 256))
    g, out, idx, w, launches = run(m, x, mode)
    assert launches == 1
    g.set_path(qgmoe.PATH_CUDA_CORE)
    r_out, r_idx, r_w = g.forward_batch(x, return_routing=True)
    assert np.array_equal(idx, r_idx) and np.array_equal(w, r_w)
    if bits >= 16:
        assert np.array_equal(out, r_out)
    ref, ridx, rw, _, probs = O.moe_forward(m, x, mode, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, 32 if bits == 16 else bits)


@pytest.mark.parametrize("bits", [32, 8, 4])
@pytest.mark.parametrize("T", [1, 5])
def test_decode_kernel_without_speculation(bits, T):
    """Every expert computed after the exact routing (the path a missed
    candidate takes): the same bits as with speculation."""
    m = host_case(H=512, E=32, k=6, I=256, Is=256, bits=bits, seed=420 + T)
    x = O.randn(420, T, (T, 512))
    _, out, idx, w, launches = run(m, x, O.ROUTER_TOPK, False)
    assert launches == 1
    _, s_out, s_idx, s_w, _ = run(m, x, O.ROUTER_TOPK, True)
    assert np.array_equal(idx, s_idx) and np.array_equal(w, s_w)
    assert np.array_equal(out, s_out)
    ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, bits)


@pytest.mark.parametrize("name,Ts", [("c1", (1, 2, 8)), ("c2", (1, 4, 8))])
def test_decode_kernel_at_benchmark_shapes(name, Ts):
    c = CONFIGS[name]
    m, dev = device_case(**c)
    g = make_gpu_moe(m, O.ROUTER_TOPK, dev)
    for T in Ts:
        x = O.randn(c["seed"], 100 + T, (T, c["H"]))
        out, idx, w = g.forward_batch(x, return_routing=True)
        assert g.last_launch_count() == 1
        ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
        assert not check_routing(idx, w, ridx, rw, probs)
        check_outputs(out, ref, c["bits"])


def test_decode_kernel_graph_replay_and_nan():
    """Repeated identical calls replay a captured graph of the kernel (its
    barrier counter keeps counting across replays); a NaN activation routes
    like the reference (experts 0..k-1, NaN out)."""
    m = host_case(H=256, E=16, k=4, I=256, Is=256, bits=8, seed=410)
    g = make_gpu_moe(m, O.ROUTER_TOPK)
    x = O.randn(410, 1, (5, 256))
    x[2, 7] = np.nan
    first = g.forward_batch(x)
    for _ in range(4):
        assert np.array_equal(g.forward_batch(x), first, equal_nan=True)
    ref, ridx, *_ = O.moe_forward(m, x)
    check_outputs(first, ref, 8)
    assert np.all(np.isnan(first[2])) and not np.isnan(first[[0, 1, 3, 4]]).any()


def test_decode_kernel_alternating_batches():
    """Different batch sizes in turn on one handle: each launch's flags are
    told apart by its barrier epoch, none is reset in between."""
    m = host_case(H=256, E=16, k=4, I=256, Is=0, bits=4, seed=430)
    g = make_gpu_moe(m, O.ROUTER_TOPK)
    for T in (1, 7, 2, 8, 1, 3):
        x = O.randn(430, T, (T, 256))
        out, idx, w = g.forward_batch(x, return_routing=True)
        assert g.last_launch_count() == 1
        ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
        assert not check_routing(idx, w, ridx, rw, probs)
        check_outputs(out, ref, 4)


def test_general_path_beyond_eight_tokens():
    """Nine tokens: more than the decode kernel takes, so the general path
    runs (several launches) with the same routing bar."""
    c = CONFIGS["c2"]
    m, dev = device_case(**c)
    g = make_gpu_moe(m, O.ROUTER_TOPK, dev)
    x = O.randn(c["seed"], 109, (9, c["H"]))
    out, idx, w = g.forward_batch(x, return_routing=True)
    assert g.last_launch_count() > 1
    ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
    assert not check_routing(idx, w, ridx, rw, probs)
    check_outputs(out, ref, c["bits"])


def test_decode_kernel_wait_limit_runs_out_and_recovers():
    """A wait that runs out: with a 1 us limit the kernel's grid barriers and
    routing-flag waits give up, the call reports QGMOE_ERR_TIMEOUT (device
    flag 8) instead of hanging, and the next call with the default limit is correct
    again (the barrier count and flags were restarted)."""
    m = host_case(H=256, E=16, k=4, I=256, Is=0, bits=8, seed=440)
    g = make_gpu_moe(m, O.ROUTER_TOPK)
    g.set_graphs(False)
    x = O.randn(440, 1, (2, 256))
    good = g.forward_batch(x)
    g.set_wait_limit(1)
    with pytest.raises(qgmoe.QgmoeError) as ei:
        for _ in range(3):  # a fast GPU might finish inside the limit once
            g.forward_batch(x)
    assert ei.value.status == qgmoe.ERR_TIMEOUT
    assert int(re.search(r"device flag 0x([0-9a-f]+)", str(ei.value)).group(1), 16) & 8
    g.set_wait_limit(0)
    for _ in range(2):
        assert np.array_equal(g.forward_batch(x), good)
    ref, *_ = O.moe_forward(m, x)
    check_outputs(good, ref, 8)


def test_decode_kernel_many_batches_at_config1():
    """Twelve different 8-token batches on one handle at config 1 (shared
    expert, E=16): every CTA's combine reads routing entries that other
    threads of the CTA stage, so each batch's output must match the oracle
    whatever the timing (a missing barrier there once let a combine read
    the previous launch's slots)."""
    c = CONFIGS["c1"]
    m, dev = device_case(**c)
    g = make_gpu_moe(m, O.ROUTER_TOPK, dev)
    for i in range(12):
        x = O.randn(c["seed"] + i, 200, (8, c["H"]))
        out, idx, w = g.forward_batch(x, return_routing=True)
        ref, ridx, rw, _, probs = O.moe_forward(m, x, want_probs=True)
        assert not check_routing(idx, w, ridx, rw, probs)
        check_outputs(out, ref, c["bits"])
