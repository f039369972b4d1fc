"""The allocation-free router entry point (qgmoe_route_static).

It exists for callers that cannot call cudaMalloc (a host runtime that owns
all device memory, a stream-capture region, a fixed-budget serving loop), so
its scratch lives in a static device array instead.  Its routing must match
the oracle's and what the regular entry point (qgmoe_forward_device with
sel_idx / sel_w) returns for the same activations and router weights, on two
calls in a row: the array keeps the previous call's contents, so the second
call checks that the counters are cleared.  Batches of up to 32 tokens take
the fused top-k + scatter CTA, larger ones the separate kernels.  This file
is named to be collected last; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import check_routing, host_case, make_gpu_moe

pytestmark = pytest.mark.gpu


def _route_static(x, router, T, H, E, k, mode, idx, w, flags, stream):
    return qgmoe.lib().qgmoe_route_static(
        x.data_ptr(), router.data_ptr(), T, H, E, k, mode, idx.data_ptr(), w.data_ptr(),
        flags.data_ptr() if flags is not None else None, stream.cuda_stream)


@pytest.mark.parametrize("T", [1, 7, 32, 100, 300])
@pytest.mark.parametrize("mode", [O.ROUTER_TOPK, O.ROUTER_PREFIX])
def test_route_static_matches_oracle_and_forward_twice(mode, T):
    import torch
    H, E, k, I = 512, 64, 6, 64
    m = host_case(H=H, E=E, k=k, I=I, Is=0, bits=8, seed=90)
    handle = make_gpu_moe(m, mode)
    stream = torch.cuda.Stream()
    xh = O.randn(90, T, (T, H))
    if T >= 7:
        xh[5, 17] = np.nan  # routes to experts 0..k-1 with NaN weights, as the reference
    x = torch.from_numpy(xh).cuda()
    router = torch.from_numpy(m.router).cuda()
    out = torch.empty_like(x)
    ref_idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    ref_w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    handle.forward_device(x, out, sel_idx=ref_idx, sel_w=ref_w, stream=stream)
    handle.sync(stream)
    _o, oidx, ow, _sg, probs = O.moe_forward(m, xh, mode, want_probs=True)
    flags = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for _ in range(2):
        idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, k), -1.0, dtype=torch.float32, device="cuda")
        rc = _route_static(x, router, T, H, E, k, mode, idx, w, flags, stream)
        assert rc == 0, qgmoe.last_error()
        stream.synchronize()
        assert int(flags.item()) == 0
        assert torch.equal(idx, ref_idx)
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-5, atol=1e-7)
        assert not check_routing(idx.cpu().numpy(), w.cpu().numpy(), oidx, ow, probs,
                                 f"static T={T}")


def test_route_static_without_flags_word():
    import torch
    H, E, k, T = 256, 16, 4, 40
    m = host_case(H=H, E=E, k=k, I=64, Is=0, bits=8, seed=91)
    stream = torch.cuda.Stream()
    xh = O.randn(91, 1, (T, H))
    x = torch.from_numpy(xh).cuda()
    router = torch.from_numpy(m.router).cuda()
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    assert _route_static(x, router, T, H, E, k, 0, idx, w, None, stream) == 0
    stream.synchronize()
    _o, oidx, ow, _sg, probs = O.moe_forward(m, xh, 0, want_probs=True)
    assert not check_routing(idx.cpu().numpy(), w.cpu().numpy(), oidx, ow, probs)


def test_route_static_rejects_sizes_beyond_the_array():
    import torch
    H, E, k, T = 2048, 1024, 8, 4096
    x = torch.zeros((1, H), device="cuda")
    router = torch.zeros((E, H), device="cuda")
    idx = torch.zeros((1, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((1, k), device="cuda")
    rc = qgmoe.lib().qgmoe_route_static(x.data_ptr(), router.data_ptr(), T, H, E, k, 0,
                                        idx.data_ptr(), w.data_ptr(), None, None)
    assert rc == -1
    assert "scratch" in qgmoe.last_error()
