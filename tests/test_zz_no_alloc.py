"""The allocation-free router entry point (qgmoe_route_static).

It exists for callers that cannot call cudaMalloc (a host runtime that owns
all device memory, a stream-capture region, a fixed-budget serving loop), so
its scratch lives in a static device array instead.  Its routing must match
what the regular entry point (qgmoe_forward_device with sel_idx / sel_w)
returns for the same activations and router weights, on two calls in a row:
the array keeps the previous call's contents, so the second call checks that
the counters are cleared.  This file is named to be collected last; it also
passes on its own in a fresh process.
"""
import numpy as np
import pytest

import qg_oracle as O
import qgmoe
from moe_cases import host_case, make_gpu_moe

pytestmark = pytest.mark.gpu


def _route_static(x, router, T, H, E, k, mode, idx, w, stream):
    return qgmoe.lib().qgmoe_route_static(x.data_ptr(), router.data_ptr(), T, H, E, k, mode,
                                          idx.data_ptr(), w.data_ptr(), stream.cuda_stream)


@pytest.mark.parametrize("mode", [O.ROUTER_TOPK, O.ROUTER_PREFIX])
def test_route_static_matches_forward_routing_twice(mode):
    import torch
    H, E, k, I, T = 512, 64, 6, 64, 100
    m = host_case(H=H, E=E, k=k, I=I, Is=0, bits=8, seed=90)
    handle = make_gpu_moe(m, mode)
    stream = torch.cuda.Stream()
    x = torch.from_numpy(O.randn(90, 1, (T, H))).cuda()
    router = torch.from_numpy(m.router).cuda()
    out = torch.empty_like(x)
    ref_idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    ref_w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    handle.forward_device(x, out, sel_idx=ref_idx, sel_w=ref_w, stream=stream)
    handle.sync(stream)
    for _ in range(2):
        idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
        w = torch.full((T, k), -1.0, dtype=torch.float32, device="cuda")
        rc = _route_static(x, router, T, H, E, k, mode, idx, w, stream)
        assert rc == 0, qgmoe.last_error()
        stream.synchronize()
        assert torch.equal(idx, ref_idx)
        np.testing.assert_allclose(w.cpu().numpy(), ref_w.cpu().numpy(), rtol=1e-5, atol=1e-7)


def test_route_static_rejects_sizes_beyond_the_array():
    import torch
    H, E, k, T = 2048, 1024, 8, 4096
    x = torch.zeros((1, H), device="cuda")
    router = torch.zeros((E, H), device="cuda")
    idx = torch.zeros((1, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((1, k), device="cuda")
    rc = qgmoe.lib().qgmoe_route_static(x.data_ptr(), router.data_ptr(), T, H, E, k, 0,
                                        idx.data_ptr(), w.data_ptr(), None)
    assert rc == -1
    assert "scratch" in qgmoe.last_error()
