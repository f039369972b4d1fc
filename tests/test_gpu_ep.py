"""Expert-parallel forward on 2 GPUs: each rank owns half the experts and a
token shard; its output must match the single-GPU layer on the same tokens
(same kernels, so the tolerance is the north-star one) and the oracle on a
token sample.  Two exchanges: NCCL all-to-all driven by the host
(qgmoe.ep.ExpertParallelMoE) and the library's own peer-memory exchange
(qgmoe.ep.PeerExpertParallelMoE, uneven shards, repeated steps).  Skipped
when fewer than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

W = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, result_dir, mode="nccl"):
    import datetime
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(repo, "qwen-go_b200"), os.path.join(repo, "oracle"),
              os.path.join(repo, "tests")):
        sys.path.insert(0, p)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import qg_oracle as O
    import qgmoe
    from qgmoe.ep import ExpertParallelMoE, PeerExpertParallelMoE

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=W,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    H, E, k, I, bits, T_all = 256, 16, 4, 128, 8, 600
    m = O.make_moe(H, E, k, I, 0, bits, seed=88)
    x_all = O.randn(88, 100, (T_all, H))
    if mode != "peer":
        lo, hi = rank * T_all // W, (rank + 1) * T_all // W
    else:  # uneven shards: 220 / 380 tokens
        cut = 220
        lo, hi = (0, cut) if rank == 0 else (cut, T_all)
    G = E // W
    from qgmoe.ep import owned_experts, round_robin_slots
    slot = (np.random.default_rng(5).permutation(E).astype(np.int32) if mode == "peer_perm"
            else round_robin_slots(E, W).astype(np.int32))
    mine = owned_experts(slot, rank, W)              # experts owned here, local order
    gu_rows = np.concatenate([np.arange(e * 2 * I, (e + 1) * 2 * I) for e in mine])
    dn_rows = np.concatenate([np.arange(e * H, (e + 1) * H) for e in mine])
    layer = qgmoe.MoeMLP(n_embed=H, n_experts=E, top_k=k, n_moe_mlp=I, bits=bits, device=rank,
                         ep_world=W, ep_rank=rank, ep_slot=slot, router=m.router,
                         gate_up_q=np.ascontiguousarray(m.q["gate_up"][gu_rows]),
                         gate_up_scale=np.ascontiguousarray(m.s16["gate_up"][gu_rows]),
                         down_q=np.ascontiguousarray(m.q["down"][dn_rows]),
                         down_scale=np.ascontiguousarray(m.s16["down"][dn_rows]))
    ep = ExpertParallelMoE(layer) if mode == "nccl" else PeerExpertParallelMoE(layer, 400)
    peer = mode != "nccl"
    if mode == "peer_skip":
        _skip_step(rank, layer, ep, x_all[lo:hi], result_dir)
        dist.barrier()
        dist.destroy_process_group()
        return
    x = torch.from_numpy(x_all[lo:hi]).cuda()
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    for _ in range(3):  # later passes check the reused buffers (and exchange epochs)
        with torch.cuda.stream(s):
            out.zero_()
            ep.forward(x, out, s)
        s.synchronize()
    if peer:
        rc = qgmoe.lib().qgmoe_sync(layer.h, None)
        assert rc == 0, qgmoe.last_error()
    np.save(os.path.join(result_dir, f"ep{rank}.npy"), out.cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def _skip_step(rank, layer, ep, xs, result_dir):
    """Two good steps on both ranks, then rank 1 leaves out the third (it
    launches nothing: between steps, no kernel in flight) while rank 0 runs
    it with a 50 ms wait limit: rank 0's kernels give up on rank 1's flags
    and its sync reports the timeout."""
    import torch

    import qgmoe
    x = torch.from_numpy(xs).cuda()
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    for _ in range(2):
        ep.forward(x, out, s)
        s.synchronize()
    assert qgmoe.lib().qgmoe_sync(layer.h, None) == 0, qgmoe.last_error()
    torch.distributed.barrier()
    status = 0
    if rank == 0:
        layer.set_wait_limit(50000)
        ep.forward(x, out, s)
        s.synchronize()
        status = qgmoe.lib().qgmoe_sync(layer.h, None)
    with open(os.path.join(result_dir, f"skip{rank}.txt"), "w") as f:
        f.write(str(status))


def test_two_gpu_peer_exchange_times_out_when_a_rank_skips_a_step(tmp_path):
    import torch
    if torch.cuda.device_count() < W:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    import qgmoe
    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path), "peer_skip"), nprocs=W, join=True)
    assert int((tmp_path / "skip0.txt").read_text()) == qgmoe.ERR_TIMEOUT
    assert int((tmp_path / "skip1.txt").read_text()) == 0


@pytest.mark.parametrize("mode", ["nccl", "peer", "peer_perm"])
def test_two_gpu_expert_parallel_matches_single_gpu(tmp_path, mode):
    import torch
    if torch.cuda.device_count() < W:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    import qg_oracle as O
    import qgmoe
    from moe_cases import check_outputs, make_gpu_moe

    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path), mode), nprocs=W, join=True)
    H, E, k, I, bits, T_all = 256, 16, 4, 128, 8, 600
    m = O.make_moe(H, E, k, I, 0, bits, seed=88)
    x_all = O.randn(88, 100, (T_all, H))
    ep_out = np.concatenate([np.load(tmp_path / f"ep{r}.npy") for r in range(W)])
    single = make_gpu_moe(m, O.ROUTER_TOPK)
    single.set_path(qgmoe.PATH_TENSOR)
    ref = single.forward_batch(x_all)
    np.testing.assert_allclose(ep_out, ref, rtol=1e-3, atol=1e-3)
    sample = np.arange(0, T_all, 37)
    oref, *_ = O.moe_forward(m, x_all[sample])
    check_outputs(ep_out[sample], oref, bits)
