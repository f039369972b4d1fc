"""Expert-parallel data flow on CPU: two gloo ranks run qgmoe.ep.run_exchange
(the same exchange code the GPU layer uses) with a CPU model of the three
kernels -- dispatch sorted by (owner rank, local expert), experts applied by
the receiving rank to rows regrouped by local expert, rank-ordered combine --
and must reproduce the single-process oracle forward of their token shard."""
import os
import socket

import numpy as np
import pytest

W = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, port, result_dir, placement="rr"):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(repo, "qwen-go_b200"), os.path.join(repo, "oracle")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import qg_oracle as O
    from qgmoe.ep import dispatch_key, owned_experts, round_robin_slots, run_exchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W)
    H, E, k, I, bits, T_all = 64, 8, 3, 32, 8, 26
    G = E // W
    place = (round_robin_slots(E, W) if placement == "rr"
             else np.array([5, 2, 7, 0, 4, 1, 6, 3], np.int32))  # any permutation
    mine = owned_experts(place, rank, W)
    m = O.make_moe(H, E, k, I, 0, bits, seed=77)
    x_all = O.randn(77, 100, (T_all, H))
    lo, hi = rank * T_all // W, (rank + 1) * T_all // W
    x = x_all[lo:hi]
    T = hi - lo
    ref, idx, w, _, _ = O.moe_forward(m, x)

    state = {}

    def dispatch():
        keys = dispatch_key(idx.reshape(-1), E, W, place)
        order = np.argsort(keys, kind="stable")       # pair ids in slot order
        slot = np.empty_like(order)
        slot[order] = np.arange(order.size)
        state["slot"] = slot
        rows = torch.from_numpy(x[order // k].copy())
        counts = np.bincount(keys, minlength=E).reshape(W, G).astype(np.int32)
        return rows, counts

    def expert_rows(e, rows):
        gu = O.linear_rows(bits, None, m.q["gate_up"][e * 2 * I:(e + 1) * 2 * I],
                           m.s["gate_up"][e * 2 * I:(e + 1) * 2 * I], rows, 2 * I)
        g = gu[:, :I]
        g = (g / (np.float32(1) + np.exp(-g.astype(np.float64)).astype(np.float32))).astype(np.float32)
        h = (g * gu[:, I:]).astype(np.float32)
        return O.linear_rows(bits, None, m.q["down"][e * H:(e + 1) * H],
                             m.s["down"][e * H:(e + 1) * H], h, H)

    def experts(recv_rows, recv_counts):
        rows = recv_rows.numpy()
        out = np.zeros_like(rows)
        off = 0
        for src in range(W):
            for j in range(G):
                n = int(recv_counts[src, j])
                if n:
                    e = mine[j]                 # the global id of local expert j
                    out[off:off + n] = expert_rows(e, rows[off:off + n])
                off += n
        return torch.from_numpy(out)

    def combine(back_rows):
        back = back_rows.numpy()
        out = np.zeros((T, H), np.float32)
        for t in range(T):
            for r in range(k):
                out[t] = (out[t] + (w[t, r] * back[state["slot"][t * k + r]]).astype(np.float32)
                          ).astype(np.float32)
        return out

    out = run_exchange(dispatch, experts, combine)
    np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.stack([out, ref]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("placement", ["rr", "permuted"])
def test_two_rank_exchange_reproduces_oracle(tmp_path, placement):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(port, str(tmp_path), placement), nprocs=W, join=True)
    for r in range(W):
        out, ref = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(out, ref, rtol=1e-6, atol=1e-7)


def test_dispatch_key_groups_by_owner_then_local_index():
    from qgmoe.ep import dispatch_key
    E, W = 16, 4
    keys = [dispatch_key(e, E, W) for e in range(E)]
    assert sorted(keys) == list(range(E))
    for e in range(E):
        assert keys[e] // (E // W) == e % W and keys[e] % (E // W) == e // W


def test_balanced_placement_is_a_permutation_and_evens_the_load():
    from qgmoe.ep import balanced_slots, owned_experts, round_robin_slots
    E, W = 128, 8
    load = (np.arange(E) + 1.0) ** -0.7 * 4096  # skewed expert loads whose hottest
    assert load.max() < 0.75 * load.sum() / W   # expert fits well inside one rank
    slot = balanced_slots(load, W)
    assert sorted(slot.tolist()) == list(range(E))
    G = E // W
    per_rank = np.zeros(W)
    for r in range(W):
        mine = owned_experts(slot, r, W)
        assert len(mine) == G and all(slot[e] // G == r for e in mine)
        assert all(slot[e] % G == j for j, e in enumerate(mine))
        per_rank[r] = load[mine].sum()
    rr = round_robin_slots(E, W)
    rr_rank = np.array([load[[e for e in range(E) if rr[e] // G == r]].sum() for r in range(W)])
    # lower bound with E/W experts per rank: the mean, and the hottest expert
    # together with the E/W - 1 lightest others
    lb = max(load.sum() / W, load.max() + np.sort(load)[:G - 1].sum())
    assert per_rank.max() <= 1.01 * lb
    assert rr_rank.max() > 1.2 * per_rank.max()


# --------------------------------------------------------------------------
# The peer-memory exchange's index arithmetic (qwen-go_b200/csrc/qg_peer.cu),
# restated: where k_px_send stores each row in its owner's grouped buffer,
# and the (source, send position) k_px_tables maps each received row back to.
# --------------------------------------------------------------------------


def _px_send_positions(cnt, me):
    """k_px_send: position at owner d of source `me`'s rows for d's local
    expert g -- the rows of d's experts before g (all sources), then those of
    the sources before `me` in d's order d, d+1, ..., d-1 (mod W)."""
    W, _, G = cnt.shape
    pos = np.zeros((W, G), np.int64)
    for d in range(W):
        for g in range(G):
            p = int(cnt[:, d, :g].sum())
            s = d
            while s != me:
                p += int(cnt[s, d, g])
                s = (s + 1) % W
            pos[d, g] = p
    return pos


def _px_out_map(cnt, me):
    """k_px_tables at owner `me`: for each grouped row, (source, position of
    the row in that source's send order)."""
    W, _, G = cnt.shape
    gbase = np.concatenate([[0], np.cumsum(cnt[:, me, :].sum(axis=0))])
    seg = np.zeros((G, W), np.int64)
    dst0 = np.zeros((G, W), np.int64)
    for g in range(G):
        for j in range(W):
            s = (me + j) % W
            r = int(gbase[g])
            s2 = me
            while s2 != s:
                r += int(cnt[s2, me, g])
                s2 = (s2 + 1) % W
            seg[g, j] = r
            dst0[g, j] = int(cnt[s, :me, :].sum()) + int(cnt[s, me, :g].sum())
    out = []
    for r in range(int(gbase[-1])):
        g = int(np.searchsorted(gbase, r, side="right") - 1)
        j = W - 1
        while j > 0 and seg[g, j] > r:
            j -= 1
        s = (me + j) % W
        out.append((s, int(dst0[g, j] + r - seg[g, j])))
    return out


@pytest.mark.parametrize("W_", [2, 3, 4, 8])
def test_peer_exchange_positions_are_a_bijection(W_):
    """Every source row lands in exactly one slot of its owner's grouped
    buffer, the rows of one local expert are contiguous, and the owner's map
    sends each output back to the source position it came from -- for random
    (and some empty) count matrices at 2-8 ranks."""
    rng = np.random.default_rng(W_)
    G = 5
    for trial in range(6):
        cnt = rng.integers(0, 7, size=(W_, W_, G))
        if trial == 1:
            cnt[:, :, 2] = 0          # an expert nobody routes to
        if trial == 2:
            cnt[1 % W_] = 0           # a source with no tokens
        for d in range(W_):
            owner_rows = {}
            for me in range(W_):
                pos = _px_send_positions(cnt, me)
                # source me's send order: keys (d, g) d-major, rows in order
                p = 0
                for dd in range(W_):
                    for g in range(G):
                        for jj in range(int(cnt[me, dd, g])):
                            if dd == d:
                                r = int(pos[d, g]) + jj
                                assert r not in owner_rows
                                owner_rows[r] = (me, p, g)
                            p += 1
            R = int(cnt[:, d, :].sum())
            assert sorted(owner_rows) == list(range(R))
            gbase = np.concatenate([[0], np.cumsum(cnt[:, d, :].sum(axis=0))])
            for r, (_, _, g) in owner_rows.items():
                assert gbase[g] <= r < gbase[g + 1]
            back = _px_out_map(cnt, d)
            for r in range(R):
                assert back[r] == owner_rows[r][:2], (W_, trial, d, r)


@pytest.mark.parametrize("W_", [2, 3, 8])
@pytest.mark.parametrize("nw", [8, 13, 64, 4736])
def test_peer_send_warps_cover_every_row_once(W_, nw):
    """k_px_send's warp split: warp wg sends to rank (me + wg % W) % W the
    rows wg / W, wg / W + nwd, ... of that destination, nwd the number of
    warps with that slot; together the warps cover each row exactly once."""
    rng = np.random.default_rng(nw + W_)
    if nw < W_:
        return  # the launcher gives at least one warp per destination
    rows = rng.integers(0, 50, size=W_)
    for me in range(W_):
        seen = [np.zeros(n, np.int64) for n in rows]
        for wg in range(nw):
            j = wg % W_
            d = (me + j) % W_
            wi, nwd = wg // W_, (nw - j + W_ - 1) // W_
            for p in range(wi, int(rows[d]), nwd):
                seen[d][p] += 1
        assert all(np.all(s == 1) for s in seen)
