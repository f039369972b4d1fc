"""Expert-parallel MoE layer: one process per GPU, rows exchanged over
torch.distributed (NCCL on GPUs; gloo in the CPU tests of the data flow).

Experts are owned round-robin: expert e lives on rank e % W with local index
e // W, so the Zipf-heavy low expert ids spread over all ranks.  Each rank
routes its own token shard over all E experts; the per-token arithmetic is
moeMLP.forward's (model/moe.go:41-99), only the place where each expert runs
changes.  One forward:

  1. dispatch  -> send rows [T*k, H] fp16 sorted by (owner rank, local expert)
                  and counts [W, G] (G = E / W)
  2. exchange counts (all_to_all, G ints per peer)
  3. exchange rows   (all_to_all_single with per-peer row splits)
  4. experts   -> this rank's expert outputs for the received rows, same order
  5. exchange rows back (the reverse splits)
  6. combine   -> out [T, H], the rank-ordered weighted sum (model/moe.go:82-85)

`run_exchange` holds steps 2-6's bookkeeping and takes the three compute
steps as callables, so the CPU tests drive the same code with a CPU model of
the kernels.
"""
from __future__ import annotations

import ctypes as C

import numpy as np


def dispatch_key(e, E: int, W: int, slot=None):
    """Sort key of expert e: owner rank * (E/W) + local index; `slot` (the
    placement, a permutation of 0..E-1) or round-robin (e % W, e // W)."""
    if slot is not None:
        return np.asarray(slot)[e]
    return (e % W) * (E // W) + e // W


def round_robin_slots(E: int, W: int) -> np.ndarray:
    e = np.arange(E)
    return dispatch_key(e, E, W)


def balanced_slots(load, W: int) -> np.ndarray:
    """Placement by measured load: experts in decreasing load, each to the
    rank with the least load so far among those with a free place (E/W
    places per rank); local indices in increasing expert id.  Returns
    slot[e] = rank * (E/W) + local index."""
    load = np.asarray(load, np.float64)
    E = load.size
    G = E // W
    tot = np.zeros(W)
    owned = [[] for _ in range(W)]
    for e in np.argsort(-load, kind="stable"):
        free = [r for r in range(W) if len(owned[r]) < G]
        r = min(free, key=lambda q: (tot[q], q))
        owned[r].append(int(e))
        tot[r] += load[e]
    # then swap pairs between the most loaded rank and the others while that
    # lowers the maximum (the greedy pass must also fill every rank to E/W)
    for _ in range(4 * E):
        a = int(np.argmax(tot))
        best = None
        for b in range(W):
            if b == a:
                continue
            for i, x in enumerate(owned[a]):
                for j, y in enumerate(owned[b]):
                    d = load[x] - load[y]
                    if d <= 0:
                        continue
                    m = max(tot[a] - d, tot[b] + d)
                    if m < tot[a] - 1e-9 and (best is None or m < best[0]):
                        best = (m, b, i, j, d)
        if best is None:
            break
        _, b, i, j, d = best
        owned[a][i], owned[b][j] = owned[b][j], owned[a][i]
        tot[a] -= d
        tot[b] += d
    slot = np.empty(E, np.int32)
    for r in range(W):
        for j, e in enumerate(sorted(owned[r])):
            slot[e] = r * G + j
    return slot


def owned_experts(slot, rank: int, W: int):
    """Experts of `rank` in local order under placement `slot`."""
    slot = np.asarray(slot)
    G = slot.size // W
    mine = np.empty(G, np.int64)
    for e in range(slot.size):
        if slot[e] // G == rank:
            mine[slot[e] % G] = e
    return mine.tolist()


def exchange_counts(counts: np.ndarray, group=None, device=None) -> np.ndarray:
    """counts [W, G] (rows this rank sends to each peer, per local expert of
    that peer) -> [W, G] rows this rank receives from each peer."""
    import torch
    import torch.distributed as dist
    W, G = counts.shape
    send = torch.from_numpy(np.ascontiguousarray(counts, np.int32).reshape(-1))
    if device is not None:
        send = send.to(device)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.cpu().numpy().reshape(W, G)


def exchange_rows(rows, send_splits, recv_splits, group=None):
    """All-to-all of row blocks: rows[sum(send_splits), H] -> [sum(recv_splits), H]."""
    import torch
    import torch.distributed as dist
    out = torch.empty((int(sum(recv_splits)),) + tuple(rows.shape[1:]), dtype=rows.dtype,
                      device=rows.device)
    dist.all_to_all_single(out, rows, output_split_sizes=[int(v) for v in recv_splits],
                           input_split_sizes=[int(v) for v in send_splits], group=group)
    return out


def run_exchange(dispatch, experts, combine, group=None, device=None, timer=None):
    """Steps 1-6.  dispatch() -> (send_rows [n, H], counts [W, G]);
    experts(recv_rows, recv_counts) -> out_rows (same order);
    combine(back_rows) -> result.  `timer(name)` (optional) marks stage ends."""
    send_rows, counts = dispatch()
    if timer:
        timer("dispatch")
    recv_counts = exchange_counts(counts, group, device)
    send_splits = counts.sum(axis=1)
    recv_splits = recv_counts.sum(axis=1)
    recv_rows = exchange_rows(send_rows, send_splits, recv_splits, group)
    if timer:
        timer("a2a_dispatch")
    out_rows = experts(recv_rows, recv_counts)
    if timer:
        timer("experts")
    back_rows = exchange_rows(out_rows, recv_splits, send_splits, group)
    if timer:
        timer("a2a_combine")
    res = combine(back_rows)
    if timer:
        timer("combine")
    return res


IPC_HANDLE_BYTES = 64


class PeerExpertParallelMoE:
    """The GPU layer with the row exchange over NVLink peer memory
    (qgmoe_ep_px_*): the library maps every rank's exchange region and moves
    rows with its own kernels, so a forward is one stream of kernels with no
    host synchronisation.  Construction is collective (all ranks, same
    max_tokens); forward(x, out) works on this rank's token shard."""

    def __init__(self, layer, max_tokens: int, group=None):
        import torch
        import torch.distributed as dist
        from . import _check, lib
        self.layer = layer
        self.W = layer.ep_world
        L = lib()
        mine = np.zeros(IPC_HANDLE_BYTES, np.uint8)
        _check(L.qgmoe_ep_px_setup(layer.h, int(max_tokens), mine.ctypes.data_as(C.c_void_p)),
               "qgmoe_ep_px_setup")
        dev = torch.device("cuda", torch.cuda.current_device())
        t = torch.from_numpy(mine).to(dev)
        parts = [torch.empty_like(t) for _ in range(self.W)]
        dist.all_gather(parts, t, group=group)
        allh = np.ascontiguousarray(torch.cat(parts).cpu().numpy())
        _check(L.qgmoe_ep_px_connect(layer.h, allh.ctypes.data_as(C.c_void_p)),
               "qgmoe_ep_px_connect")
        dist.barrier(group=group)

    def forward(self, x, out, stream=None):
        import torch
        from . import _check, _ptr, _stream_ptr, lib
        s = stream or torch.cuda.current_stream(x.device)
        _check(lib().qgmoe_ep_px_forward(self.layer.h, _ptr(x), x.shape[0], _ptr(out),
                                         _stream_ptr(s)), "qgmoe_ep_px_forward")
        return out


class ExpertParallelMoE:
    """The GPU layer: an expert-parallel MoeMLP handle (ep_world = W) plus
    the NCCL exchanges.  forward(x, out) works on this rank's token shard."""

    def __init__(self, layer, group=None):
        self.layer = layer
        self.group = group
        self.W = layer.ep_world
        self.G = layer.n_experts // self.W
        self._send = None

    def _buffer(self, n, H, device):
        import torch
        if self._send is None or self._send.shape[0] < n or self._send.device != device:
            self._send = torch.empty((max(n, 1), H), dtype=torch.float16, device=device)
        return self._send[:n]

    def forward(self, x, out, stream=None, timer=None):
        import torch
        from . import _check, _ptr, _stream_ptr, lib
        L = lib()
        T, H = x.shape
        k = self.layer.top_k
        s = stream or torch.cuda.current_stream(x.device)
        sp = _stream_ptr(s)

        def dispatch():
            send = self._buffer(T * k, H, x.device)
            _check(L.qgmoe_ep_dispatch(self.layer.h, _ptr(x), T, _ptr(send), sp),
                   "qgmoe_ep_dispatch")
            counts = np.zeros(self.W * self.G, np.int32)
            _check(L.qgmoe_ep_send_counts(self.layer.h,
                                          counts.ctypes.data_as(C.POINTER(C.c_int32)), sp),
                   "qgmoe_ep_send_counts")
            return send, counts.reshape(self.W, self.G)

        def experts(recv_rows, recv_counts):
            R = recv_rows.shape[0]
            out_rows = torch.empty_like(recv_rows)
            rc_host = np.ascontiguousarray(recv_counts, np.int32).reshape(-1)
            _check(L.qgmoe_ep_experts(self.layer.h, _ptr(recv_rows), R,
                                      rc_host.ctypes.data_as(C.POINTER(C.c_int32)),
                                      _ptr(out_rows), sp), "qgmoe_ep_experts")
            return out_rows

        def combine(back_rows):
            _check(L.qgmoe_ep_combine(self.layer.h, _ptr(back_rows), T, _ptr(out), None, None,
                                      sp), "qgmoe_ep_combine")
            return out

        with torch.cuda.stream(s):
            return run_exchange(dispatch, experts, combine, self.group, x.device, timer)
