#!/usr/bin/env python
"""Benchmark of the B200 MoE layer (qwen-go moeMLP.forward, model/moe.go:41-99).

Default workload = config 3 of the benchmark plan: the Qwen3-30B-A3B-shaped layer
(H=2048, E=128, top-8, I=768, int8 group-32 experts with fp16 scales, f32
router) in prefill over 4096 tokens whose routing follows a Zipf(1.1) skew.
One step = one full MoE-layer forward over the batch.  Inputs are synthetic
(seeded counter-based generator); weights are random-init of that
architecture.  The weights (641.7 MB) exceed the 126 MB L2, so no flush is
needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  --impl reference times the CPU restatement
of the reference's Go MoE forward (token-parallel over all host cores).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(REPO, "qwen-go_b200"), os.path.join(REPO, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

CONFIGS = {
    # name: shapes, bits, tokens, seed, zipf skew
    "c1": dict(H=1024, E=16, k=4, I=512, Is=1024, bits=8, T=32, seed=1, zipf=False,
               desc="c1 int8 decode MoE layer (H=1024, E=16, top-4, I=512, shared 1024)"),
    "c2": dict(H=2048, E=128, k=8, I=768, Is=0, bits=4, T=64, seed=2, zipf=False,
               desc="c2 int4 decode MoE layer (Qwen3-30B-A3B-shaped)"),
    "c3": dict(H=2048, E=128, k=8, I=768, Is=0, bits=8, T=4096, seed=3, zipf=True,
               desc="c3 int8 prefill MoE layer (Qwen3-30B-A3B-shaped), Zipf(1.1) routing"),
}
L2_BYTES = 126 * 2**20
MU = 1.0  # activation mean for the Zipf construction


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch
# of the dominant kernel, from the ncu --set full captures summarised in
# profiles/ (same workload, same kernel build): (config, tokens, kernel) ->
# (bytes, summary file).  Other workloads report null.
NCU_TRAFFIC = {
    ("c3", 4096, "gate_up"): (568.004864e6 + 52.227584e6, "profiles/full_c3_prefill_t4096.md"),
    ("c2", 64, "gate_up"): (219.797248e6 + 5.550848e6, "profiles/full_c2_decode_t64.md"),
    ("c2", 1, "decode"): (22.441472e6, "profiles/full_k_decode_c2.md"),
    ("c2", 8, "decode"): (136.638976e6 + 4.069632e6, "profiles/full_k_decode_c2.md"),
}


def ncu_traffic(config, T, kernel):
    hit = NCU_TRAFFIC.get((config, T, kernel))
    return (hit[0], hit[1]) if hit else (None, None)


def weight_bytes(cfg):
    """Bytes of one expert's gate_up + down weights (codes + fp16 scales)."""
    H, I, bits = cfg["H"], cfg["I"], cfg["bits"]
    n = 3 * H * I
    if bits == 32:
        return n * 4
    return n * bits // 8 + (n // 32) * 2


def layer_flops(cfg, T):
    H, E, k, I, Is = cfg["H"], cfg["E"], cfg["k"], cfg["I"], cfg["Is"]
    return 2 * T * k * 3 * H * I + 2 * T * E * H + (2 * T * 3 * H * Is if Is else 0)


# --------------------------------------------------------------------------
# Zipf routing construction (weights-side bias, the reference math unchanged)
# --------------------------------------------------------------------------


def zipf_target(T, k, E, s=1.1):
    f = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    total = T * k
    cap = float(T)
    tgt = np.zeros(E)
    free = np.ones(E, bool)
    rem = float(total)
    for _ in range(E):
        share = f * free
        t = rem * share / share.sum()
        over = (t > cap) & free
        if not over.any():
            tgt[free] = t[free]
            break
        tgt[over] = cap
        free &= ~over
        rem = total - tgt[~free].sum()
    return tgt


def calibrate_zipf(router, x, k):
    """Picks c so that adding b_e = -1.1 ln(e+1) c / (mu H) to router row e
    (rows first centred, so the skew comes from b_e alone) makes the TOPK
    selection histogram closest (L1, sorted) to Zipf(1.1) capped at T."""
    E, H = router.shape
    T = x.shape[0]
    base = x.astype(np.float64) @ router.astype(np.float64).T           # [T, E]
    xs = x.astype(np.float64).sum(axis=1, keepdims=True)                 # [T, 1]
    tgt = np.sort(zipf_target(T, k, E))[::-1]
    best = (None, math.inf, None)
    for c in np.arange(0.0, 2.001, 0.05):
        b = -1.1 * np.log(np.arange(E) + 1.0) * c
        logits = base + xs * (b / (MU * H))[None, :]
        sel = np.argpartition(-logits, k - 1, axis=1)[:, :k]
        hist = np.bincount(sel.ravel(), minlength=E)
        d = np.abs(np.sort(hist)[::-1] - tgt).sum()
        if d < best[1]:
            best = (float(round(c, 2)), d, hist)
    return best[0], best[2]


def zipf_bias_rows(E, H, c):
    b = -1.1 * np.log(np.arange(E) + 1.0) * c
    return (b / (MU * H)).astype(np.float32)


# --------------------------------------------------------------------------
# Layer construction
# --------------------------------------------------------------------------


def build_gpu_layer(cfg, device, ep_world=1, ep_rank=0, keep_host=True, placement="balanced"):
    """Generates the layer on the GPU with the library's generator/quantiser.
    With ep_world > 1 only the experts this rank owns are generated, from the
    same counter-based streams at their offsets, so every rank holds exactly
    its slice of the single-GPU layer.  Placement: "balanced" (skewed
    routing: experts spread over the ranks by the expert loads measured on the
    calibration sample, rank 0's choice broadcast to all ranks) or
    "round-robin" (expert e on rank e % W).
    Returns (MoeMLP, x [T, H] for all tokens, host copies, routing info)."""
    import torch
    import qgmoe

    H, E, k, I, Is, bits, seed = (cfg[n] for n in ("H", "E", "k", "I", "Is", "bits", "seed"))
    dev = torch.device("cuda", device)

    def g(stream, shape, std=0.02, offset=0):
        t = torch.empty(shape, dtype=torch.float32, device=dev)
        return qgmoe.randn_device(t, seed, stream, std, offset=offset)

    router = g(0, (E, H))
    info = {}
    x = g(100, (cfg["T"], H), 1.0)
    if cfg["zipf"]:
        x += MU
        router -= router.mean(dim=1, keepdim=True)
        xs = x[:1024].cpu().numpy()
        c, hist = calibrate_zipf(router.cpu().numpy(), xs, k)
        router += torch.from_numpy(zipf_bias_rows(E, H, c)).to(dev)[:, None]
        info["zipf_c"] = c
    args = dict(router=router)
    host = {"router": router.cpu().numpy()} if keep_host else {}
    slot = None
    if ep_world > 1:
        from qgmoe.ep import balanced_slots, owned_experts, round_robin_slots
        if placement == "balanced" and cfg["zipf"]:
            slot = balanced_slots(hist, ep_world)
            import torch.distributed as dist
            if dist.is_initialized():  # every rank takes rank 0's placement
                t = torch.from_numpy(slot.astype(np.int64)).to(dev)
                dist.broadcast(t, 0)
                slot = t.cpu().numpy().astype(np.int32)
            info["placement"] = "balanced by calibration-sample expert load"
        else:
            slot = round_robin_slots(E, ep_world).astype(np.int32)
            info["placement"] = "round-robin: expert e on rank e % N"
        mine = owned_experts(slot, ep_rank, ep_world)  # local expert order
        G = E // ep_world
        if cfg["zipf"]:
            load = np.zeros(ep_world)
            for e in range(E):
                load[slot[e] // G] += hist[e]
            info["rank_load_share"] = [round(float(v) / float(load.sum()), 4) for v in load]
    else:
        mine = list(range(E))

    def expert_stack(stream, rows_per_e, cols):
        if ep_world == 1:
            return g(stream, (E * rows_per_e, cols))
        return torch.cat([g(stream, (rows_per_e, cols), offset=e * rows_per_e * cols)
                          for e in mine])

    mats = {"gate_up": lambda: expert_stack(1, 2 * I, H), "down": lambda: expert_stack(2, H, I)}
    if Is:
        args["shared_gate"] = g(3, (H,))
        if keep_host:
            host["shared_gate"] = args["shared_gate"].cpu().numpy()
        mats.update(shared_gate=lambda: g(4, (Is, H)), shared_up=lambda: g(5, (Is, H)),
                    shared_down=lambda: g(6, (H, Is)))
    for name, make in mats.items():
        w = make()
        if bits == 32:
            key = {"gate_up": "gate_up", "down": "down"}.get(name, name + "_proj")
            args[key] = w
            if keep_host:
                host[name] = w.cpu().numpy()
        else:
            q, _s32, s16 = qgmoe.quantize_device(w, bits)
            args[name + "_q"] = q
            args[name + "_scale"] = s16
            if keep_host:
                host[name + "_q"] = q.cpu().numpy()
                host[name + "_s"] = s16.cpu().numpy().view(np.float16).astype(np.float32)
        del w
    torch.cuda.synchronize(dev)
    layer = qgmoe.MoeMLP(n_embed=H, n_experts=E, top_k=k, n_moe_mlp=I, n_shared_mlp=Is, bits=bits,
                         router_mode=qgmoe.ROUTER_TOPK, device=device, ep_world=ep_world,
                         ep_rank=ep_rank, ep_slot=slot, **args)
    del args
    torch.cuda.empty_cache()
    return layer, x, host, info


def oracle_weights(cfg, host):
    import qg_oracle as O
    H, E, k, I, Is, bits = (cfg[n] for n in ("H", "E", "k", "I", "Is", "bits"))
    m = O.MoeWeights(H=H, E=E, k=k, I=I, Is=Is, bits=bits, router=host["router"],
                     shared_gate=host.get("shared_gate"))
    if bits == 32:
        m.gate_up = host["gate_up"].reshape(E, 2 * I, H)
        m.down = host["down"].reshape(E, H, I)
        if Is:
            m.sh_gate, m.sh_up, m.sh_down = (host["shared_gate"], host["shared_up"],
                                             host["shared_down"])
    else:
        for name, key in (("gate_up", "gate_up"), ("down", "down"), ("shared_gate", "sh_gate"),
                          ("shared_up", "sh_up"), ("shared_down", "sh_down")):
            if name + "_q" in host:
                m.q[key] = host[name + "_q"]
                m.s[key] = host[name + "_s"]
    return m


def oracle_layer_cpu(cfg, threads):
    """The same layer generated entirely on the CPU by the oracle's generator
    and quantiser (used by the reference arm, which runs no GPU code)."""
    import qg_oracle as O
    from concurrent.futures import ThreadPoolExecutor
    H, E, k, I, Is, bits, seed = (cfg[n] for n in ("H", "E", "k", "I", "Is", "bits", "seed"))

    def gen(stream, shape, std=0.02):
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        chunk = (n + threads - 1) // threads

        def part(i):
            lo, hi = i * chunk, min(n, (i + 1) * chunk)
            if lo < hi:
                out[lo:hi] = O.randn(seed, stream, (hi - lo,), std, offset=lo)
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(part, range(threads)))
        return out.reshape(shape)

    host = {"router": gen(0, (E, H))}
    x = gen(100, (cfg["T"], H), 1.0)
    info = {}
    if cfg["zipf"]:
        x += MU
        host["router"] -= host["router"].mean(axis=1, keepdims=True)
        c, hist = calibrate_zipf(host["router"], x[:1024], k)
        host["router"] += zipf_bias_rows(E, H, c)[:, None]
        info["zipf_c"] = c
        info["calibration_expert_load_top8"] = sorted(hist.tolist(), reverse=True)[:8]
    mats = {"gate_up": (1, (E * 2 * I, H)), "down": (2, (E * H, I))}
    if Is:
        host["shared_gate"] = gen(3, (H,))
        mats.update(shared_gate=(4, (Is, H)), shared_up=(5, (Is, H)), shared_down=(6, (H, Is)))
    for name, (stream, shape) in mats.items():
        w = gen(stream, shape)
        if bits == 32:
            host[name] = w
        else:
            q, s = O.quantize(w, bits)
            host[name + "_q"] = q
            host[name + "_s"] = O.f16_round(s)
    return oracle_weights(cfg, host), x, info


# --------------------------------------------------------------------------
# Clock sampling
# --------------------------------------------------------------------------


class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons of one GPU during
    the timed regions: NVML polled every ~2 ms from a thread, so even a
    region of a few ms gets several samples."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_device):
        self.dev = cuda_device
        self.samples = []  # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self.stop = threading.Event()
        self.t = None
        self.nvml = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.dev)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)

    def __enter__(self):
        try:
            nv, h = self._handle()
            self.nvml = nv
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_r = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons

            def run():
                while not self.stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             int(get_r(h))))
                    except Exception:
                        pass
                    time.sleep(0.002)
            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
        except Exception:
            self.nvml = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml, 2 ms poll"}


# --------------------------------------------------------------------------
# Arms
# --------------------------------------------------------------------------


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline_ours(cfg, host, x_host, budget_s=12.0):
    """The oracle (C restatement of moe.go, -O2, no FMA contraction), one
    thread, as decodeLayers calls mlp.forward: token by token."""
    import qg_oracle as O
    m = oracle_weights(cfg, host)
    t0 = time.perf_counter()
    O.moe_forward(m, x_host[:1])
    t1 = max(time.perf_counter() - t0, 1e-4)
    n = int(max(1, min(cfg["T"], budget_s / t1)))
    t0 = time.perf_counter()
    O.moe_forward(m, x_host[1:1 + n] if n + 1 <= cfg["T"] else x_host[:n])
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} of the {cfg['T']} tokens, same weights, serial per token "
                      f"(oracle/qg_oracle.c, 1 thread; the Go reference's MoE is serial, "
                      f"model/model.go:507-514)"}


def oracle_expert_load(m, x, threads):
    """Expert load of the whole batch as the oracle routes it (serial-order
    f32 logits, then the reference's top-k): the same histogram the GPU
    arm reports from its own routing, over every token, not the sample."""
    import ctypes as C
    from concurrent.futures import ThreadPoolExecutor

    import qg_oracle as O
    L, f32p = O.lib(), C.POINTER(C.c_float)
    T, H = x.shape
    E, k = m.router.shape[0], m.k
    router = np.ascontiguousarray(m.router, np.float32)
    idx = np.zeros((T, k), np.int32)

    def part(i):
        logits = np.zeros(E, np.float32)
        for t in range(i, T, threads):
            xt = np.ascontiguousarray(x[t], np.float32)
            L.qgo_matmul_vec(xt.ctypes.data_as(f32p), router.ctypes.data_as(f32p), H, E,
                             logits.ctypes.data_as(f32p))
            idx[t] = O.route_token(logits, k, O.ROUTER_TOPK)[0]
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(part, range(threads)))
    return np.bincount(idx.ravel(), minlength=E)


def run_reference(args, cfg):
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    import qg_oracle as O
    threads = os.cpu_count() or 1
    m, x, info = oracle_layer_cpu(cfg, threads)
    hist = oracle_expert_load(m, x, threads)
    info["expert_load_top8"] = sorted(hist.tolist(), reverse=True)[:8]
    info["expert_load_min"] = int(hist.min())
    # size one step to a bounded token sample (a few seconds on all cores)
    t0 = time.perf_counter()
    O.moe_forward_mt(m, x[:threads], threads)
    per_tok = max((time.perf_counter() - t0) / threads, 1e-6)  # wall per token per core
    budget = float(os.environ.get("QG_REF_STEP_S", "6"))
    n = int(max(threads, min(cfg["T"], budget * threads / max(per_tok * threads, 1e-6))))
    n = min(n, cfg["T"])
    for _ in range(args.warmup):
        O.moe_forward_mt(m, x[:n], threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.moe_forward_mt(m, x[:n], threads)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    val = n * args.steps / tot
    line = {
        "impl": "reference", "metric": "MoE-layer tokens/s", "value": val, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": dict(config_json(cfg, world), **info),
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{n} of {cfg['T']} tokens per step, token-parallel over "
                                   f"{threads} threads (the Go reference runs the MoE serially "
                                   f"per token; this restatement spreads tokens over cores)"},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def dtype_label(cfg, layer):
    """The arithmetic the timed expert products run in: the tensor path
    multiplies fp16 activations by fp16 dequantised weights into f32
    accumulators (f32 in, f32 out); the router and the CUDA-core path are
    f32 throughout."""
    if cfg["bits"] in (8, 4):
        return (f"fp16 tensor-core operands (activations, int{cfg['bits']} weights dequantised to "
                f"fp16), f32 accumulate, f32 I/O; f32 router")
    return "f32"


def config_json(cfg, world):
    wb = weight_bytes(cfg)
    return {"workload": cfg["desc"], "H": cfg["H"], "E": cfg["E"], "top_k": cfg["k"],
            "I": cfg["I"], "shared_I": cfg["Is"], "bits": cfg["bits"],
            "scale": "fp16 group-32", "tokens": cfg["T"], "router": "topk f32",
            "l2": ("no flush: weights %.1f MB > 126 MB L2" % (cfg["E"] * wb / 1e6)
                   if cfg["E"] * wb > L2_BYTES else "L2 flushed between steps"),
            "parallelism": "single GPU" if world == 1 else f"ep{world}",
            "batch": "T tokens per GPU (weak scaling over GPUs)"}


def stage_bytes(cfg, stage, distinct, T):
    """Algorithmic HBM bytes of one decode stage: the weights of the experts
    the batch routed to (gate_up = 2/3 of an expert, down = 1/3), the shared
    expert's share, and the stage's activations (f32 in and out)."""
    H, E, I, Is = cfg["H"], cfg["E"], cfg["I"], cfg["Is"]
    bpw = {32: 4.0, 16: 2.0, 8: 1.0 + 2 / 32, 4: 0.5 + 2 / 32}[cfg["bits"]]
    if stage == "route":
        return (E + (1 if Is else 0)) * H * 4 + T * H * 4
    if stage == "gate_up":
        return (distinct * 2 * I * H + 2 * Is * H) * bpw + T * H * 4
    if stage == "down":
        return (distinct * I * H + Is * H) * bpw + T * H * 4
    if stage == "decode":  # the one-launch decode kernel: router, experts, x in, out
        return ((E + (1 if Is else 0)) * H * 4 + (distinct * 3 * I * H + 3 * Is * H) * bpw
                + 2 * T * H * 4)
    return T * H * 4 * (cfg["k"] + 1)  # combine: k rows in, one out


def time_forwards(layer, x, out, sel, steps, flush, stream, dev):
    """K forwards bracketed one by one by CUDA events on the launching stream
    (an L2 flush, when given, runs before each event pair); then the same K
    forwards with per-stage events (graphs off).  Returns (total ms, stage ms
    per forward, forwards timed)."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    torch.cuda.synchronize(dev)
    for i in range(steps):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush.zero_()
        evs[i][0].record(stream)
        layer.forward_device(x, out, sel_idx=sel, stream=stream)
        evs[i][1].record(stream)
    torch.cuda.synchronize(dev)
    layer.sync(stream)
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    layer.set_timing(True)
    for _ in range(steps):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush.zero_()
        layer.forward_device(x, out, sel_idx=sel, stream=stream)
    stage_ms, nf = layer.read_timing()
    layer.set_timing(False)
    layer.sync(stream)
    return total_ms, {k: v / max(nf, 1) for k, v in stage_ms.items()}, nf


def measure_decode(name, T, steps, dev, peaks):
    """One decode configuration: tokens/s of the layer forward (graph replay,
    L2 flushed before every forward when the layer fits in L2), the stage
    times, and the dominant stage's algorithmic HBM bytes against the
    measured copy bandwidth."""
    import torch
    cfg = dict(CONFIGS[name])
    cfg["T"] = T
    layer, x, _host, _info = build_gpu_layer(cfg, dev, keep_host=False)
    out = torch.empty_like(x)
    sel = torch.empty((T, cfg["k"]), dtype=torch.int32, device=x.device)
    fits_l2 = cfg["E"] * weight_bytes(cfg) + 3 * cfg["Is"] * cfg["H"] * 2 <= L2_BYTES
    flush = (torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=x.device)
             if fits_l2 else None)
    stream = torch.cuda.Stream(dev)
    for _ in range(5):
        layer.forward_device(x, out, sel_idx=sel, stream=stream)
    layer.sync(stream)
    distinct = int((np.bincount(sel.cpu().numpy().ravel(), minlength=cfg["E"]) > 0).sum())
    total_ms, stages, _ = time_forwards(layer, x, out, sel, steps, flush, stream, dev)
    dom = max(("decode", "gate_up", "down", "route"), key=lambda s: stages.get(s, 0.0))
    by = stage_bytes(cfg, dom, distinct, T)
    gbs = by / (stages[dom] / 1e3) / 1e9
    res = {"config": name, "tokens": T, "tokens_per_s": T * steps / (total_ms / 1e3),
           "forward_us": 1e3 * total_ms / steps, "distinct_experts": distinct,
           "stage_us": {k: round(1e3 * v, 2) for k, v in stages.items()},
           "dominant": dom, "dominant_bytes": int(by), "dominant_gbs": gbs,
           "hbm_frac": gbs / peaks["hbm_gbs"], "l2": "flushed" if flush is not None else
           "weights > L2", "launches": layer.last_launch_count()}
    layer.close()
    del x, out, sel, flush
    torch.cuda.empty_cache()
    return res


def run_stack(dev):
    """Config 4's MoE layers: 48 int8 layers of the Qwen3-MoE shape (H=2048,
    E=128, top-8, I=768, ~31 GB of weights, so nothing stays in L2), a
    512-token prefill and 256 single-token decode steps layer after layer
    through qgmoe_forward from the plain-C host tests/c/stack_host.c (the
    call a cgo shim makes, the residual kept on the host as decodeLayers
    does).  Attention, embeddings and sampling are outside the rebuilt path.
    Reports the host's JSON line (MoE tokens/s = tokens / time inside
    qgmoe_forward; loop tokens/s includes the host's norm and residual)."""
    import torch
    from qgmoe.build import build_host
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    exe = build_host("stack_host")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", str(dev)))
    r = subprocess.run([exe, "bench", "48", "2048", "128", "8", "768", "8", "512", "256", "4"],
                       capture_output=True, text=True, timeout=900, env=env)
    if r.returncode != 0:
        return {"error": (r.stderr or r.stdout).strip()[-300:]}
    res = json.loads(r.stdout.strip().splitlines()[-1])
    res["workload"] = ("c4: 48 int8 MoE layers (H=2048, E=128, top-8, I=768), 512-token "
                       "prefill + 256 decode steps through qgmoe_forward from a C host; "
                       "synthetic N(0,1) activations, seed 4")
    return res


def run_ours(args, cfg):
    import torch
    import qgmoe

    world, rank, local = dist_setup(args.gpus)
    dev = local
    torch.cuda.set_device(dev)
    if world > 1:
        return run_ep(args, cfg, world, rank, local)
    peaks, peak_src = load_peaks()
    layer, x, host, info = build_gpu_layer(cfg, dev)
    layer.set_path({"auto": qgmoe.PATH_AUTO, "cuda_core": qgmoe.PATH_CUDA_CORE,
                    "tensor": qgmoe.PATH_TENSOR}[args.path])
    info["path"] = args.path
    T, H, k = cfg["T"], cfg["H"], cfg["k"]
    out = torch.empty_like(x)
    sel = torch.empty((T, k), dtype=torch.int32, device=x.device)
    flush = None
    if cfg["E"] * weight_bytes(cfg) <= L2_BYTES:
        flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=x.device)
    # A dedicated stream: the library's NULL-stream argument means "the
    # handle's own stream", so torch's default stream must not be passed.
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize(dev)
    for _ in range(max(args.warmup, 3)):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush.zero_()
        layer.forward_device(x, out, sel_idx=sel, stream=stream)
    layer.sync(stream)
    hist = np.bincount(sel.cpu().numpy().ravel(), minlength=cfg["E"])
    distinct = int((hist > 0).sum())

    # ---- timed regions (device events on the launching stream) ----
    # Repeated identical forwards replay a CUDA graph inside the library.
    # Each forward is bracketed by its own event pair, so the L2 flush that
    # precedes it (small layers) stays outside the timed sum; the second pass
    # records an event between consecutive stages (graphs off).
    barrier(world)
    with ClockSampler(dev) as clk:
        total_ms, stages, nf = time_forwards(layer, x, out, sel, args.steps, flush, stream, dev)
        total_ms = max_over_ranks(total_ms, world)
        ms_per_step = total_ms / args.steps
        forward_ms = sum(stages.values())
        value = T * world * args.steps / (total_ms / 1e3)

        # ---- end to end through the public host API (pinned buffers) ----
        xh = x.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        L = qgmoe.lib()
        for _ in range(2):
            rc = L.qgmoe_forward(layer.h, xh.data_ptr(), T, oh.data_ptr(), None, None)
            assert rc == 0, qgmoe.last_error()
        e2e_steps = max(1, min(args.steps, 20))
        barrier(world)
        e2e_s = 0.0
        for _ in range(e2e_steps):
            if flush is not None:
                with torch.cuda.stream(stream):
                    flush.zero_()
                stream.synchronize()
            t0 = time.perf_counter()
            L.qgmoe_forward(layer.h, xh.data_ptr(), T, oh.data_ptr(), None, None)
            e2e_s += time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s, world)
    e2e = {"value": T * world * e2e_steps / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": T * H * 4, "d2h_bytes_per_step": T * H * 4,
           "api": "qgmoe_forward (host pointers, blocking)"}

    # ---- roofline of the dominant kernel ----
    dom = max(stages, key=stages.get)
    dom_ms = stages[dom]
    prefill = cfg["T"] >= 512
    traffic, traffic_src = ncu_traffic(args.config, T, dom)
    if prefill:
        Iw = 2 * cfg["I"] if dom == "gate_up" else cfg["I"]
        flops = 2.0 * T * k * Iw * H if dom in ("gate_up", "down") else 2.0 * T * cfg["E"] * H
        achieved = flops / (dom_ms / 1e3) / 1e12
        peak = peaks["bf16_tflops"]
        roof = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{peak_src} bf16 dense (MEASURED_PEAKS.json bf16_tflops)",
                "algorithmic_per_launch": f"{flops / 1e9:.1f} GFLOP", "traffic": traffic}
    else:
        bytes_ = stage_bytes(cfg, dom, distinct, T)
        achieved = bytes_ / (dom_ms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"{peak_src} HBM copy",
                "algorithmic_per_launch": f"{bytes_ / 1e6:.2f} MB", "traffic": traffic}
    if traffic is not None:
        roof["traffic_unit"] = "DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)"
        roof["traffic_source"] = traffic_src
    launches = layer.last_launch_count()
    layer.close()
    del layer, out, sel, flush
    torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_ours(cfg, host, x.cpu().numpy())
    del x

    # ---- the decode configurations (1 GPU, replicas only) ----
    decode = None
    if args.config == "c3" and not args.no_decode:
        decode = [measure_decode(name, t, max(args.steps, 50), dev, peaks)
                  for name, ts in (("c1", (1, 8, 32)), ("c2", (1, 16, 64))) for t in ts]
    stack = None
    if args.config == "c3" and not args.no_stack:
        stack = run_stack(dev)

    if rank == 0:
        cfgj = config_json(cfg, world)
        cfgj.update(info)
        cfgj["expert_load_top8"] = sorted(hist.tolist(), reverse=True)[:8]
        cfgj["expert_load_min"] = int(hist.min())
        cfgj["distinct_experts"] = distinct
        line = {
            "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype_label(cfg, None), "data": "synthetic",
            "config": cfgj, "stage_ms": stages, "forward_ms_device": forward_ms,
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
        }
        if decode is not None:
            line["decode"] = decode
        if stack is not None:
            line["c4_stack"] = stack
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_ep(args, cfg, world, rank, local):
    """Config 3 over `world` GPUs: expert parallelism (experts round-robin,
    E/W per rank), every rank routing its own batch of T tokens (tokens
    r*T .. (r+1)*T-1 of one generated stream).  Rows move through the
    library's peer-memory exchange (default) or, with --ep-nccl, through NCCL
    all-to-all driven by the host.  Weak scaling: the work per GPU stays one
    T-token layer."""
    import torch
    import torch.distributed as dist
    import qgmoe
    from qgmoe.ep import ExpertParallelMoE, PeerExpertParallelMoE

    dev = local
    layer, x0, _host, info = build_gpu_layer(cfg, dev, world, rank, keep_host=False,
                                             placement=args.ep_placement)
    T, H = cfg["T"], cfg["H"]
    T_all = T * world
    x = torch.empty((T, H), dtype=torch.float32, device=x0.device)
    qgmoe.randn_device(x, cfg["seed"], 100, 1.0, offset=rank * T * H)
    if cfg["zipf"]:
        x += MU
    del x0
    out = torch.empty_like(x)
    peer = not args.ep_nccl
    ep = PeerExpertParallelMoE(layer, T) if peer else ExpertParallelMoE(layer)
    stream = torch.cuda.Stream(dev)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            ep.forward(x, out, stream)
    stream.synchronize()

    # ---- timed region: device events on the launching stream, max over ranks
    barrier(world)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                ep.forward(x, out, stream)
            ev1.record(stream)
        torch.cuda.synchronize(dev)
    total_ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    value = T_all * args.steps / (total_ms / 1e3)

    # ---- stage durations: a second pass with events between the stages ----
    stages = {}
    if peer:
        layer.set_timing(True)
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                ep.forward(x, out, stream)
        stream.synchronize()
        st_ms, nf = layer.read_timing()
        layer.set_timing(False)
        stages = {kk: v / max(nf, 1) for kk, v in st_ms.items()}
    else:
        marks = []

        def timer(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            marks.append((name, ev))

        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                start = torch.cuda.Event(enable_timing=True)
                start.record(stream)
                marks.append(("start", start))
                ep.forward(x, out, stream, timer=timer)
        torch.cuda.synchronize(dev)
        prev = None
        for name, ev in marks:
            if name != "start":
                stages[name] = stages.get(name, 0.0) + prev.elapsed_time(ev)
            prev = ev
        stages = {kk: v / args.steps for kk, v in stages.items()}
    all_stages = [None] * world  # every rank's stage durations (ms), rank order
    dist.all_gather_object(all_stages, stages)
    stage_range = {kk: [round(min(r.get(kk, 0.0) for r in all_stages), 4),
                        round(max(r.get(kk, 0.0) for r in all_stages), 4)] for kk in stages}
    barrier(world)

    # ---- roofline: the expert stage (grouped GEMMs on this rank) ----
    peaks, peak_src = load_peaks()
    exp_ms = max_over_ranks(stages.get("experts", stages.get("gate_up", 0.0) +
                                       stages.get("down_return", 0.0)), world)
    k, I = cfg["k"], cfg["I"]
    flops = 2.0 * T * k * 3 * I * H  # rows per rank on average = T*k
    achieved = flops / (exp_ms / 1e3) / 1e12 if exp_ms > 0 else 0.0
    roof = {"bound": "tensor", "kernel": "experts (gate_up + down grouped GEMMs, slowest rank)",
            "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_tflops"],
            "peak_source": f"{peak_src} bf16 dense (MEASURED_PEAKS.json bf16_tflops)",
            "algorithmic_per_launch": f"{flops / 1e9:.1f} GFLOP per rank (mean)", "traffic": None}

    # ---- end to end: pinned host shard -> device -> layer -> host ----
    xh = x.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    e2e_steps = max(1, min(args.steps, 20))
    barrier(world)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            x.copy_(xh, non_blocking=True)
            ep.forward(x, out, stream)
            oh.copy_(out, non_blocking=True)
            stream.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": T_all * e2e_steps / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": T_all * H * 4, "d2h_bytes_per_step": T_all * H * 4,
           "api": ("qgmoe_ep_px_forward via qgmoe.ep.PeerExpertParallelMoE" if peer else
                   "qgmoe_ep_* via qgmoe.ep.ExpertParallelMoE") + " (pinned host shards)"}

    if rank == 0:
        cfgj = config_json(cfg, world)
        cfgj.update(info)
        cfgj["exchange"] = ("library kernels over NVLink peer memory (CUDA IPC), no host sync"
                            if peer else "NCCL all_to_all_single (host-side split sizes)")
        cfgj["tokens_per_rank"] = T
        cfgj["tokens"] = T_all
        line = {
            "metric": "MoE-layer tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": dtype_label(cfg, None), "data": "synthetic",
            "config": cfgj, "stage_ms_rank0": stages, "stage_ms_min_max_over_ranks": stage_range,
            "roofline": roof, "cpu_baseline": None,
            "e2e": e2e, "gpu_launches": (layer.last_launch_count() if peer else 4 + 3 + 1)
            * args.steps, "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    barrier(world)
    del ep
    layer.close()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3", choices=sorted(CONFIGS))
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--path", default="auto", choices=["auto", "cuda_core", "tensor"],
                    help="expert-product path (qgmoe_set_path)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="config 3: skip the decode configurations in the line")
    ap.add_argument("--no-stack", action="store_true",
                    help="config 3: skip the 48-layer config-4 stack in the line")
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "round-robin"],
                    help="N > 1: expert placement over the ranks")
    ap.add_argument("--ep-nccl", action="store_true",
                    help="N > 1: move rows with NCCL all-to-all instead of peer memory")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.tokens:
        cfg["T"] = args.tokens
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
