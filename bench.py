"""Benchmark of the fused FP8 block-scale MoE (DeepSeek-V3 routing) on B200.

One step = one call of the operator on one batch of synthetic input (seeded, shapes and
distributions of the operator definition; no dataset is available offline). The headline
workload is the decode configuration T=64 (seed 4) with 32 local experts. With N > 1 GPUs each
rank runs its own token batch (seed 4 + rank) against its own contiguous 32-expert shard
(local_expert_offset = 32 * rank mod 256): per-GPU work is fixed, there is no data exchange in
this operator, so scaling is weak. The NCCL expert-parallel variant with dispatch/combine
all-to-all is ``--workload ep``.

Prints ONE JSON line on rank 0. ``--impl reference`` times the reference algorithm's CPU
restatement (the oracle port; the reference itself is Triton-only) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from flashinfer_b200 import _lib, moe as fmoe, workload as wl  # noqa: E402

METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
SMALL_T = 64           # T <= SMALL_T: fused route/plan/scatter cluster kernel
SPLIT_MAX_T = 32       # T <= SPLIT_MAX_T: split-K finish kernel after each GEMM


def kernels_per_call(T: int) -> int:
    """Launches of one call: route+hist, scan, scatter, gather, gemm1, gemm2, combine; for
    T <= SMALL_T the fused plan kernel replaces the first three, and for T <= SPLIT_MAX_T a
    split-K finish kernel follows each GEMM."""
    if T <= SPLIT_MAX_T:
        return 7
    if T <= SMALL_T:
        return 5
    return 7


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ------------------------------------------------------------------------------- accounting
def call_accounting(ids: np.ndarray, local_start: int, e_local: int, T: int):
    """P, active experts, algorithmic FLOPs and bytes of one call (minimum traffic: the active
    experts' weights and scales, the per-token inputs and output)."""
    loc = ids.astype(np.int64) - local_start
    hit = (loc >= 0) & (loc < e_local)
    P = int(hit.sum())
    active = int(np.unique(loc[hit]).size)
    H, I = wl.HIDDEN, wl.INTER
    flops = P * wl.flops_per_pair()
    total_bytes = active * wl.bytes_per_expert() + T * wl.bytes_per_token() + 512
    w1_bytes = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    gemm1_bytes = active * w1_bytes + P * (H + 4 * H // 128) + P * (2 * I + 4 * I // 128)
    w2_bytes = H * I + (H // 128) * (I // 128) * 4
    gemm2_bytes = active * w2_bytes + P * (2 * I + 4 * I // 128) + P * H * 2
    return {"P": P, "active_experts": active, "flops": flops, "bytes": total_bytes,
            "gemm1_bytes": gemm1_bytes, "gemm1_flops": P * 2 * H * 2 * I,
            "gemm2_bytes": gemm2_bytes, "gemm2_flops": P * 2 * I * H * 2}


# ------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        try:
            self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            self.reasons |= nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(0.002)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._loop, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._ok:
            self._stop.set()
            self._t.join()
            if not self.samples:
                self._sample()

    def summary(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ------------------------------------------------------------------------------- dist
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------- GPU arm
def make_inputs(cfg: wl.Config, device):
    act = cfg.activations()
    return act, [t.to(device) for t in (act.routing_logits, act.routing_bias,
                                         act.hidden_states, act.hidden_states_scale)]


def time_calls(inputs, weights, local_start, rsf, n, phase=True):
    """Runs n calls; returns (mean ms per call from one bracketing event pair,
    per-phase mean ms from the per-call phase events)."""
    lg, b, hs, sc = inputs
    w1, s1, w2, s2 = weights
    out = torch.empty((lg.shape[0], wl.HIDDEN), dtype=torch.bfloat16, device=lg.device)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(n)] if phase else None
    ptrs = []
    if phase:
        for row in evs:          # create the underlying cudaEvent_t handles
            for e in row:
                e.record()
        torch.cuda.synchronize()
        ptrs = [(ctypes_array(row)) for row in evs]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(n):
        launch(lg, b, hs, sc, w1, s1, w2, s2, local_start, rsf, out, ptrs[i] if phase else None)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / n
    phases = None
    if phase:
        acc = np.zeros(5)
        for row in evs:
            acc += [row[j].elapsed_time(row[j + 1]) for j in range(5)]
        phases = (acc / n).tolist()
    return ms, phases, out


def time_graph(inputs, weights, local_start, rsf, n, reps=3):
    """Mean ms per call of one CUDA graph of n calls (captured untimed), best of reps replays."""
    lg, b, hs, sc = inputs
    out = torch.empty((lg.shape[0], wl.HIDDEN), dtype=torch.bfloat16, device=lg.device)
    launch(lg, b, hs, sc, *weights, local_start, rsf, out, None)  # workspace allocated outside
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(lg.device)
    cap.wait_stream(torch.cuda.current_stream(lg.device))
    with torch.cuda.graph(g, stream=cap):
        for _ in range(n):
            launch(lg, b, hs, sc, *weights, local_start, rsf, out, None)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        g.replay()
        s1.record()
        torch.cuda.synchronize()
        best = min(best, s0.elapsed_time(s1) / n)
    del g
    return best


def ctypes_array(events):
    import ctypes
    arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
    return arr


def launch(lg, b, hs, sc, w1, s1, w2, s2, local_start, rsf, out, phase_ptrs):
    import ctypes
    device = hs.device
    T, e_local = lg.shape[0], w1.shape[0]
    ws, lay = fmoe.workspace_for(device, T, e_local, wl.HIDDEN, wl.INTER)
    a = _lib.FmoeArgs()
    a.routing_logits, a.logits_dtype = lg.data_ptr(), _lib.DTYPE_F32
    a.routing_bias, a.bias_dtype = b.data_ptr(), _lib.DTYPE_BF16
    a.hidden_states, a.hidden_states_scale = hs.data_ptr(), sc.data_ptr()
    a.gemm1_weights, a.gemm1_weights_scale = w1.data_ptr(), s1.data_ptr()
    a.gemm2_weights, a.gemm2_weights_scale = w2.data_ptr(), s2.data_ptr()
    a.output = out.data_ptr()
    a.num_tokens, a.hidden_size, a.intermediate_size = T, wl.HIDDEN, wl.INTER
    a.num_experts, a.num_local_experts, a.top_k, a.n_group, a.topk_group = 256, e_local, 8, 8, 4
    a.local_expert_offset, a.routed_scaling_factor = local_start, rsf
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    if phase_ptrs is not None:
        a.phase_events = ctypes.cast(phase_ptrs, ctypes.c_void_p)
        a.num_phase_events = len(phase_ptrs)
    rc = _lib.load().fmoe_run(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "fmoe_run")


def traffic_from_profiles(workload: str):
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p))
    return d.get(workload, {}).get("gemm1_dram_bytes")


def cpu_oracle_seconds(cfg: wl.Config, local_start: int, e_local: int, ntok: int):
    from oracle import moe as omoe
    from oracle import routing as orouting
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    ids, w = ids[:ntok], w[:ntok]
    active = sorted({int(e) - local_start for e in ids.reshape(-1)
                     if 0 <= int(e) - local_start < e_local})
    W1, S1, W2, S2 = {}, [np.zeros((32, 56), np.float32)] * e_local, {}, [np.zeros((56, 16), np.float32)] * e_local
    for le in active:
        q1, s1, q2, s2 = wl.WeightBank.get(local_start + le)
        W1[le], W2[le] = q1.view(torch.uint8).numpy(), q2.view(torch.uint8).numpy()
        S1[le], S2[le] = s1.numpy(), s2.numpy()
    hs = act.hidden_states.view(torch.uint8).numpy()[:ntok]
    sc = act.hidden_states_scale.numpy()[:, :ntok]
    t0 = time.perf_counter()
    omoe.moe_reference(hs, sc, W1, S1, W2, S2, ids, w, local_start)
    return time.perf_counter() - t0


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def quant_lines(device, peaks):
    """Input quantisation kernel (bf16 -> e4m3 + per-128 scales) at the decode and the largest
    prefill size: device time per call (CUDA events around 50 calls, inputs resident; at
    T=16384 the 352 MB per call exceed L2) against the measured HBM copy bandwidth."""
    rows = []
    for T in (64, 16384):
        g = torch.Generator().manual_seed(T)
        x = torch.randn(T, wl.HIDDEN, generator=g).to(torch.bfloat16).to(device)
        q = torch.empty((T, wl.HIDDEN), dtype=torch.uint8, device=device)
        sc = torch.empty((wl.HIDDEN // 128, T), dtype=torch.float32, device=device)
        lib = _lib.load()
        args = (ctypes.c_void_p(x.data_ptr()), T, wl.HIDDEN, ctypes.c_void_p(q.data_ptr()),
                ctypes.c_void_p(sc.data_ptr()),
                ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
        for _ in range(3):
            assert lib.fmoe_quantize_activations(*args) == 0
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 50
        s0.record()
        for _ in range(n):
            lib.fmoe_quantize_activations(*args)
        s1.record()
        torch.cuda.synchronize()
        us = s0.elapsed_time(s1) / n * 1e3
        nbytes = T * (2 * wl.HIDDEN + wl.HIDDEN + 4 * (wl.HIDDEN // 128))
        rows.append({"T": T, "us_per_call": round(us, 2), "bytes": nbytes,
                     "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                     "frac_hbm": round(nbytes / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 3)})
    return rows


def run_sweep(device, weights, peaks):
    rows = []
    fp8_peak = 2.0 * peaks["bf16_tflops"]
    for name, cfg in wl.CONFIGS.items():
        act, inp = make_inputs(cfg, device)
        from oracle import routing as orouting  # routing ids for accounting only
        ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
        acc = call_accounting(ids, 0, 32, cfg.T)
        time_calls(inp, weights, 0, cfg.rsf, 3, phase=False)
        ms_plain, _, _ = time_calls(inp, weights, 0, cfg.rsf, 20, phase=False)  # plain launches
        ms = time_graph(inp, weights, 0, cfg.rsf, 20)                           # CUDA graph
        _, ph, _ = time_calls(inp, weights, 0, cfg.rsf, 10)                     # phase breakdown
        us = ms * 1e3
        t_roof = max(acc["flops"] / (fp8_peak * 1e12), acc["bytes"] / (peaks["hbm_gbs"] * 1e9))
        rows.append({"config": name, "T": cfg.T, "P": acc["P"], "active_experts": acc["active_experts"],
                     "us_per_call": round(us, 2), "us_per_call_plain_launches": round(ms_plain * 1e3, 2),
                     "tflops": round(acc["flops"] / (ms * 1e-3) / 1e12, 2),
                     "hbm_tbs": round(acc["bytes"] / (ms * 1e-3) / 1e12, 3),
                     "roofline_us": round(t_roof * 1e6, 2), "roofline_frac": round(t_roof * 1e6 / us, 3),
                     "phase_us": [round(x * 1e3, 2) for x in ph]})
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="t64_s4")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="headline loop as plain launches instead of one CUDA graph of K calls")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="run warm-up calls plus one call of --workload on GPU 0 and exit "
                         "(the command the committed ncu summaries capture)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    if args.impl == "reference":
        return reference_arm(args)
    if args.profile:
        return profile_once(args)
    if args.workload in ("ep", "ep_hot"):
        return ep_arm(args)

    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local if world > 1 else 0)
    peaks = measured_peaks()
    base = wl.CONFIGS[args.workload]
    local_start = (32 * rank) % 256
    cfg = wl.Config(base.name, base.T, base.seed + rank, local_expert_offset=local_start)
    weights = tuple(t.to(device) for t in wl.local_weights(32, local_start))
    act, inp = make_inputs(cfg, device)
    from oracle import routing as orouting  # accounting of the workload's routed pairs
    ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    acc = call_accounting(ids, local_start, 32, cfg.T)

    # warm-up, then EXACTLY K timed steps bracketed by barrier + synchronize. The headline loop
    # records no events between kernels (an event between two kernels breaks the programmatic
    # dependent launch that overlaps their launch latency). By default the K calls are captured
    # once, untimed, into one CUDA graph (kernel nodes keep their programmatic-dependency edges),
    # and the timed region is one replay of it: K calls, no host launch overhead.
    time_calls(inp, weights, local_start, cfg.rsf, args.warmup, phase=False)
    out = torch.empty((cfg.T, wl.HIDDEN), dtype=torch.bfloat16, device=device)
    lg, b, hs, sc = inp
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device)
        cap.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                launch(lg, b, hs, sc, *weights, local_start, cfg.rsf, out, None)
        torch.cuda.synchronize()
        graph.replay()  # untimed: the first launch of a graph also uploads it to the device
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clocks:
        start.record()
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                launch(lg, b, hs, sc, *weights, local_start, cfg.rsf, out, None)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    del graph
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world)

    # instrumented loop (the same K steps, with CUDA events on the launching stream around every
    # phase): the GEMM1 launch duration for the roofline and the phase breakdown
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    for row in evs:
        for e in row:
            e.record()
    ptrs = [ctypes_array(row) for row in evs]
    barrier(world)
    torch.cuda.synchronize()
    for i in range(args.steps):
        launch(lg, b, hs, sc, *weights, local_start, cfg.rsf, out, ptrs[i])
    torch.cuda.synchronize()
    barrier(world)
    gemm1_ms_local = float(np.mean([r[2].elapsed_time(r[3]) for r in evs]))
    phases_local = np.mean([[r[j].elapsed_time(r[j + 1]) for j in range(5)] for r in evs], axis=0)
    gemm1_ms = max_over_ranks(gemm1_ms_local, world)

    # end to end through the public API with pinned host buffers, copies inside the timed region
    host_in = [t.pin_memory() for t in (act.routing_logits, act.routing_bias,
                                         act.hidden_states, act.hidden_states_scale)]
    host_out = torch.empty((cfg.T, wl.HIDDEN), dtype=torch.bfloat16).pin_memory()
    dev_in = [torch.empty_like(t, device=device) for t in host_in]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = host_out.numel() * host_out.element_size()

    def e2e_step():
        for d, h in zip(dev_in, host_in):
            d.copy_(h, non_blocking=True)
        o = fmoe.run(*dev_in, *weights, local_start, cfg.rsf, out)
        host_out.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        e2e_step()
    e2.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / args.steps, world)

    result = None
    if rank == 0:
        tokens = cfg.T * world
        gemm1_bytes = acc["gemm1_bytes"]
        achieved = gemm1_bytes / (gemm1_ms * 1e-3) / 1e9
        result = {
            "metric": METRIC, "value": round(tokens / (ms * 1e-3), 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "us_per_call": round(ms * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic (seeded; operator-definition shapes and distributions)",
            "config": {"workload": f"configs[1] decode T={cfg.T} seed {base.seed}+rank, 32 local "
                                   f"experts per GPU (offset 32*rank mod 256)",
                       "T_per_gpu": cfg.T, "hidden": wl.HIDDEN, "intermediate": wl.INTER,
                       "experts_global": 256, "experts_local": 32, "top_k": 8,
                       "P_rank0": acc["P"], "active_experts_rank0": acc["active_experts"],
                       "parallelism": f"expert-shard replicas x{world}",
                       "launch": ("plain launches" if args.no_graph else
                                  "one CUDA graph of the K calls (captured and first replayed "
                                  "untimed), timed over one replay"),
                       "l2": "inputs larger than L2: each call streams "
                             f"{acc['active_experts'] * wl.bytes_per_expert() / 1e6:.0f} MB of weights"},
            "roofline": {"kernel": "k_gemm<1> (GEMM1 + SwiGLU)", "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 3),
                         "peak_source": peaks["source"],
                         "algorithmic_bytes": gemm1_bytes,
                         "avg_launch_us": round(gemm1_ms * 1e3, 2),
                         "timing": "CUDA events around k_gemm<1> on the launching stream, "
                                   "K instrumented steps after the headline loop",
                         "traffic": traffic_from_profiles(args.workload)},
            "phase_us_rank0": dict(zip(["route+plan", "gather", "gemm1", "gemm2", "combine"],
                                       [round(x * 1e3, 2) for x in phases_local])),
            "call_roofline": {"flops": acc["flops"], "bytes": acc["bytes"],
                              "hbm_tbs": round(acc["bytes"] / (ms * 1e-3) / 1e12, 3),
                              "frac_hbm": round(acc["bytes"] / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)},
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms, 5)},
            "gpu_launches": kernels_per_call(cfg.T) * args.steps,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_sweep:
            result["sweep"] = run_sweep(device, weights, peaks)
            result["input_quantization"] = quant_lines(device, peaks)
        if world == 1 and not args.no_cpu_baseline:
            ntok = 8
            secs = min(cpu_oracle_seconds(cfg, local_start, 32, ntok) for _ in range(2))
            result["cpu_baseline"] = {"value": round(ntok / secs, 3), "unit": "tokens/s",
                                      "cores": blas_threads(), "kind": "port",
                                      "sample": f"first {ntok} tokens of the workload batch through "
                                                f"the numpy oracle (oracle/moe.py), best of 2"}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


def ep_arm(args):
    """global T=16384 tokens sharded evenly over N ranks, 256 experts sharded
    contiguously (256/N per rank), NCCL dispatch/combine (flashinfer_b200.ep); strong scaling."""
    from flashinfer_b200.ep import ExpertParallelMoE
    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local if world > 1 else 0)
    hot = 1.5 if args.workload == "ep_hot" else 0.0
    seed = 11 if hot else 10
    T_global = 16384
    per = T_global // world
    act = wl.make_activations(T_global, seed, hot_group=0 if hot else None, hot=hot)
    rows = slice(rank * per, (rank + 1) * per)
    host_in = [act.routing_logits[rows].contiguous(), act.routing_bias,
               act.hidden_states[rows].contiguous(),
               act.hidden_states_scale[:, rows].contiguous()]
    epr = 256 // world
    ws = [wl.expert_weights(e, device=str(device)) for e in range(rank * epr, (rank + 1) * epr)]
    weights = [torch.stack([w[i] for w in ws]) for i in range(4)]
    del ws
    inp = [t.to(device) for t in host_in]
    ep = ExpertParallelMoE()
    out = torch.empty((per, wl.HIDDEN), dtype=torch.bfloat16, device=device)
    for _ in range(args.warmup):
        ep.forward(*inp, *weights, wl.RSF_DEFAULT, out)
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clocks:
        start.record()
        for _ in range(args.steps):
            ep.forward(*inp, *weights, wl.RSF_DEFAULT, out)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    sent, recv = ep.last_counts
    # end to end: pinned host inputs in, bf16 rows out, every step
    pinned = [t.pin_memory() for t in host_in]
    host_out = torch.empty((per, wl.HIDDEN), dtype=torch.bfloat16).pin_memory()
    dev_in = [torch.empty_like(t, device=device) for t in pinned]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = host_out.numel() * host_out.element_size()

    def e2e_step():
        for d, h in zip(dev_in, pinned):
            d.copy_(h, non_blocking=True)
        ep.forward(*dev_in, *weights, wl.RSF_DEFAULT, out)
        host_out.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier(world)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        e2e_step()
    e2.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2) / args.steps, world)
    if rank == 0:
        from flashinfer_b200.ep import record_bytes
        print(json.dumps({
            "metric": METRIC, "value": round(T_global / (ms * 1e-3), 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "us_per_call": round(ms * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic (seeded activations; weights drawn on the GPU, same distributions)",
            "config": {"workload": f"configs[4] expert parallel, global T={T_global}, "
                                   f"{'hot group 0 (+1.5)' if hot else 'uniform'} logits, seed {seed}",
                       "experts_per_gpu": epr, "tokens_per_gpu": per,
                       "parallelism": f"ep{world} (NCCL all-to-all dispatch + combine)",
                       "dispatch_records_rank0": sum(sent),
                       "dispatch_bytes_rank0": sum(sent) * record_bytes(wl.HIDDEN),
                       "combine_bytes_rank0": sum(sent) * wl.HIDDEN * 4,
                       "received_tokens_rank0": sum(recv)},
            "e2e": {"value": round(T_global / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "ms_per_step": round(e2e_ms, 4)},
            "clocks": clocks.summary(),
        }), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def profile_once(args):
    device = torch.device("cuda", 0)
    cfg = wl.CONFIGS[args.workload]
    weights = tuple(t.to(device) for t in wl.local_weights(32, 0))
    _, inp = make_inputs(cfg, device)
    time_calls(inp, weights, 0, cfg.rsf, args.warmup + 1, phase=False)
    torch.cuda.synchronize()


def reference_arm(args):
    """CPU restatement of the reference algorithm (the oracle port) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = wl.CONFIGS[args.workload]
    ntok = 8
    for _ in range(min(args.warmup, 1)):
        cpu_oracle_seconds(cfg, 0, 32, ntok)
    t = [cpu_oracle_seconds(cfg, 0, 32, ntok) for _ in range(max(1, min(args.steps, 5)))]
    value = ntok / float(np.mean(t))
    cores = blas_threads()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": len(t), "warmup": args.warmup,
        "ms_per_step": round(float(np.mean(t)) * 1e3, 2), "higher_is_better": True,
        "dtype": "f32", "data": "synthetic", "vs_baseline": None,
        "config": {"workload": f"configs[1] decode T={cfg.T} seed {cfg.seed}, 32 local experts"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"first {ntok} tokens of the T={cfg.T} batch per step (numpy "
                                   f"restatement of the reference's fp32 expert loop)"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
