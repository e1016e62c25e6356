"""Benchmark of the fused FP8 block-scale MoE (DeepSeek-V3 routing) on B200.

One step = one call of the operator on one batch of synthetic input (seeded, the shapes and
distributions of the operator definition; no dataset is available offline). The headline is the
expert-parallel workload of the operator's benchmark plan: a global batch of
T=16384 tokens (uniform N(0,1) logits, seed 10) over all 256 experts, split over the N GPUs --
N ranks of 16384/N tokens and 256/N experts each, tokens and partial outputs moved between the
GPUs by the peer transport of ``flashinfer_b200.ep`` (stores into the other GPUs' memory over
NVLink). At N=1 the same global batch runs on one GPU with all 256 experts local, so the values
at N = 1, 2, 4, 8 form a strong-scaling curve. The hot-group variant (+1.5 on group 0, seed 11)
is timed as an extra key, and at N=1 the single-GPU configurations (configs[0-3]), the input
quantisation, the reference's own Triton operator and the measured FP8 tensor peak are added.

Prints ONE JSON line on rank 0. ``--impl reference`` times the reference algorithm's CPU
restatement (the oracle port: the reference itself is Triton-only) on the host cores, on a
bounded sample of the same workload. ``--workload <config>`` times one single-GPU configuration
of the benchmark plan instead (the command the committed ncu summaries profile).
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

T_EP = 16384            # configs[4] global batch
EP_WORKLOADS = {"ep": ("uniform logits", 10, 0.0), "ep_hot": ("hot group 0 (+1.5)", 11, 1.5)}

METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
SMALL_T = 64           # T <= SMALL_T: fused route/plan/scatter cluster kernel
SPLIT_MAX_T = 8        # T <= SPLIT_MAX_T: split-K finish kernel after each GEMM
GEMV_MAX_T = _lib.GEMV_MAX_T  # T <= GEMV_MAX_T: plan kernel + two matrix-vector kernels


def kernels_per_call(T: int) -> int:
    """Launches of one call: route+hist, scan, scatter, gather, gemm1, gemm2, combine; for
    T <= SMALL_T the fused plan kernel replaces the first three, for T <= SPLIT_MAX_T a split-K
    finish kernel follows each GEMM, and for T <= GEMV_MAX_T the call is the plan kernel and the
    two matrix-vector kernels."""
    if T <= GEMV_MAX_T:
        return 3
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
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
def max_vec_over_ranks(x, world: int):
    if world == 1:
        return [float(v) for v in x]
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


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


def time_graph(inputs, weights, local_start, rsf, n, reps=5):
    """Per-replay mean ms per call of one CUDA graph of n calls (captured and first replayed
    untimed), for each of `reps` replays."""
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
    times = []
    for _ in range(reps):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        g.replay()
        s1.record()
        torch.cuda.synchronize()
        times.append(s0.elapsed_time(s1) / n)
    del g
    return times


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


def cpu_oracle_seconds(act: wl.Activations, rsf: float, tokens, local_start: int = 0,
                       e_local: int = 256):
    """Seconds the numpy oracle (the reference's fp32 algorithm) takes for the given tokens of a
    batch, with experts [local_start, local_start + e_local) local; weights drawn beforehand."""
    from oracle import moe as omoe
    from oracle import routing as orouting
    tokens = np.asarray(tokens)
    ids, w = orouting.route(act.routing_logits.numpy()[tokens], act.routing_bias.float().numpy(),
                            rsf)
    need = sorted({int(e) for e in ids.reshape(-1) if local_start <= int(e) < local_start + e_local})

    class Scales(dict):
        def __len__(self):
            return e_local

    W1, S1, W2, S2 = {}, Scales(), {}, Scales()
    for e in need:
        q1, s1, q2, s2 = wl.WeightBank.get(e)
        W1[e - local_start], W2[e - local_start] = q1.view(torch.uint8).numpy(), q2.view(torch.uint8).numpy()
        S1[e - local_start], S2[e - local_start] = s1.numpy(), s2.numpy()
    hs = act.hidden_states.view(torch.uint8).numpy()[tokens]
    sc = act.hidden_states_scale.numpy()[:, tokens]
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


def run_sweep(device, weights, peaks, fp8_peak):
    """Every single-GPU configuration of the benchmark plan: median (and best) of 5 replays of one
    CUDA graph of 20 calls, the SM clock sampled during the replays, a plain-launch loop and the
    phase breakdown beside it."""
    rows = []
    for name, cfg in wl.CONFIGS.items():
        act, inp = make_inputs(cfg, device)
        from oracle import routing as orouting  # routing ids for accounting only
        ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
        acc = call_accounting(ids, 0, 32, cfg.T)
        time_calls(inp, weights, 0, cfg.rsf, 3, phase=False)
        ms_plain, _, _ = time_calls(inp, weights, 0, cfg.rsf, 20, phase=False)  # plain launches
        with ClockSampler(device.index or 0) as clk:
            times = time_graph(inp, weights, 0, cfg.rsf, 20)                    # CUDA graph
        _, ph, _ = time_calls(inp, weights, 0, cfg.rsf, 10)                     # phase breakdown
        ms = statistics.median(times)
        us = ms * 1e3
        t_roof = max(acc["flops"] / (fp8_peak * 1e12), acc["bytes"] / (peaks["hbm_gbs"] * 1e9))
        c = clk.summary()
        rows.append({"config": name, "T": cfg.T, "P": acc["P"], "active_experts": acc["active_experts"],
                     "us_per_call": round(us, 2), "us_per_call_best": round(min(times) * 1e3, 2),
                     "us_per_call_plain_launches": round(ms_plain * 1e3, 2),
                     "tflops": round(acc["flops"] / (ms * 1e-3) / 1e12, 2),
                     "hbm_tbs": round(acc["bytes"] / (ms * 1e-3) / 1e12, 3),
                     "roofline_us": round(t_roof * 1e6, 2), "roofline_frac": round(t_roof * 1e6 / us, 3),
                     "phase_us": [round(x * 1e3, 2) for x in ph],
                     "sm_mhz": c.get("sm_mhz"), "clock_reasons": c.get("reasons")})
    return rows


def fp8_peak(device):
    """Dense FP8 tensor rate of this GPU with the GEMMs' MMA (fmoe_fp8_mma_peak): a ~10 ms burst
    and a ~1 s sustained run (clocks settle under the power cap), TFLOP/s."""
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=device)
    flops = ctypes.c_double()
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)

    def run(kb, n):
        _lib.check(lib.fmoe_fp8_mma_peak(kb, ctypes.c_void_p(status.data_ptr()),
                                         ctypes.byref(flops), stream), "fmoe_fp8_mma_peak")
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(n):
            lib.fmoe_fp8_mma_peak(kb, ctypes.c_void_p(status.data_ptr()), ctypes.byref(flops),
                                  stream)
        s1.record()
        torch.cuda.synchronize()
        return flops.value * n / (s0.elapsed_time(s1) * 1e-3) / 1e12

    burst = max(run(30000, 1) for _ in range(3))
    with ClockSampler(device.index or 0) as clk:
        sustained = run(400000, 6)
    assert int(status.item()) == 0, "fp8 peak kernel: a bounded wait ran out"
    c = clk.summary()
    return {"burst_tflops": round(burst, 1), "sustained_tflops": round(sustained, 1),
            "sustained_sm_mhz": c.get("sm_mhz"), "sustained_reasons": c.get("reasons"),
            "kernel": "fmoe_fp8_mma_peak: one CTA per SM, tcgen05.mma kind::f8f6f4 M128 N256 K32 "
                      "chains from shared memory (the GEMMs' instruction), no memory traffic"}


def triton_reference(device, weights, names, our_rows):
    """The reference's own GPU operator (solution/triton/kernel.py::run, installed unmodified in
    baseline/_ref) on the same seeded inputs as ours: CUDA-event time per call (3 warm-up calls,
    then 20 timed, median of 3 loops; the reference synchronises the host inside each call) and
    its output against ours."""
    path = os.path.join(ROOT, "baseline", "_ref", "solution", "triton", "kernel.py")
    if not os.path.exists(path):
        return {"unavailable": "baseline/_ref not installed (baseline/install_ref.sh)"}
    import importlib.util
    spec = importlib.util.spec_from_file_location("reference_triton_kernel", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ours = {r["config"]: r for r in our_rows}
    rows = []
    for name in names:
        cfg = wl.CONFIGS[name]
        act, inp = make_inputs(cfg, device)
        out_ref = torch.empty((cfg.T, wl.HIDDEN), dtype=torch.bfloat16, device=device)
        try:
            for _ in range(3):
                mod.run(*inp, *weights, 0, cfg.rsf, out_ref)
            torch.cuda.synchronize()
            loops = []
            for _ in range(3):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                for _ in range(20):
                    mod.run(*inp, *weights, 0, cfg.rsf, out_ref)
                s1.record()
                torch.cuda.synchronize()
                loops.append(s0.elapsed_time(s1) / 20)
        except Exception as e:  # report, do not hide: the line says why
            rows.append({"config": name, "error": f"{type(e).__name__}: {e}"[:300]})
            continue
        ours_out = fmoe.run(*inp, *weights, 0, cfg.rsf)
        torch.cuda.synchronize()
        diff = (ours_out.float() - out_ref.float()).abs()
        tol = 1e-2 + 1e-2 * out_ref.float().abs()
        us = statistics.median(loops) * 1e3
        row = {"config": name, "T": cfg.T, "triton_us_per_call": round(us, 1),
               "max_abs_diff_vs_ours": round(float(diff.max()), 5),
               "frac_within_1e-2_of_ours": round(float((diff <= tol).float().mean()), 6)}
        if name in ours:
            row["ours_us_per_call"] = ours[name]["us_per_call"]
            row["speedup_vs_triton"] = round(us / ours[name]["us_per_call"], 2)
        rows.append(row)
    return rows


# ------------------------------------------------------------------------------- headline
def ep_inputs(name: str, world: int, rank: int, device):
    """This rank's slice of the configs[4] global batch (CPU activations -> device)."""
    _, seed, hot = EP_WORKLOADS[name]
    act = wl.make_activations(T_EP, seed, hot_group=0 if hot else None, hot=hot)
    per = T_EP // world
    rows = slice(rank * per, (rank + 1) * per)
    host = [act.routing_logits[rows].contiguous(), act.routing_bias,
            act.hidden_states[rows].contiguous(), act.hidden_states_scale[:, rows].contiguous()]
    return act, host, [t.to(device) for t in host]


def ep_forward_fn(ep, world, weights, rsf):
    """One step of the layer on this rank: through the expert-parallel layer for N > 1, the
    operator itself (all 256 experts local, phase events available) for N = 1."""
    def step(inp, out, phase_ptrs=None):
        if world == 1:
            launch(*inp, *weights, 0, rsf, out, phase_ptrs)
        else:
            ep.forward(*inp, *weights, rsf, out)
    return step


def time_steps(step, inp, out, n, world):
    barrier(world)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(n):
        step(inp, out)
    s1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(s0.elapsed_time(s1) / n, world)


def ep_arm(args):
    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local if world > 1 else 0)
    peaks = measured_peaks()
    per = T_EP // world
    epr = 256 // world
    rsf = wl.RSF_DEFAULT
    # this rank's experts, drawn on the device (same distributions as the CPU draws; timing only)
    ws = [wl.expert_weights(e, device=str(device)) for e in range(rank * epr, (rank + 1) * epr)]
    weights = tuple(torch.stack([w[i] for w in ws]) for i in range(4))
    del ws
    from flashinfer_b200.ep import ExpertParallelMoE
    ep = ExpertParallelMoE(capacity=per) if world > 1 else None
    step = ep_forward_fn(ep, world, weights, rsf)
    act, host_in, inp = ep_inputs(args.workload, world, rank, device)
    out = torch.empty((per, wl.HIDDEN), dtype=torch.bfloat16, device=device)

    # warm-up, then EXACTLY K timed steps bracketed by barrier + synchronize, max over ranks
    for _ in range(args.warmup):
        step(inp, out)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index or 0) as clocks:
        start.record()
        for _ in range(args.steps):
            step(inp, out)
        end.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)

    # instrumented loop (the same K steps with CUDA events between the phases, on the launching
    # stream): the phase breakdown and the GEMM1 launch duration for the roofline
    n_loc = 6
    loc_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_loc)] for _ in range(args.steps)]
    ep_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]
    for row in loc_ev + ep_ev:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    barrier(world)
    for i in range(args.steps):
        if world == 1:
            step(inp, out, ctypes_array(loc_ev[i]))
        else:
            ep.phase_events, ep.local_phase_events = ep_ev[i], loc_ev[i]
            step(inp, out)
    torch.cuda.synchronize()
    if ep is not None:
        ep.phase_events = ep.local_phase_events = None
    barrier(world)
    loc = np.mean([[r[j].elapsed_time(r[j + 1]) for j in range(5)] for r in loc_ev], axis=0)
    loc_max = max_vec_over_ranks(loc, world)
    ep_ph = None
    if world > 1:
        ep_ph = max_vec_over_ranks(np.mean([[r[j].elapsed_time(r[j + 1]) for j in range(6)]
                                            for r in ep_ev], axis=0), world)
    gemm1_ms_local = float(loc[2])
    received = ep.counts() if ep is not None else [per]

    # routed pairs of every rank's experts (accounting): the global routing, on the CPU
    from oracle import routing as orouting
    ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), rsf)
    pairs_per_rank = np.bincount(ids.reshape(-1) // epr, minlength=world)
    gemm1_flops_rank = int(pairs_per_rank[rank]) * 2 * wl.HIDDEN * 2 * wl.INTER
    gemm1_tflops_local = gemm1_flops_rank / (gemm1_ms_local * 1e-3) / 1e12
    gemm1_tflops_min = -max_over_ranks(-gemm1_tflops_local, world)

    # hot-group variant (extra key): the same layer on the other logits distribution
    other = "ep_hot" if args.workload == "ep" else "ep"
    _, _, inp_o = ep_inputs(other, world, rank, device)
    for _ in range(args.warmup):
        step(inp_o, out)
    ms_other = time_steps(step, inp_o, out, args.steps, world)
    del inp_o

    # end to end through the public API: pinned host inputs in, bf16 rows out, every step
    pinned = [t.pin_memory() for t in host_in]
    host_out = torch.empty((per, wl.HIDDEN), dtype=torch.bfloat16).pin_memory()
    dev_in = [torch.empty_like(t, device=device) for t in pinned]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = host_out.numel() * host_out.element_size()

    def e2e_step():
        for d, h in zip(dev_in, pinned):
            d.copy_(h, non_blocking=True)
        if world == 1:
            fmoe.run(*dev_in, *weights, 0, rsf, out)
        else:
            ep.forward(*dev_in, *weights, rsf, out)
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

    result = None
    if rank == 0:
        fp8 = fp8_peak(device)
        fp8_peak_sus = fp8["sustained_tflops"]
        flops = int(ids.size) * wl.flops_per_pair()
        nbytes = 256 * wl.bytes_per_expert() + T_EP * wl.bytes_per_token() + 512
        # our kernels per step and rank: N=1 -- route, histogram (256 local experts: routing over
        # every SM, then the per-block counts), scan, scatter, gather, GEMM1, GEMM2, combine;
        # N>1 -- route, dispatch plan + send, the pre-routed operator's 7, reduce
        launches = (8 if world == 1 else 11) * args.steps * world
        result = {
            "metric": METRIC, "value": round(T_EP / (ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "us_per_call": round(ms * 1e3, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic (seeded activations of the operator definition; weights drawn on "
                    "the GPU from the same distributions)",
            "config": {
                "workload": f"configs[4] expert parallel: global T={T_EP} "
                            f"({EP_WORKLOADS[args.workload][0]}, seed {EP_WORKLOADS[args.workload][1]}), "
                            f"256 experts over {world} GPU(s)",
                "tokens_per_gpu": per, "experts_per_gpu": epr, "hidden": wl.HIDDEN,
                "intermediate": wl.INTER, "top_k": 8,
                "parallelism": (f"ep{world}: tokens and partial rows moved by stores into the "
                                f"other GPUs' memory over NVLink (CUDA IPC), NCCL all-reduce "
                                f"barriers" if world > 1 else
                                "1 GPU, all 256 experts local (no collectives)"),
                "pairs_per_gpu": [int(x) for x in pairs_per_rank],
                "received_tokens_rank0": [int(x) for x in received],
                "launch": "plain launches",
                "l2": f"inputs larger than L2: each step streams {nbytes / 1e9:.1f} GB of weights "
                      f"over the GPUs"},
            "phase_us": ({k: round(v * 1e3, 1) for k, v in zip(
                ["route", "dispatch", "barrier_1", "local_moe", "barrier_2", "reduce"], ep_ph)}
                if ep_ph is not None else None),
            "local_phase_us_max_over_ranks": {k: round(v * 1e3, 1) for k, v in zip(
                ["route+plan", "gather", "gemm1", "gemm2", "combine"], loc_max)},
            "roofline": {"kernel": "k_gemm<1> (GEMM1 + SwiGLU)", "bound": "tensor",
                         "achieved": round(gemm1_tflops_local, 1), "peak": fp8_peak_sus,
                         "unit": "TFLOP/s", "frac": round(gemm1_tflops_local / fp8_peak_sus, 3),
                         "peak_source": "measured: sustained FP8 MMA rate of this GPU "
                                        "(fmoe_fp8_mma_peak, ~1 s under the power cap)",
                         "algorithmic_flops": gemm1_flops_rank,
                         "avg_launch_us": round(gemm1_ms_local * 1e3, 1),
                         "slowest_rank_tflops": round(gemm1_tflops_min, 1),
                         "timing": "CUDA events around k_gemm<1> on the launching stream, rank 0, "
                                   "K instrumented steps after the headline loop",
                         "traffic": traffic_from_profiles("ep_gemm1")},
            "call_roofline": {"flops": flops, "bytes": nbytes,
                              "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                              "frac_fp8_sustained_x_gpus": round(
                                  flops / (ms * 1e-3) / 1e12 / (fp8_peak_sus * world), 3)},
            "fp8_peak": fp8,
            "other_workload": {"workload": other, "value": round(T_EP / (ms_other * 1e-3), 1),
                               "unit": "tokens/s", "ms_per_step": round(ms_other, 4)},
            "e2e": {"value": round(T_EP / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_sweep:
            dev_w = tuple(t[:32].contiguous() for t in weights)  # experts 0..31 (GPU draws)
            result["sweep"] = run_sweep(device, dev_w, peaks, fp8_peak_sus)
            result["input_quantization"] = quant_lines(device, peaks)
            if not args.no_triton:
                result["triton_reference"] = triton_reference(
                    device, dev_w, ["t1_s1", "t16_s0", "t64_s4", "t256_s5", "t1024_s6",
                                    "t4096_s7", "t16384_s9"], result["sweep"])
        if world == 1 and not args.no_cpu_baseline:
            tok = [0, T_EP // 2]
            secs = min(cpu_oracle_seconds(act, rsf, tok) for _ in range(2))
            result["cpu_baseline"] = {"value": round(len(tok) / secs, 4), "unit": "tokens/s",
                                      "cores": blas_threads(), "kind": "port",
                                      "sample": f"{len(tok)} tokens of the global batch over all "
                                                f"256 experts through the numpy oracle "
                                                f"(oracle/moe.py), best of 2"}
    if ep is not None:
        ep.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)


# ------------------------------------------------------------------------------- one config
def config_arm(args):
    """One single-GPU configuration of the benchmark plan (--workload <config>), 32 local
    experts: graph-replayed K calls, phase breakdown and GEMM1 roofline."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    peaks = measured_peaks()
    cfg = wl.CONFIGS[args.workload]
    weights = tuple(t.to(device) for t in wl.local_weights(32, 0))
    act, inp = make_inputs(cfg, device)
    from oracle import routing as orouting
    ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    acc = call_accounting(ids, 0, 32, cfg.T)
    time_calls(inp, weights, 0, cfg.rsf, args.warmup, phase=False)
    with ClockSampler(0) as clocks:
        times = time_graph(inp, weights, 0, cfg.rsf, args.steps, reps=1)
    ms = times[0]
    _, ph, _ = time_calls(inp, weights, 0, cfg.rsf, args.steps)
    gemm1_ms = ph[2]
    achieved = acc["gemm1_bytes"] / (gemm1_ms * 1e-3) / 1e9
    print(json.dumps({
        "metric": METRIC, "value": round(cfg.T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "us_per_call": round(ms * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3", "data": "synthetic",
        "config": {"workload": f"{cfg.name}: T={cfg.T}, 32 local experts", "P": acc["P"],
                   "active_experts": acc["active_experts"],
                   "launch": "one CUDA graph of the K calls, one replay timed"},
        "phase_us": dict(zip(["route+plan", "gather", "gemm1", "gemm2", "combine"],
                             [round(x * 1e3, 2) for x in ph])),
        "roofline": {"kernel": "k_gemm<1>", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 3),
                     "traffic": traffic_from_profiles(args.workload)},
        "gpu_launches": kernels_per_call(cfg.T) * args.steps,
        "clocks": clocks.summary()}), flush=True)


def profile_once(args):
    """Warm-up calls plus one call of --workload on GPU 0 (the command the committed ncu
    summaries capture); an expert-parallel workload runs at N=1 (all 256 experts local)."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    if args.workload.startswith("quant_t"):
        # input quantisation (fmoe_quantize_activations) of a seeded bf16 batch of T tokens
        T = int(args.workload[len("quant_t"):])
        g = torch.Generator().manual_seed(T)
        x = torch.randn(T, wl.HIDDEN, generator=g).to(torch.bfloat16).to(device)
        for _ in range(args.warmup + 1):
            fmoe.quantize_activations(x)
        torch.cuda.synchronize()
        return
    if args.workload == "ep_dispatch":
        # the expert-parallel data plane at full width on one GPU: 2 ranks of the configs[4] batch
        # emulated as 2 buffers of this GPU (route, dispatch into both, reduce from both); the
        # partial rows the reduction reads are whatever the buffers hold (traffic, not values)
        world, per = 2, T_EP // 2
        lay = _lib.ep_layout(world, per, wl.HIDDEN)
        bufs = [torch.zeros(lay.total_bytes, dtype=torch.uint8, device=device) for _ in range(world)]
        peers = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
        act, _, _ = ep_inputs("ep", 1, 0, torch.device("cpu"))
        lib = _lib.load()
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        ranks = []
        for r in range(world):
            rows = slice(r * per, (r + 1) * per)
            ranks.append([t.to(device) for t in (act.routing_logits[rows].contiguous(),
                                                 act.routing_bias,
                                                 act.hidden_states[rows].contiguous(),
                                                 act.hidden_states_scale[:, rows].contiguous())])
        tds = [torch.empty((per, world), dtype=torch.int32, device=device) for _ in range(world)]
        outs = [torch.empty((per, wl.HIDDEN), dtype=torch.bfloat16, device=device)
                for _ in range(world)]
        for _ in range(args.warmup + 1):
            for r in range(world):
                lg, b, hs, sc = ranks[r]
                ids, w = fmoe.route(lg, b, wl.RSF_DEFAULT)
                _lib.check(lib.fmoe_ep_dispatch(p(ids), p(w), p(hs), p(sc), per, per, wl.HIDDEN,
                                                world, r, peers, p(tds[r]), stream), "dispatch")
            for r in range(world):
                _lib.check(lib.fmoe_ep_reduce(p(tds[r]), p(bufs[r]), per, per, wl.HIDDEN, world,
                                              p(outs[r]), stream), "reduce")
        torch.cuda.synchronize()
        return
    if args.workload in EP_WORKLOADS:
        ws = [wl.expert_weights(e, device="cuda") for e in range(256)]
        weights = tuple(torch.stack([w[i] for w in ws]) for i in range(4))
        del ws
        _, _, inp = ep_inputs(args.workload, 1, 0, device)
        out = torch.empty((T_EP, wl.HIDDEN), dtype=torch.bfloat16, device=device)
        for _ in range(args.warmup + 1):
            launch(*inp, *weights, 0, wl.RSF_DEFAULT, out, None)
        torch.cuda.synchronize()
        return
    cfg = wl.CONFIGS[args.workload]
    weights = tuple(t.to(device) for t in wl.local_weights(32, 0))
    _, inp = make_inputs(cfg, device)
    time_calls(inp, weights, 0, cfg.rsf, args.warmup + 1, phase=False)
    torch.cuda.synchronize()


def reference_arm(args):
    """The reference algorithm on the host cores: its CPU restatement (the oracle port; the
    reference itself is Triton-only) on a bounded sample of the headline workload per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    name = args.workload if args.workload in EP_WORKLOADS else "ep"
    act, _, _ = ep_inputs(name, 1, 0, torch.device("cpu"))
    tok = [0, T_EP // 2]
    cpu_oracle_seconds(act, wl.RSF_DEFAULT, tok[:1])  # draws the weights, warms the BLAS
    t = [cpu_oracle_seconds(act, wl.RSF_DEFAULT, tok) for _ in range(max(1, min(args.steps, 3)))]
    value = len(tok) / float(np.mean(t))
    cores = blas_threads()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tokens/s",
        "n_gpus": world, "steps": len(t), "warmup": args.warmup,
        "ms_per_step": round(float(np.mean(t)) * 1e3, 2), "higher_is_better": True,
        "dtype": "f32", "data": "synthetic", "vs_baseline": None,
        "config": {"workload": f"configs[4] expert parallel: global T={T_EP} "
                               f"({EP_WORKLOADS[name][0]}, seed {EP_WORKLOADS[name][1]}), "
                               f"256 experts"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": cores,
                         "kind": "port",
                         "sample": f"{len(tok)} tokens of the global batch per step over all 256 "
                                   f"experts (numpy restatement of the reference's fp32 expert "
                                   f"loop, oracle/moe.py)"},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="ep",
                    help="ep (configs[4], the headline) | ep_hot | one of the single-GPU configs "
                         "| quant_t<T> | ep_dispatch (--profile only: the input quantisation "
                         "kernel; the expert-parallel dispatch and reduction on one GPU)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-triton", action="store_true")
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
    if args.workload in EP_WORKLOADS:
        return ep_arm(args)
    return config_arm(args)


if __name__ == "__main__":
    main()
