"""Benchmark of the ternary i2_s path on B200: one JSON line on rank 0.

Workload (a "step"): the BitNet-b1.58-2B-shape FFN block at prefill M=300 tokens --
RMSNorm(2560, eps 1e-5) -> ternary gate/up 2560->6912 -> squared-ReLU gate product -> RMSNorm(6912) ->
ternary down 6912->2560 -- i.e. three i2_s mul_mats (31.85 G ternary int ops) plus their fused
neighbours, on seeded synthetic inputs (weights ternary P(0)=0.4, one scale U(0.5,2) per matrix;
activations N(0,1); norm weights N(1,0.1)). There are no checkpoints here; the inputs are random-init.

  value   = whole-job ternary int-op throughput (TOP/s) with inputs resident in HBM: each step replays a
            CUDA graph of one b2s_ffn_block call (four kernels) over one of 16 rotating weight/activation
            sets (~261 MB, more than twice the 126 MB L2, so weights stream from HBM as they would across
            30 layers).
  e2e     = the same metric through the public C ABI call b2s_ffn_block, with the step's activations
            copied host->device from pinned memory and the output copied back, inside the timed region;
            consecutive steps are pipelined over three streams (copies of neighbouring steps overlap the
            FFN block), as a server streaming batches would run them.
  roofline= the gate/up tensor-core GEMM (the dominant kernel), timed with CUDA events around its launch in
            replays of the same step issued as four calls, against the measured tensor peak.
  cpu_baseline = the threaded SIMD port of the oracle on the host cores (rank 0, N=1 only).

--impl reference times the reference's CPU implementation of the path. The reference's own i2_s CPU
kernels (BitNet's ggml fork) are not in the reference tree, so this is the oracle port, with all host
threads, on the same workload.

Multi-GPU: one process per GPU (torchrun); the FFN block batches are independent (data parallel, no
collective on the data path); timing is the max over ranks; scaling "weak".

--workload bitvla: the batched model-server run -- 64 independent random-init BitVLA-shape observations
(224x224 image + 32 text tokens each; 27-layer ternary ViT, connector, 30-layer ternary decoder prefill of
288 tokens) sharded data parallel over the ranks with no collective (strong scaling: the 64 observations
are the whole job). Each rank runs its share as forwards of --obs-batch observations through the
library's graph-captured engine. value = observations/s of the whole job; p50 latency = median forward
time of one batch (every observation in it waits that long); e2e = the same through b2s_bitvla_predict
(uint8 host images in, host actions out).

--workload sweep: the i2_s GEMM roofline sweep, M in {1, 16, 256, 4096, 16384} x (K,N) in {(2560,2560),
(2560,6912), (6912,2560), (1152,4304)} on pre-quantized int8 activations. Each point replays a CUDA graph
of back-to-back launches over rotating weight copies (> 2x L2 of weights per pass), so weights stream
from HBM; it reports TOP/s and algorithmic GB/s per launch against the measured peaks (HBM-bound for
M <= 16, tensor-bound from M = 256).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "robot.cpp_b200"))

METRIC = "ternary GEMM int8 TOPS & HBM GB/s vs roofline; BitVLA obs/sec @1/2/4/8 GPU"
M, H, F, EPS = 300, 2560, 6912, 1e-5
OPS_PER_STEP = 2 * M * F * H * 2 + 2 * M * H * F  # gate + up + down = 31.85e9
GATE_UP_OPS = 2 * 2 * M * F * H
N_SETS = 16


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 2000 FFN blocks; 10 BitVLA jobs of --observations each)")
    p.add_argument("--warmup", type=int, default=None, help="untimed warm-up steps (default: 20 FFN, 3 BitVLA)")
    p.add_argument("--impl", default="b2s", choices=["b2s", "reference"])
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="bounded CPU-baseline sample length")
    p.add_argument("--workload", default="ffn", choices=["ffn", "bitvla", "sweep"])
    p.add_argument("--observations", type=int, default=64, help="bitvla: observations in the whole job")
    p.add_argument("--obs-batch", type=int, default=8, help="bitvla: observations per forward")
    p.add_argument("--sweep-m", default="", help="sweep: comma-separated M values (default: all five)")
    a = p.parse_args()
    if a.steps is None:
        a.steps = 10 if a.workload == "bitvla" else 2000
    if a.warmup is None:
        a.warmup = 3 if a.workload == "bitvla" else 20
    return a


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ------------------------------------------------------------------------------------------- CPU leg
def cpu_ffn_sample(seconds: float, nthreads: int):
    """Times the oracle's threaded port on full FFN blocks for about `seconds` (>= 2 iterations)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    from b2s import workloads as wl
    f = wl.ffn_block(seed=1, M=M, H=H, F=F, eps=EPS)
    args = (f.x, f.g1, f.g2, f.eps, f.w_gate.packed, f.w_up.packed, f.w_down.packed, f.H, f.F, nthreads)
    oracle.fast_ffn_block(*args)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.fast_ffn_block(*args)
        n += 1
        dt = time.perf_counter() - t0
        if n >= 2 and dt >= seconds:
            break
    return n, dt


def run_reference(a, world, rank):
    if rank != 0:
        return
    nthreads = cpu_threads()
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from b2s import workloads as wl
    f = wl.ffn_block(seed=1, M=M, H=H, F=F, eps=EPS)
    args = (f.x, f.g1, f.g2, f.eps, f.w_gate.packed, f.w_up.packed, f.w_down.packed, f.H, f.F, nthreads)
    for _ in range(max(1, min(a.warmup, 3))):
        oracle.fast_ffn_block(*args)
    # Each step is one full FFN block; cap the number of timed steps so the run stays within minutes.
    t_one0 = time.perf_counter()
    oracle.fast_ffn_block(*args)
    t_one = time.perf_counter() - t_one0
    steps = max(1, min(a.steps, int(120.0 / max(t_one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.fast_ffn_block(*args)
    dt = time.perf_counter() - t0
    value = steps * OPS_PER_STEP / dt / 1e12
    sample = (f"{steps} full FFN blocks (M={M}, H={H}, F={F}) on {nthreads} threads, "
              f"{['scalar', 'AVX2', 'AVX512-VNNI'][oracle.fast_isa()]}; {cpu_model()}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TOP/s",
        "n_gpus": world, "steps": steps, "warmup": a.warmup, "ms_per_step": round(dt / steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xternary->int32",
        "data": "synthetic (seeded random-init ternary weights, N(0,1) activations)",
        "config": {"workload": "ffn_block_bitnet2b_m300", "M": M, "hidden": H, "ffn": F,
                   "parallelism": "host threads", "l2": "CPU"},
        "cpu_baseline": {"value": round(value, 6), "unit": "TOP/s", "cores": nthreads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.period, self._stop, self._t = period_s, threading.Event(), None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                bits = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b and b != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------- GPU leg
def run_b2s(a, world, rank, local):
    import numpy as np
    import torch
    import b2s
    from b2s import workloads as wl

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2s.lib()
    b2s.check(b2s.lib().b2s_device_check())
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    # ---- inputs: set 0 from the seeded host generator; sets 1..15 are byte rotations of it on device
    f = wl.ffn_block(seed=1 + rank, M=M, H=H, F=F, eps=EPS)
    base = {k: torch.from_numpy(getattr(f, k).packed).to(dev) for k in ("w_gate", "w_up", "w_down")}
    dims = {"w_gate": (F, H), "w_up": (F, H), "w_down": (H, F)}
    sets = []
    x0 = torch.from_numpy(f.x).to(dev)
    for i in range(N_SETS):
        ws = {}
        for k, buf in base.items():
            nb = buf.numel() - 32
            b = buf.clone()
            if i:
                b[:nb] = torch.roll(buf[:nb], shifts=i * 4099)
            ws[k] = (b, b2s.i2s_tensor(b, *dims[k]))
        x = x0 if i == 0 else torch.roll(x0, shifts=i * 37, dims=1).contiguous()
        sets.append((ws, x))
    g1, g2 = torch.from_numpy(f.g1).to(dev), torch.from_numpy(f.g2).to(dev)
    ldq_h, ldq_f = (H + 15) // 16 * 16, (F + 15) // 16 * 16
    q1 = torch.empty((M, ldq_h), dtype=torch.int8, device=dev)[:, :H]
    q2 = torch.empty((M, ldq_f), dtype=torch.int8, device=dev)[:, :F]
    s1, s2 = (torch.empty(M, dtype=torch.float32, device=dev) for _ in range(2))
    u1, u2 = (torch.empty(M, dtype=torch.int32, device=dev) for _ in range(2))
    P = torch.empty((M, F), dtype=torch.float32, device=dev)
    Y = torch.empty((M, H), dtype=torch.float32, device=dev)
    rot_bytes = sum(b.numel() for ws, _ in sets for b, _ in ws.values()) + sum(x.numel() * 4 for _, x in sets)

    stream = torch.cuda.Stream(device=dev)
    ws_bytes = b2s.ffn_block_workspace_size(M, H, F)
    wsp = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)

    # The timed step is the library's one-call FFN block (b2s_ffn_block: four kernels chained by
    # programmatic dependent launch, split-K partials through the caller's workspace).
    def step(i):
        ws, x = sets[i % N_SETS]
        b2s.ffn_block(x, g1, g2, EPS, ws["w_gate"][1], ws["w_up"][1], ws["w_down"][1], Y, wsp, stream=stream)

    # The same four kernels as separate calls with CUDA events around the gate/up GEMM: the per-launch
    # duration of the roofline kernel, replayed after the timed region.
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(N_SETS)]

    def step_probe(i):
        ws, x = sets[i % N_SETS]
        b2s.rms_norm_act_quant(x, g1, EPS, q1, s1, u1, stream=stream)
        ev[i % N_SETS][0].record(stream)
        b2s.ffn_gate_up_sqrelu_q8(ws["w_gate"][1], ws["w_up"][1], q1, s1, u1, P, stream=stream)
        ev[i % N_SETS][1].record(stream)
        b2s.rms_norm_act_quant(P, g2, EPS, q2, s2, u2, stream=stream)
        b2s.mul_mat_q8(ws["w_down"][1], q2, s2, u2, Y, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(3, a.warmup)):
            step(i)
            step_probe(i)
    stream.synchronize()
    assert b2s.device_error() == 0

    graphs, probes = [], []
    for i in range(N_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(i)
        graphs.append(g)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step_probe(i)
        probes.append(g)
    with torch.cuda.stream(stream):
        for i in range(max(3, a.warmup)):
            graphs[i % N_SETS].replay()
    stream.synchronize()

    def barrier():
        if pg is not None:
            pg.barrier()

    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            t_start.record(stream)
            for i in range(a.steps):
                graphs[i % N_SETS].replay()
            t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = t_start.elapsed_time(t_end)
    assert b2s.device_error() == 0

    n_probe = max(2 * N_SETS, min(a.steps, 400))
    k_sum, k_n = 0.0, 0
    with torch.cuda.stream(stream):
        for i in range(n_probe):
            probes[i % N_SETS].replay()
            if (i + 1) % N_SETS == 0:  # read the events of the last N_SETS replays before they are re-recorded
                stream.synchronize()
                if i >= N_SETS:  # the first round is a warm-up
                    k_sum += sum(e0.elapsed_time(e1) for e0, e1 in ev)
                    k_n += N_SETS
    stream.synchronize()
    k_ms = [k_sum / k_n]
    assert b2s.device_error() == 0

    # ---- e2e: the public one-call API with host buffers, copies inside the timed region. Consecutive steps
    # are pipelined over three streams, as a server feeding a stream of batches would run them: the H2D copy
    # of step i+1 and the D2H copy of step i-1 overlap the FFN block of step i (three device buffer slots).
    # Runs of up to 64 steps are captured as CUDA graphs (fork/join over the three streams) so that host
    # launch overhead does not pace the pipeline; the pipeline drains at each graph boundary.
    NBUF, GSTEPS = 3, 64
    xh = [x.cpu().pin_memory() for _, x in sets]
    yh = [torch.empty((M, H), dtype=torch.float32).pin_memory() for _ in range(NBUF)]
    xd = [torch.empty((M, H), dtype=torch.float32, device=dev) for _ in range(NBUF)]
    yd = [torch.empty((M, H), dtype=torch.float32, device=dev) for _ in range(NBUF)]
    s_h2d, s_d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_run(i0, n):
        """Steps i0 .. i0+n-1 on the three streams (called eagerly or under graph capture on `stream`)."""
        ev_in = [torch.cuda.Event() for _ in range(NBUF)]   # H2D of the slot done
        ev_ff = [torch.cuda.Event() for _ in range(NBUF)]   # FFN of the slot done (x slot free, y ready)
        ev_out = [torch.cuda.Event() for _ in range(NBUF)]  # D2H of the slot done (y slot free)
        fork = torch.cuda.Event()
        fork.record(stream)
        s_h2d.wait_event(fork)
        s_d2h.wait_event(fork)
        for j in range(n):
            i, b = i0 + j, j % NBUF
            ws, _ = sets[i % N_SETS]
            if j >= NBUF:
                s_h2d.wait_event(ev_ff[b])
            with torch.cuda.stream(s_h2d):
                xd[b].copy_(xh[i % N_SETS], non_blocking=True)
            ev_in[b].record(s_h2d)
            stream.wait_event(ev_in[b])
            if j >= NBUF:
                stream.wait_event(ev_out[b])
            b2s.ffn_block(xd[b], g1, g2, EPS, ws["w_gate"][1], ws["w_up"][1], ws["w_down"][1], yd[b], wsp,
                          stream=stream)
            ev_ff[b].record(stream)
            s_d2h.wait_event(ev_ff[b])
            with torch.cuda.stream(s_d2h):
                yh[b].copy_(yd[b], non_blocking=True)
            ev_out[b].record(s_d2h)
        for b in range(min(n, NBUF)):  # join the side streams back into `stream`
            stream.wait_event(ev_out[b])

    e2e_run(0, max(3, a.warmup))
    torch.cuda.synchronize()
    runs = [GSTEPS] * (a.steps // GSTEPS) + ([a.steps % GSTEPS] if a.steps % GSTEPS else [])
    e2e_graphs = {}
    for n in sorted(set(runs)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            e2e_run(0, n)
        e2e_graphs[n] = g
    with torch.cuda.stream(stream):
        for n in sorted(set(runs)):
            e2e_graphs[n].replay()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e_start.record(stream)
        for n in runs:
            e2e_graphs[n].replay()
        e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e_ms = e_start.elapsed_time(e_end)
    assert b2s.device_error() == 0
    assert torch.isfinite(yh[(runs[-1] - 1) % NBUF]).all()
    for g in e2e_graphs.values():
        g.reset()

    # ---- max over ranks
    if pg is not None:
        t = torch.tensor([ms, e_ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
    for g in graphs:
        g.reset()
    if pg is not None:
        pg.destroy_process_group()
    if rank != 0:
        return

    pk, pk_kind = peaks()
    tensor_peak_tops = 2.0 * pk.get("bf16_tflops_sustained", pk["bf16_tflops"])  # int8 dense = 2x bf16 dense
    k_avg_ms = sum(k_ms) / len(k_ms)
    achieved = GATE_UP_OPS / (k_avg_ms * 1e-3) / 1e12
    traffic = None  # DRAM read+write bytes per gate/up launch from the committed ncu capture summary
    try:
        import re
        with open(os.path.join(ROOT, "profiles", "gemm_i2s_tc_ffn_block_m300.md")) as fh:
            mt = re.search(r"traffic_bytes_per_launch \(gate/up, read \+ write\): (\d+)", fh.read())
        traffic = int(mt.group(1)) if mt else None
    except OSError:
        pass
    value = world * a.steps * OPS_PER_STEP / (ms * 1e-3) / 1e12
    e2e = world * a.steps * OPS_PER_STEP / (e_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TOP/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xternary->int32 (fp32 in/out)",
        "data": "synthetic (seeded random-init ternary weights, N(0,1) activations)",
        "config": {"workload": "ffn_block_bitnet2b_m300", "M": M, "hidden": H, "ffn": F, "eps": EPS,
                   "parallelism": f"dp{world} (independent FFN batches per GPU)",
                   "l2": f"{N_SETS} rotating weight/activation sets, {rot_bytes / 1e6:.0f} MB > 2x L2",
                   "step": "b2s_ffn_block in a CUDA graph: rmsnorm+actquant, tcgen05 gate/up+sqrelu, "
                           "rmsnorm+actquant, tcgen05 down (split-K through the workspace)"},
        "e2e": {"value": round(e2e, 3), "unit": "TOP/s", "h2d_bytes_per_step": M * H * 4,
                "d2h_bytes_per_step": M * H * 4, "ms_per_step": round(e_ms / a.steps, 5),
                "api": "b2s_ffn_block (C ABI) with pinned host buffers",
                "pipeline": "3 streams, 3 device buffer slots: H2D(i+1) and D2H(i-1) overlap FFN(i); "
                            "CUDA graphs of 64 steps (the pipeline drains between graphs)"},
        "roofline": {"kernel": "gemm_i2s_tc_kernel (gate/up, mode 1)", "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": round(tensor_peak_tops, 1), "unit": "TOP/s",
                     "frac": round(achieved / tensor_peak_tops, 4), "traffic": traffic,
                     "avg_launch_us": round(k_avg_ms * 1e3, 3),
                     "launch_timing": f"CUDA events around the gate/up launch, {k_n} replays after the timed region",
                     "peak_basis": f"int8 dense = 2x {pk_kind} cuBLAS bf16 sustained "
                                   f"({pk.get('bf16_tflops_sustained', pk['bf16_tflops'])} TFLOP/s)"},
        "gpu_launches": 4 * a.steps,
        "clocks": clk.summary(),
    }
    if world == 1:
        nthreads = cpu_threads()
        n, dt = cpu_ffn_sample(a.cpu_seconds, nthreads)
        import oracle
        line["cpu_baseline"] = {
            "value": round(n * OPS_PER_STEP / dt / 1e12, 5), "unit": "TOP/s", "cores": nthreads, "kind": "port",
            "sample": f"{n} full FFN blocks in {dt:.1f} s, {['scalar', 'AVX2', 'AVX512-VNNI'][oracle.fast_isa()]}, "
                      f"{cpu_model()}"}
    print(json.dumps(line), flush=True)


def run_bitvla_reference(a, world, rank):
    """The oracle's forward (the CPU restatement of the path) on all host threads, one observation per step."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    nthreads = cpu_threads()
    cfg = oracle.bitvla_config()
    imgs, toks, _ = bitvla_inputs(1, 0, cfg.image_size, cfg.n_text, cfg.vocab)
    steps = max(1, min(a.steps, 3))
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.bitvla_forward(cfg, 1234, imgs, toks, nthreads)
    dt = time.perf_counter() - t0
    value = steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "obs/s", "n_gpus": world,
            "steps": steps, "warmup": 0, "ms_per_step": round(dt / steps * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8xternary->int32",
            "data": "synthetic (seeded random-init BitVLA-shape weights)",
            "config": {"workload": "bitvla_server_64obs", "parallelism": "host threads"},
            "cpu_baseline": {"value": round(value, 5), "unit": "obs/s", "cores": nthreads, "kind": "port",
                             "sample": f"{steps} observation forwards, {cpu_model()}"},
            "e2e": {"value": round(value, 5), "unit": "obs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- BitVLA server run
def bitvla_inputs(n_obs: int, first: int, image_size: int, n_text: int, vocab: int):
    """Observation i: seeded U(0,1) image (also as uint8 for the host API) and uniform token ids."""
    import numpy as np
    imgs = np.empty((n_obs, 3, image_size, image_size), np.float32)
    toks = np.empty((n_obs, n_text), np.int32)
    for j in range(n_obs):
        g = np.random.Generator(np.random.PCG64(1000 + first + j))
        imgs[j] = g.random((3, image_size, image_size), dtype=np.float32)
        toks[j] = g.integers(0, vocab, n_text)
    u8 = np.ascontiguousarray((imgs * 255.0 + 0.5).astype(np.uint8).transpose(0, 2, 3, 1))
    return imgs, toks, u8


def kernels_per_forward(cfg) -> int:
    """Library kernels in one captured forward: patch embedding; 9 per ViT layer (norm+quant, qkv,
    attention, quant, o, norm+quant, fc1, quant, fc2); connector 4; text embedding; 10 per decoder layer
    (norm+quant, qkv, RoPE, attention, norm+quant, o, norm+quant, gate/up, norm+quant, down); final norm;
    action head."""
    return 1 + 9 * cfg.vit_layers + 4 + (1 if cfg.n_text > 0 else 0) + 10 * cfg.dec_layers + 2


def run_bitvla(a, world, rank, local):
    import numpy as np
    import torch
    import b2s
    from b2s import bitvla

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2s.check(b2s.lib().b2s_device_check())
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    cfg = bitvla.default_config()
    total = a.observations
    lo, hi = total * rank // world, total * (rank + 1) // world
    mine = hi - lo
    B = max(1, min(a.obs_batch, mine))
    batches = [(i, min(B, mine - i)) for i in range(0, mine, B)]
    model = bitvla.Model(cfg, 1234, max_batch=B)  # same seed on every rank: replicated weights
    imgs, toks, u8 = bitvla_inputs(mine, lo, cfg.image_size, cfg.n_text, cfg.vocab)
    d_img = torch.from_numpy(imgs).to(dev)
    d_tok = torch.from_numpy(toks).to(dev)
    A = cfg.action_chunk * cfg.action_dim
    d_act = torch.empty((mine, A), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(ev=None):
        for j, (i0, nb) in enumerate(batches):
            if ev is not None:
                ev[j][0].record(stream)
            model.forward(d_img[i0:i0 + nb], d_tok[i0:i0 + nb], None, d_act[i0:i0 + nb], stream=stream)
            if ev is not None:
                ev[j][1].record(stream)

    for _ in range(max(3, a.warmup)):
        step()
    stream.synchronize()
    assert b2s.device_error() == 0

    def barrier():
        if pg is not None:
            pg.barrier()

    steps = a.steps
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in batches]
           for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for k in range(steps):
            step(evs[k])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1)
    lat = sorted(e0.elapsed_time(e1) for ev in evs for e0, e1 in ev)
    assert b2s.device_error() == 0

    # e2e: host uint8 images + tokens in, host actions out, through the predict API
    h_act = np.empty((mine, A), np.float32)

    def e2e_step():
        for i0, nb in batches:
            model.predict(u8[i0:i0 + nb], toks[i0:i0 + nb], h_act[i0:i0 + nb], stream=stream)

    e2e_step()
    barrier()
    torch.cuda.synchronize()
    te = time.perf_counter()
    for _ in range(steps):
        e2e_step()
    torch.cuda.synchronize()
    e_ms = (time.perf_counter() - te) * 1e3
    barrier()
    if pg is not None:
        t = torch.tensor([ms, e_ms], dtype=torch.float64, device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, e_ms = float(t[0]), float(t[1])
        pg.destroy_process_group()
    tern_mb = model.ternary_bytes() / 1e6
    model.close()
    if rank != 0:
        return
    ops = bitvla.ternary_ops(cfg)
    pk, pk_kind = peaks()
    tensor_peak_tops = 2.0 * pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    value = steps * total / (ms * 1e-3)
    fwd_ms = statistics.median(lat)
    achieved = ops * B / (fwd_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "obs/s", "n_gpus": world, "steps": steps,
        "warmup": a.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8xternary->int32 (fp32 attention, norms, residual)",
        "data": "synthetic (seeded random-init BitVLA-shape weights, U(0,1) images, uniform tokens)",
        "config": {"workload": "bitvla_server_64obs", "observations": total, "obs_per_forward": B,
                   "image": cfg.image_size, "vit_layers": cfg.vit_layers, "decoder_layers": cfg.dec_layers,
                   "tokens": bitvla.seq_len(cfg), "parallelism": f"dp{world} (observations sharded, no collective)",
                   "l2": f"{tern_mb:.0f} MB of ternary weights streamed per forward (> 126 MB L2)"},
        "latency_ms": {"p50": round(fwd_ms, 3), "p90": round(lat[int(0.9 * (len(lat) - 1))], 3),
                       "unit": "ms per forward of obs_per_forward observations"},
        "e2e": {"value": round(steps * total / (e_ms * 1e-3), 3), "unit": "obs/s",
                "h2d_bytes_per_step": total * (3 * cfg.image_size ** 2 + 4 * cfg.n_text),
                "d2h_bytes_per_step": total * A * 4, "api": "b2s_bitvla_predict (C ABI), host uint8 images"},
        "roofline": {"kernel": "whole forward (ternary int ops / forward time)", "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": round(tensor_peak_tops, 1), "unit": "TOP/s",
                     "frac": round(achieved / tensor_peak_tops, 4), "traffic": None,
                     "peak_basis": f"int8 dense = 2x {pk_kind} cuBLAS bf16 sustained"},
        "gpu_launches": steps * len(batches) * kernels_per_forward(cfg),
        "clocks": clk.summary(),
    }
    if world == 1:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # CPU baseline leg only
        nthreads = cpu_threads()
        ocfg = oracle.bitvla_config()
        t_c = time.perf_counter()
        oracle.bitvla_forward(ocfg, 1234, imgs[:1], toks[:1], nthreads)
        dt = time.perf_counter() - t_c
        line["cpu_baseline"] = {"value": round(1.0 / dt, 5), "unit": "obs/s", "cores": nthreads, "kind": "port",
                                "sample": f"1 observation (full forward) in {dt:.1f} s, {cpu_model()}"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- GEMM sweep
def run_sweep(a, world, rank, local):
    import torch
    import b2s
    from b2s import workloads as wl

    if world > 1:
        run_sweep_nsplit(a, world, rank, local)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2s.check(b2s.lib().b2s_device_check())
    pk, pk_kind = peaks()
    hbm = pk["hbm_gbs"]
    tensor_peak = 2.0 * pk.get("bf16_tflops", 1590.0)  # launches timed alone: the burst figure
    stream = torch.cuda.Stream(device=dev)
    ms_list = [int(x) for x in a.sweep_m.split(",")] if a.sweep_m else list(wl.SWEEP_M)
    rows = []
    for K, N in wl.SWEEP_KN:
        g = wl.rng(K + N)
        w = wl.weight(g, N, K)
        base = torch.from_numpy(w.packed).to(dev)
        Kp = (K + 127) // 128 * 128
        if K % 128:
            rb = torch.empty(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device=dev)
            b2s.repack_rows(base, rb, N, K, stream=stream)
            stream.synchronize()
            base = rb
        wbytes = N * Kp // 4
        R = max(2, min(256, -(-(2 * 126 * 2**20 + 8 * 2**20) // wbytes)))
        copies = []
        for r in range(R):
            b = base.clone()
            if r:
                b[:wbytes] = torch.roll(base[:wbytes], shifts=r * 4099)
            copies.append((b, b2s.i2s_tensor(b, N, K, rowpadded=bool(K % 128))))
        for M in ms_list:
            ldq = (K + 15) // 16 * 16
            q = torch.randint(-127, 128, (M, ldq), dtype=torch.int8, device=dev)[:, :K]
            s = torch.rand(M, device=dev) + 0.5
            u = q.to(torch.int32).sum(dim=1).to(torch.int32)
            y = torch.empty((M, N), dtype=torch.float32, device=dev)
            launches = R if M <= 4096 else max(2, min(R, 16))
            def seq():
                for r in range(launches):
                    b2s.mul_mat_q8(copies[r % R][1], q, s, u, y, stream=stream)
            with torch.cuda.stream(stream):
                seq()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                seq()
            with torch.cuda.stream(stream):
                for _ in range(3):
                    graph.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 5
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
            stream.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * launches)
            assert b2s.device_error() == 0
            ops = 2.0 * M * N * K
            byts = wbytes + M * K + 8 * M + 4 * M * N
            tops, gbs = ops / us / 1e6, byts / us / 1e3
            bound = "hbm" if M <= 16 else "tensor"
            rows.append({"M": M, "K": K, "N": N, "path": "gemv" if M <= 16 else "tcgen05", "us": round(us, 3),
                         "TOP/s": round(tops, 1), "GB/s": round(gbs, 1), "bound": bound,
                         "frac": round(gbs / hbm if bound == "hbm" else tops / tensor_peak, 4)})
            graph.reset()
            del q, s, u, y
        del copies
        torch.cuda.empty_cache()
    big = [r["TOP/s"] for r in rows if r["M"] >= 4096]
    line = {"metric": METRIC, "value": round(sum(big) / max(1, len(big)), 1), "unit": "TOP/s (mean over M >= 4096)",
            "n_gpus": 1, "steps": 5, "warmup": 3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xternary->int32", "data": "synthetic (ternary P(0)=0.4, random int8 activations)",
            "config": {"workload": "i2s_gemm_sweep", "l2": "rotating weight copies, > 2x L2 of weights per pass",
                       "peaks": f"{pk_kind}: HBM {hbm} GB/s, int8 = 2x bf16 burst {tensor_peak:.0f} TOP/s"},
            "sweep": rows}
    print(json.dumps(line), flush=True)


def run_sweep_nsplit(a, world, rank, local):
    """M = 16384 N-split over the ranks: rank r owns weight rows [n0_r, n1_r) and its GEMM epilogue stores
    its column slice straight into rank 0's output buffer over NVLink (CUDA IPC mapping, plain peer
    stores). Timing: max over ranks of `launches` back-to-back GEMMs. Roofline of the fused GEMM+gather:
    the slower of (ops / int8 peak) and (bytes crossing into rank 0 / measured 770 GB/s per direction)."""
    import datetime
    import torch
    import torch.distributed as dist
    import b2s
    from b2s import workloads as wl
    from b2s.nsplit import PeerBuffer, row_ranges, nsplit_mul_mat_q8, shard_i2s_rows

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    b2s.check(b2s.lib().b2s_device_check())
    pk, pk_kind = peaks()
    tensor_peak = 2.0 * pk.get("bf16_tflops", 1590.0)
    link_gbs = 770.0
    M = 16384
    stream = torch.cuda.Stream(device=dev)
    rows = []
    for K, N in wl.SWEEP_KN:
        g = wl.rng(K + N)
        w = wl.weight(g, N, K)
        n0, n1 = row_ranges(N, world)[rank]
        shard = torch.from_numpy(shard_i2s_rows(w.packed, N, K, n0, n1)).to(dev)
        W = b2s.i2s_tensor(shard, n1 - n0, K)
        ldq = (K + 15) // 16 * 16
        gq = torch.Generator(device=dev)
        gq.manual_seed(K * 7 + N)
        q = torch.randint(-127, 128, (M, ldq), dtype=torch.int8, device=dev, generator=gq)[:, :K]
        sc = torch.rand(M, device=dev, generator=gq) + 0.5
        u = q.to(torch.int32).sum(dim=1).to(torch.int32)
        yb = PeerBuffer(M * N * 4)
        launches = 8
        with torch.cuda.stream(stream):
            for _ in range(2):
                nsplit_mul_mat_q8(b2s, W, q, sc, u, M, yb.ptr, N, n0, stream=stream)
        stream.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(launches):
                nsplit_mul_mat_q8(b2s, W, q, sc, u, M, yb.ptr, N, n0, stream=stream)
            e1.record(stream)
        stream.synchronize()
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        assert b2s.device_error() == 0
        us = float(t[0]) * 1e3 / launches
        ops = 2.0 * M * N * K
        cross = 4.0 * M * (N - (row_ranges(N, world)[0][1]))  # fp32 output columns stored into rank 0 by peers
        t_roof = max(ops / (tensor_peak * 1e12) * 1e6, cross / (link_gbs * 1e9) * 1e6)
        rows.append({"M": M, "K": K, "N": N, "gpus": world, "us": round(us, 2), "TOP/s": round(ops / us / 1e6, 1),
                     "nvlink_bytes_into_root": int(cross), "roofline_us": round(t_roof, 2),
                     "frac": round(t_roof / us, 4),
                     "bound": "nvlink" if cross / (link_gbs * 1e9) > ops / (tensor_peak * 1e12) else "tensor"})
        dist.barrier()
        yb.close()
        del q, sc, u, shard
    dist.destroy_process_group()
    if rank == 0:
        line = {"metric": METRIC, "value": round(sum(r["TOP/s"] for r in rows) / len(rows), 1),
                "unit": "TOP/s (mean over shapes, whole job)", "n_gpus": world, "steps": 8, "warmup": 2,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xternary->int32",
                "data": "synthetic", "config": {"workload": "i2s_gemm_nsplit_m16384",
                                                "parallelism": f"N-split over {world} GPUs, output gathered "
                                                               "into rank 0 by epilogue peer stores"},
                "sweep": rows}
        print(json.dumps(line), flush=True)


def main():
    a = parse()
    world, rank, local = dist_env()
    if a.workload == "sweep":
        run_sweep(a, world, rank, local)
        return
    if a.workload == "bitvla":
        if a.impl == "reference":
            run_bitvla_reference(a, world, rank)
        else:
            run_bitvla(a, world, rank, local)
        return
    if a.impl == "reference":
        run_reference(a, world, rank)
        return
    run_b2s(a, world, rank, local)


if __name__ == "__main__":
    main()
