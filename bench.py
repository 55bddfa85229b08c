"""Benchmark of the ternary i2_s path on B200: one JSON line on rank 0.

Workload (a "step"): the BitNet-b1.58-2B-shape FFN block at prefill M=300 tokens --
RMSNorm(2560, eps 1e-5) -> ternary gate/up 2560->6912 -> squared-ReLU gate product -> RMSNorm(6912) ->
ternary down 6912->2560 -- i.e. three i2_s mul_mats (31.85 G ternary int ops) plus their fused
neighbours, on seeded synthetic inputs (weights ternary P(0)=0.4, one scale U(0.5,2) per matrix;
activations N(0,1); norm weights N(1,0.1)). There are no checkpoints here; the inputs are random-init.

  value   = whole-job ternary int-op throughput (TOP/s) with inputs resident in HBM: each step replays a
            CUDA graph of the four kernels over one of 16 rotating weight/activation sets (~261 MB, more
            than twice the 126 MB L2, so weights stream from HBM as they would across 30 layers).
  e2e     = the same metric through the public C ABI call b2s_ffn_block, with the step's activations
            copied host->device from pinned memory and the output copied back, inside the timed region.
  roofline= the gate/up tensor-core GEMM (the dominant kernel), timed with CUDA events recorded inside
            the replayed graphs during the timed region, against the measured tensor peak.
  cpu_baseline = the threaded SIMD port of the oracle on the host cores (rank 0, N=1 only).

--impl reference times the reference's CPU implementation of the path. The reference's own i2_s CPU
kernels (BitNet's ggml fork) are not in the reference tree, so this is the oracle port, with all host
threads, on the same workload.

Multi-GPU: one process per GPU (torchrun); the FFN block batches are independent (data parallel, no
collective on the data path); timing is the max over ranks; scaling "weak".
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
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", default="b2s", choices=["b2s", "reference"])
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="bounded CPU-baseline sample length")
    return p.parse_args()


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
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(N_SETS)]

    def step(i, record=False):
        ws, x = sets[i % N_SETS]
        b2s.rms_norm_act_quant(x, g1, EPS, q1, s1, u1, stream=stream)
        if record:
            ev[i % N_SETS][0].record(stream)
        b2s.ffn_gate_up_sqrelu_q8(ws["w_gate"][1], ws["w_up"][1], q1, s1, u1, P, stream=stream)
        if record:
            ev[i % N_SETS][1].record(stream)
        b2s.rms_norm_act_quant(P, g2, EPS, q2, s2, u2, stream=stream)
        b2s.mul_mat_q8(ws["w_down"][1], q2, s2, u2, Y, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(3, a.warmup)):
            step(i)
    stream.synchronize()
    assert b2s.device_error() == 0

    graphs = []
    for i in range(N_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(i, record=True)
        graphs.append(g)
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
    k_ms = [e0.elapsed_time(e1) for e0, e1 in ev[:min(N_SETS, a.steps)]]
    assert b2s.device_error() == 0

    # ---- e2e: the public one-call API with host buffers, copies inside the timed region
    ws_bytes = b2s.ffn_block_workspace_size(M, H, F)
    wsp = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    xh = [x.cpu().pin_memory() for _, x in sets]
    yh = torch.empty((M, H), dtype=torch.float32).pin_memory()
    xd = torch.empty((M, H), dtype=torch.float32, device=dev)
    yd = torch.empty((M, H), dtype=torch.float32, device=dev)

    def e2e_step(i):
        ws, _ = sets[i % N_SETS]
        xd.copy_(xh[i % N_SETS], non_blocking=True)
        b2s.ffn_block(xd, g1, g2, EPS, ws["w_gate"][1], ws["w_up"][1], ws["w_down"][1], yd, wsp, stream=stream)
        yh.copy_(yd, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(max(3, a.warmup)):
            e2e_step(i)
    stream.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e_start.record(stream)
        for i in range(a.steps):
            e2e_step(i)
        e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e_ms = e_start.elapsed_time(e_end)
    assert b2s.device_error() == 0

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
                   "step": "4 kernels in a CUDA graph: rmsnorm+actquant, tcgen05 gate/up+sqrelu, "
                           "rmsnorm+actquant, tcgen05 down"},
        "e2e": {"value": round(e2e, 3), "unit": "TOP/s", "h2d_bytes_per_step": M * H * 4,
                "d2h_bytes_per_step": M * H * 4, "ms_per_step": round(e_ms / a.steps, 5),
                "api": "b2s_ffn_block (C ABI) with pinned host buffers"},
        "roofline": {"kernel": "gemm_i2s_tc_kernel (gate/up, mode 1)", "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": round(tensor_peak_tops, 1), "unit": "TOP/s",
                     "frac": round(achieved / tensor_peak_tops, 4), "traffic": traffic,
                     "avg_launch_us": round(k_avg_ms * 1e3, 3),
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


def main():
    a = parse()
    world, rank, local = dist_env()
    if a.impl == "reference":
        run_reference(a, world, rank)
        return
    run_b2s(a, world, rank, local)


if __name__ == "__main__":
    main()
