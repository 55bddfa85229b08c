"""Benchmark of the ternary i2_s path on B200: one JSON line on rank 0.

Headline (default, --workload server): the batched model-server run -- 64 independent random-init
BitVLA-shape observations (224x224 image + 32 text tokens each; 27-layer ternary ViT, connector, 30-layer
ternary decoder prefill of 288 tokens) sharded data parallel over the ranks with no collective on the data
path (strong scaling: the 64 observations are the whole job). A "step" is the whole 64-observation job;
each rank runs its share as graph-captured forwards of --obs-batch observations.
  value        = observations/s of the whole job, device-timed with CUDA events with inputs resident in
                 HBM (max over ranks); the 627 MB of packed ternary weights stream from HBM every forward.
  e2e          = the same metric through the C ABI call b2s_bitvla_predict with host buffers: uint8 HWC
                 images and token ids copied in, actions copied out, inside the timed region.
  latency_ms   = p50 / p90 of one forward of --obs-batch observations.
  roofline     = the dominant kernel family of the forward (the persistent tcgen05 GEMM), timed alone with
                 CUDA events at the decoder's gate/up shape (M = obs-batch x 288 tokens), against the
                 measured int8 peak (2x the cuBLAS bf16 burst figure).
  cpu_baseline = the oracle's forward (the CPU restatement of the path, weights resident in host memory) on
                 the host cores, rank 0, N=1.

Sub-objects of the same line (each with its own timing, described in its keys):
  ffn_block  -- the BitNet-b1.58-2B-shape FFN block at prefill M=300 (31.85 G ternary int ops per step),
                data parallel per rank, with its gate/up roofline and CPU baseline;
  gemm_c0    -- one 2560x2560 i2_s MUL_MAT of 256 tokens through b2s_mul_mat (fp32 in/out), N=1;
  sweep      -- the i2_s GEMM roofline sweep M x (K,N) on pre-quantized activations, N=1;
  nsplit     -- (N>1) the M=16384 GEMM split over the GPUs' output rows with the output gathered into rank 0
                by epilogue peer stores: compute-only and compute+gather times and a bit-exactness flag
                against the single-GPU GEMM.

--impl reference times the reference's CPU implementation of the path. The reference's own i2_s CPU
kernels (BitNet's ggml fork) are not in the reference tree, so this is the oracle port (the CPU
restatement), on all host threads, on the same workload and config; it never loads the CUDA library.

--workload ffn / sweep / roofline run one sub-workload alone (the commands some profiles under profiles/ were
taken with); roofline is the headline's GEMM measurement at the 8-observation decoder shape.
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
SEED = 1234
SWEEP_M = (1, 16, 256, 4096, 16384)
SWEEP_KN = ((2560, 2560), (2560, 6912), (6912, 2560), (1152, 4304))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 5 jobs of --observations for server, 2000 FFN blocks for ffn)")
    p.add_argument("--warmup", type=int, default=None, help="untimed warm-up steps (default: 3 server, 20 ffn)")
    p.add_argument("--impl", default="b2s", choices=["b2s", "reference"])
    p.add_argument("--workload", default="server", choices=["server", "bitvla", "ffn", "sweep", "roofline"])
    p.add_argument("--cpu-seconds", type=float, default=6.0, help="bounded CPU-baseline sample length (FFN)")
    p.add_argument("--observations", type=int, default=64, help="server: observations in the whole job")
    p.add_argument("--obs-batch", type=int, default=8, help="server: observations per forward")
    p.add_argument("--sweep-m", default="", help="sweep: comma-separated M values (default: all five)")
    p.add_argument("--sweep-kn", default="", help="sweep: comma-separated KxN shapes (default: all four)")
    p.add_argument("--batched-only", action="store_true", help="sweep: decode sizes as batched launches only")
    p.add_argument("--no-extras", action="store_true", help="server: headline only, no sub-objects")
    a = p.parse_args()
    if a.workload == "bitvla":
        a.workload = "server"
    if a.steps is None:
        a.steps = 5 if a.workload == "server" else 2000
    if a.warmup is None:
        a.warmup = 3 if a.workload == "server" else 20
    return a


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    """Measured peaks (MEASURED_PEAKS.json) or the pool's fallback, and which one was used."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def int8_peak(burst: bool):
    """int8 dense TOP/s = 2x the cuBLAS bf16 figure (sm_100's int8 MMA rate is twice its bf16 rate): the
    burst figure for a kernel timed alone, the sustained one for a kernel timed inside a long step."""
    pk, kind = peaks()
    key = "bf16_tflops" if burst else "bf16_tflops_sustained"
    v = pk.get(key, pk["bf16_tflops"])
    return 2.0 * v, f"int8 dense = 2x {kind} cuBLAS bf16 {'burst' if burst else 'sustained'} ({v} TFLOP/s)"


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


def server_config(world: int, a) -> dict:
    """The config dict of the headline workload (identical in both arms)."""
    return {"workload": "bitvla_server_64obs", "observations": a.observations, "obs_per_forward": a.obs_batch,
            "image": 224, "vit_layers": 27, "decoder_layers": 30, "tokens": 288, "seed": SEED,
            "parallelism": f"dp{world} (observations sharded, no collective)",
            "l2": "627 MB of packed ternary weights streamed per forward (> 126 MB L2)"}


def ffn_config(world: int) -> dict:
    return {"workload": "ffn_block_bitnet2b_m300", "M": M, "hidden": H, "ffn": F, "eps": EPS,
            "parallelism": f"dp{world} (independent FFN batches per GPU)",
            "l2": f"{N_SETS} rotating weight/activation sets, 261 MB > 2x L2"}


# ------------------------------------------------------------------------------------------- inputs (host)
def bitvla_inputs(n_obs: int, first: int, image_size: int = 224, n_text: int = 32, vocab: int = 128256):
    """Observation i: seeded U(0,1) image (also as uint8 HWC for the host API) and uniform token ids."""
    import numpy as np
    imgs = np.empty((n_obs, 3, image_size, image_size), np.float32)
    toks = np.empty((n_obs, n_text), np.int32)
    for j in range(n_obs):
        g = np.random.Generator(np.random.PCG64(1000 + first + j))
        imgs[j] = g.random((3, image_size, image_size), dtype=np.float32)
        toks[j] = g.integers(0, vocab, n_text)
    u8 = np.ascontiguousarray((imgs * 255.0 + 0.5).astype(np.uint8).transpose(0, 2, 3, 1))
    return imgs, toks, u8


def ffn_host_inputs(seed: int, packer):
    """Config-1 inputs: X N(0,1) [M,H], norm weights N(1,0.1), ternary weights P(0)=0.4 with one scale
    U(0.5,2) per matrix, packed by `packer(t int8 [N,K], scale) -> i2_s bytes` (the draws follow
    b2s.workloads.ffn_block, so both arms see the same bytes)."""
    import numpy as np
    g = np.random.Generator(np.random.PCG64(seed))
    x = g.standard_normal((M, H), dtype=np.float32)
    g1 = (1.0 + 0.1 * g.standard_normal(H)).astype(np.float32)
    g2 = (1.0 + 0.1 * g.standard_normal(F)).astype(np.float32)
    ws = []
    for n, k in ((F, H), (F, H), (H, F)):
        t = g.choice(np.array([-1, 0, 1], np.int8), size=(n, k), p=[0.3, 0.4, 0.3])
        sc = np.float32(g.uniform(0.5, 2.0))
        ws.append(packer(t, sc))
    return x, g1, g2, ws


# ------------------------------------------------------------------------------------------- reference arm
def run_reference(a, world, rank):
    """The oracle port on the host cores (rank 0 only); never loads the CUDA library."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    nthreads = cpu_threads()
    isa = ["scalar", "AVX2", "AVX512-VNNI"][oracle.fast_isa()]
    if a.workload == "ffn":
        x, g1, g2, ws = ffn_host_inputs(1, oracle.i2s_pack_ternary)
        args = (x, g1, g2, EPS, ws[0], ws[1], ws[2], H, F, nthreads)
        oracle.fast_ffn_block(*args)
        t1 = time.perf_counter()
        oracle.fast_ffn_block(*args)
        t_one = time.perf_counter() - t1
        steps = max(1, min(a.steps, int(60.0 / max(t_one, 1e-6))))
        t0 = time.perf_counter()
        for _ in range(steps):
            oracle.fast_ffn_block(*args)
        dt = time.perf_counter() - t0
        value, unit, cfg = steps * OPS_PER_STEP / dt / 1e12, "TOP/s", ffn_config(world)
        sample = f"{steps} full FFN blocks (M={M}, H={H}, F={F}) on {nthreads} threads, {isa}; {cpu_model()}"
        scaling = "weak"
    else:
        model = oracle.BitVLAModel(oracle.bitvla_config(), SEED, nthreads)  # weights generated once, untimed
        imgs, toks, _ = bitvla_inputs(4, 0)
        model.forward(imgs[:1], toks[:1])  # warm-up
        steps = max(1, min(a.steps, 3))
        t0 = time.perf_counter()
        for j in range(steps):
            model.forward(imgs[j + 1:j + 2], toks[j + 1:j + 2])
        dt = time.perf_counter() - t0
        model.close()
        value, unit, cfg = steps / dt, "obs/s", server_config(world, a)
        sample = (f"{steps} observation forwards (one per step; 27-layer ViT, connector, 30-layer decoder; "
                  f"weights resident in host memory) on {nthreads} threads, {isa}; {cpu_model()}")
        scaling = "strong"
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": world,
            "steps": steps, "warmup": 1, "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "int8xternary->int32",
            "data": "synthetic (seeded random-init ternary weights)", "config": cfg,
            "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": nthreads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a thread while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
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


class Dist:
    """One process per GPU over NCCL (world > 1): barriers and the max over ranks of timings."""

    def __init__(self, world, rank, dev):
        self.world, self.rank, self.dev, self.pg = world, rank, dev, None
        if world > 1:
            import datetime
            import torch.distributed as dist
            os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, vals):
        if self.pg is None:
            return list(vals)
        import torch
        t = torch.tensor(list(vals), dtype=torch.float64, device=self.dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return [float(v) for v in t.cpu()]

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()
            self.pg = None


def events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


# ------------------------------------------------------------------------------------------- headline: server
def kernels_per_forward(cfg) -> int:
    """Library kernels in one captured forward: patch embedding; 9 per ViT layer (norm+quant, qkv,
    attention, quant, o, norm+quant, fc1, quant, fc2); connector 4; text embedding; 9 per decoder layer
    (norm+quant, qkv, attention with RoPE applied to q/k as they are staged, norm+quant, o, norm+quant,
    gate/up, norm+quant, down; the tensor-core attention mode adds a separate RoPE pass); final norm;
    action head. 521 for the BitVLA shape, as the ncu launch list of one forward shows."""
    dec = 9 + (1 if getattr(cfg, "attention_tc", 0) else 0)
    return 1 + 9 * cfg.vit_layers + 4 + (1 if cfg.n_text > 0 else 0) + dec * cfg.dec_layers + 2


def run_server(a, D, local):
    import numpy as np
    import torch
    import b2s
    from b2s import bitvla

    dev = torch.device("cuda", local)
    cfg = bitvla.default_config()
    total, world, rank = a.observations, D.world, D.rank
    lo, hi = b2s.nsplit_range(total, world, rank)
    mine = hi - lo
    B = max(1, min(a.obs_batch, mine))
    batches = [(i, min(B, mine - i)) for i in range(0, mine, B)]
    model = bitvla.Model(cfg, SEED, max_batch=B)  # same seed on every rank: replicated weights
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

    steps = a.steps
    evs = [[events() for _ in batches] for _ in range(steps)]
    t0, t1 = events()
    D.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(stream)
        for k in range(steps):
            step(evs[k])
        t1.record(stream)
        torch.cuda.synchronize()
    D.barrier()
    ms = t0.elapsed_time(t1)
    lat = sorted(e0.elapsed_time(e1) for ev in evs for e0, e1 in ev)
    assert b2s.device_error() == 0
    assert torch.isfinite(d_act).all()

    # e2e: host uint8 images + tokens in, host actions out, through the predict API (it returns after the
    # actions have reached host memory); CUDA events on the same stream bracket the whole job.
    h_act = np.empty((mine, A), np.float32)

    def e2e_step():
        for i0, nb in batches:
            model.predict(u8[i0:i0 + nb], toks[i0:i0 + nb], h_act[i0:i0 + nb], stream=stream)

    e2e_step()
    e0, e1 = events()
    D.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    D.barrier()
    e_ms = e0.elapsed_time(e1)
    assert np.isfinite(h_act).all()
    tern_mb = model.ternary_bytes() / 1e6
    model.close()
    del d_img, d_tok, d_act

    # Through the request server (b2s_server: one engine on this rank's GPU, a bounded queue, batches of up to
    # B requests): every observation is submitted as its own request, then all are waited for. Host wall
    # clock around the job (the server runs its own threads and streams); per-request latency from submit to
    # completion.
    from b2s.server import Server
    srv = Server.bitvla([local], cfg, SEED, max_batch=B, queue_capacity=max(256, mine))
    for i in range(mine):  # warm-up: graph capture of the batch sizes the queue forms
        srv.wait(srv.submit(u8[i], toks[i]))
    ids = [srv.submit(u8[i], toks[i]) for i in range(mine)]
    for r in ids:
        srv.wait(r)
    D.barrier()
    s_lat = []
    t_s = time.perf_counter()
    for _ in range(steps):
        ids = [srv.submit(u8[i], toks[i]) for i in range(mine)]
        for r in ids:
            s_lat.append(srv.wait(r)[1])
    s_ms = (time.perf_counter() - t_s) * 1e3
    D.barrier()
    srv_batches = srv.engine_status()[0]["batches"]
    srv.close()
    ms, e_ms, s_ms = D.max([ms, e_ms, s_ms])
    s_lat.sort()
    value = steps * total / (ms * 1e-3)
    fwd_ms = statistics.median(lat)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "obs/s", "n_gpus": world, "steps": steps,
        "warmup": a.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8xternary->int32 (fp32 attention, norms, residual)",
        "data": "synthetic (seeded random-init BitVLA-shape weights, U(0,1) images, uniform tokens)",
        "config": server_config(world, a),
        "latency_ms": {"p50": round(fwd_ms, 3), "p90": round(lat[int(0.9 * (len(lat) - 1))], 3),
                       "unit": f"ms per forward of {B} observations"},
        "e2e": {"value": round(steps * total / (e_ms * 1e-3), 3), "unit": "obs/s",
                "h2d_bytes_per_step": total * (3 * cfg.image_size ** 2 + 4 * cfg.n_text),
                "d2h_bytes_per_step": total * A * 4, "ms_per_step": round(e_ms / steps, 4),
                "api": "b2s_bitvla_predict (C ABI): uint8 HWC host images and token ids in, host actions out"},
        "dispatcher": {"value": round(steps * total / (s_ms * 1e-3), 3), "unit": "obs/s",
                       "request_latency_ms": {"p50": round(s_lat[len(s_lat) // 2], 3),
                                              "p90": round(s_lat[int(0.9 * (len(s_lat) - 1))], 3)},
                       "api": "b2s_server_create_bitvla / b2s_server_submit / b2s_server_wait, one engine per GPU, "
                              f"up to {B} requests per batch",
                       "timing": "host wall clock around the submit/wait job (max over ranks)",
                       "batches_formed": int(srv_batches)},
        "gpu_launches": steps * len(batches) * kernels_per_forward(cfg),
        "ternary_weight_mb": round(tern_mb, 1),
        "clocks": clk.summary(),
    }
    return line, B * bitvla.seq_len(cfg)


def gemm_roofline(dev, Mtok: int):
    """The persistent tcgen05 GEMM at the decoder gate/up shape (Mtok tokens, 2560 -> 2 x 6912, squared-ReLU
    product), timed alone with CUDA events around each launch over rotating weights (> 2x L2)."""
    import torch
    import b2s
    from b2s import workloads as wl
    g = wl.rng(77)
    wg, wu = wl.weight(g, F, H), wl.weight(g, F, H)
    bg, bu = torch.from_numpy(wg.packed).to(dev), torch.from_numpy(wu.packed).to(dev)
    nb = bg.numel() - 32
    R = 32  # 32 x 8.8 MB of gate/up weights
    sets = []
    for r in range(R):
        a_, b_ = bg.clone(), bu.clone()
        if r:
            a_[:nb] = torch.roll(bg[:nb], shifts=r * 4099)
            b_[:nb] = torch.roll(bu[:nb], shifts=r * 8191)
        sets.append((a_, b_, b2s.i2s_tensor(a_, F, H), b2s.i2s_tensor(b_, F, H)))
    ldq = (H + 15) // 16 * 16
    q = torch.randint(-127, 128, (Mtok, ldq), dtype=torch.int8, device=dev)[:, :H]
    s = torch.rand(Mtok, device=dev) + 0.5
    u = q.to(torch.int32).sum(dim=1).to(torch.int32)
    p = torch.empty((Mtok, F), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    ev = [events() for _ in range(R)]
    tot, n = 0.0, 0
    with torch.cuda.stream(stream):
        for r in range(R):
            b2s.ffn_gate_up_sqrelu_q8(sets[r][2], sets[r][3], q, s, u, p, stream=stream)
        stream.synchronize()
        for rep in range(4):
            for r in range(R):
                ev[r][0].record(stream)
                b2s.ffn_gate_up_sqrelu_q8(sets[r][2], sets[r][3], q, s, u, p, stream=stream)
                ev[r][1].record(stream)
            stream.synchronize()
            tot += sum(e0.elapsed_time(e1) for e0, e1 in ev)
            n += R
    assert b2s.device_error() == 0
    us = tot / n * 1e3
    ops = 2.0 * 2 * Mtok * F * H
    peak, basis = int8_peak(burst=True)
    achieved = ops / us / 1e6
    traffic = None  # DRAM read+write bytes per launch from the committed ncu capture summary
    try:
        import re
        with open(os.path.join(ROOT, "profiles", "gemm_i2s_tcp_bitvla_gate_up_m2304.md")) as fh:
            mt = re.search(r"traffic_bytes_per_launch \(read \+ write\): (\d+)", fh.read())
        traffic = int(mt.group(1)) if mt else None
    except OSError:
        pass
    del sets, q, s, u, p
    torch.cuda.empty_cache()
    return {"kernel": "gemm_i2s_tcp_kernel (persistent tcgen05 i2_s GEMM; decoder gate/up + squared-ReLU)",
            "bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TOP/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "avg_launch_us": round(us, 3),
            "shape": f"M={Mtok} tokens, K={H}, N=2x{F}", "algorithmic_ops_per_launch": ops,
            "algorithmic_bytes_per_launch": int(2 * F * H // 4 + Mtok * H + 8 * Mtok + 4 * Mtok * F),
            "launch_timing": f"CUDA events around each of {n} launches over {R} rotating weight sets (> 2x L2)",
            "peak_basis": basis + " (launch timed alone)"}


# ------------------------------------------------------------------------------------------- config 1: FFN block
def run_ffn(a, D, local, steps: int, warmup: int):
    import torch
    import b2s
    from b2s import workloads as wl

    dev = torch.device("cuda", local)
    rank, world = D.rank, D.world
    x_h, g1_h, g2_h, packed = ffn_host_inputs(
        1 + rank, lambda t, sc: wl.i2s_quantize_host(t.astype("float32") * sc))
    base = {k: torch.from_numpy(p).to(dev) for k, p in zip(("w_gate", "w_up", "w_down"), packed)}
    dims = {"w_gate": (F, H), "w_up": (F, H), "w_down": (H, F)}
    sets = []
    x0 = torch.from_numpy(x_h).to(dev)
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
    g1, g2 = torch.from_numpy(g1_h).to(dev), torch.from_numpy(g2_h).to(dev)
    ldq_h, ldq_f = (H + 15) // 16 * 16, (F + 15) // 16 * 16
    q1 = torch.empty((M, ldq_h), dtype=torch.int8, device=dev)[:, :H]
    q2 = torch.empty((M, ldq_f), dtype=torch.int8, device=dev)[:, :F]
    s1, s2 = (torch.empty(M, dtype=torch.float32, device=dev) for _ in range(2))
    u1, u2 = (torch.empty(M, dtype=torch.int32, device=dev) for _ in range(2))
    P = torch.empty((M, F), dtype=torch.float32, device=dev)
    Y = torch.empty((M, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    wsp = torch.empty(b2s.ffn_block_workspace_size(M, H, F), dtype=torch.uint8, device=dev)

    # The timed step is the library's one-call FFN block (b2s_ffn_block: four kernels chained by
    # programmatic dependent launch, split-K partials through the caller's workspace).
    def step(i):
        ws, x = sets[i % N_SETS]
        b2s.ffn_block(x, g1, g2, EPS, ws["w_gate"][1], ws["w_up"][1], ws["w_down"][1], Y, wsp, stream=stream)

    # The same four kernels as separate calls with CUDA events around the gate/up GEMM: the per-launch
    # duration of the roofline kernel, replayed after the timed region.
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(N_SETS)]  # recorded inside captured graphs

    def step_probe(i):
        ws, x = sets[i % N_SETS]
        b2s.rms_norm_act_quant(x, g1, EPS, q1, s1, u1, stream=stream)
        ev[i % N_SETS][0].record(stream)
        b2s.ffn_gate_up_sqrelu_q8(ws["w_gate"][1], ws["w_up"][1], q1, s1, u1, P, stream=stream)
        ev[i % N_SETS][1].record(stream)
        b2s.rms_norm_act_quant(P, g2, EPS, q2, s2, u2, stream=stream)
        b2s.mul_mat_q8(ws["w_down"][1], q2, s2, u2, Y, stream=stream)

    with torch.cuda.stream(stream):
        for i in range(max(3, warmup)):
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
        for i in range(max(3, warmup)):
            graphs[i % N_SETS].replay()
    stream.synchronize()

    t_start, t_end = events()
    D.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            t_start.record(stream)
            for i in range(steps):
                graphs[i % N_SETS].replay()
            t_end.record(stream)
        torch.cuda.synchronize()
    D.barrier()
    ms = t_start.elapsed_time(t_end)
    assert b2s.device_error() == 0

    n_probe = max(2 * N_SETS, min(steps, 400))
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
    k_avg_ms = k_sum / k_n
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

    e2e_run(0, max(3, warmup))
    torch.cuda.synchronize()
    runs = [GSTEPS] * (steps // GSTEPS) + ([steps % GSTEPS] if steps % GSTEPS else [])
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
    e_start, e_end = events()
    D.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e_start.record(stream)
        for n in runs:
            e2e_graphs[n].replay()
        e_end.record(stream)
    torch.cuda.synchronize()
    D.barrier()
    e_ms = e_start.elapsed_time(e_end)
    assert b2s.device_error() == 0
    assert torch.isfinite(yh[(runs[-1] - 1) % NBUF]).all()
    for g in list(e2e_graphs.values()) + graphs + probes:
        g.reset()
    ms, e_ms = D.max([ms, e_ms])
    del sets, graphs, probes, e2e_graphs
    torch.cuda.empty_cache()

    peak, basis = int8_peak(burst=True)
    achieved = GATE_UP_OPS / (k_avg_ms * 1e-3) / 1e12
    traffic = None  # DRAM read+write bytes per gate/up launch from the committed ncu capture summary
    try:
        import re
        with open(os.path.join(ROOT, "profiles", "gemm_i2s_tc_ffn_block_m300.md")) as fh:
            mt = re.search(r"traffic_bytes_per_launch \(gate/up, read \+ write\): (\d+)", fh.read())
        traffic = int(mt.group(1)) if mt else None
    except OSError:
        pass
    value = world * steps * OPS_PER_STEP / (ms * 1e-3) / 1e12
    e2e = world * steps * OPS_PER_STEP / (e_ms * 1e-3) / 1e12
    return {
        "value": round(value, 3), "unit": "TOP/s", "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms / steps, 5), "scaling": "weak", "dtype": "int8xternary->int32 (fp32 in/out)",
        "config": ffn_config(world),
        "step": "b2s_ffn_block in a CUDA graph: rmsnorm+actquant, tcgen05 gate/up+sqrelu, rmsnorm+actquant, "
                "tcgen05 down (split-K through the workspace)",
        "e2e": {"value": round(e2e, 3), "unit": "TOP/s", "h2d_bytes_per_step": M * H * 4,
                "d2h_bytes_per_step": M * H * 4, "ms_per_step": round(e_ms / steps, 5),
                "api": "b2s_ffn_block (C ABI) with pinned host buffers",
                "pipeline": "3 streams, 3 device buffer slots: H2D(i+1) and D2H(i-1) overlap FFN(i); "
                            "CUDA graphs of 64 steps (the pipeline drains between graphs)"},
        "roofline": {"kernel": "gemm_i2s_tc_kernel (gate/up, mode 1)", "bound": "tensor",
                     "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TOP/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "avg_launch_us": round(k_avg_ms * 1e3, 3),
                     "launch_timing": f"CUDA events around the gate/up launch, {k_n} replays after the timed region",
                     "peak_basis": basis + " (launch timed alone)"},
        "gpu_launches": 4 * steps,
        "clocks": clk.summary(),
    }


def cpu_ffn_baseline(seconds: float):
    """The oracle's threaded port on full FFN blocks for about `seconds` (>= 2 iterations), rank 0, N=1."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    nthreads = cpu_threads()
    x, g1, g2, ws = ffn_host_inputs(1, oracle.i2s_pack_ternary)
    args = (x, g1, g2, EPS, ws[0], ws[1], ws[2], H, F, nthreads)
    oracle.fast_ffn_block(*args)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.fast_ffn_block(*args)
        n += 1
        dt = time.perf_counter() - t0
        if n >= 2 and dt >= seconds:
            break
    return {"value": round(n * OPS_PER_STEP / dt / 1e12, 5), "unit": "TOP/s", "cores": nthreads, "kind": "port",
            "sample": f"{n} full FFN blocks in {dt:.1f} s, {['scalar', 'AVX2', 'AVX512-VNNI'][oracle.fast_isa()]}, "
                      f"{cpu_model()}"}


def cpu_server_baseline():
    """Observations through the oracle's forward on all host threads, weights generated once beforehand
    (rank 0, N=1): one warm-up forward, then one timed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    nthreads = cpu_threads()
    model = oracle.BitVLAModel(oracle.bitvla_config(), SEED, nthreads)
    imgs, toks, _ = bitvla_inputs(2, 0)
    model.forward(imgs[:1], toks[:1])
    t_c = time.perf_counter()
    model.forward(imgs[1:], toks[1:])
    dt = time.perf_counter() - t_c
    model.close()
    return {"value": round(1.0 / dt, 5), "unit": "obs/s", "cores": nthreads, "kind": "port",
            "sample": f"1 observation (full forward, weights resident in host memory) in {dt:.1f} s on {nthreads} "
                      f"threads, {['scalar', 'AVX2', 'AVX512-VNNI'][oracle.fast_isa()]}, {cpu_model()}"}


# ------------------------------------------------------------------------------------------- config 0 and sweep
def rotating_weights(dev, K, N, seed):
    """Packed copies of one seeded ternary weight, rotated in bytes so that one pass over them streams more
    than 2x L2 from HBM; row-padded when K % 128 != 0."""
    import torch
    import b2s
    from b2s import workloads as wl
    w = wl.weight(wl.rng(seed), N, K)
    base = torch.from_numpy(w.packed).to(dev)
    Kp = (K + 127) // 128 * 128
    if K % 128:
        rb = torch.empty(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device=dev)
        b2s.repack_rows(base, rb, N, K)
        torch.cuda.synchronize()
        base = rb
    wbytes = N * Kp // 4
    R = max(2, min(256, -(-(2 * 126 * 2**20 + 8 * 2**20) // wbytes)))
    copies = []
    for r in range(R):
        b = base.clone()
        if r:
            b[:wbytes] = torch.roll(base[:wbytes], shifts=r * 4099)
        copies.append((b, b2s.i2s_tensor(b, N, K, rowpadded=bool(K % 128))))
    return copies, wbytes


def time_graph(fn, stream, launches, reps=5):
    """Per-launch µs of `fn` (which issues `launches` launches) replayed as one CUDA graph."""
    import torch
    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    stream.synchronize()
    e0, e1 = events()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    graph.reset()
    return e0.elapsed_time(e1) * 1e3 / (reps * launches)


def run_gemm_c0(local):
    """Config 0: one 2560x2560 i2_s MUL_MAT of 256 fp32 tokens (b2s_mul_mat, act-quant + GEMM, fp32 out)."""
    import torch
    import b2s
    dev = torch.device("cuda", local)
    Mt, K, N = 256, 2560, 2560
    copies, wbytes = rotating_weights(dev, K, N, 5)
    R = len(copies)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    x = torch.randn((Mt, K), device=dev, generator=g)
    y = torch.empty((Mt, N), dtype=torch.float32, device=dev)
    ws = torch.empty(b2s.mul_mat_workspace_size(copies[0][1], b2s.f32_tensor(x)), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def seq():
        for r in range(R):
            b2s.mul_mat(copies[r][1], x, y, ws, stream=stream)
    us = time_graph(seq, stream, R)
    assert b2s.device_error() == 0
    ops = 2.0 * Mt * N * K
    op_bytes = 4 * Mt * K + wbytes + 4 + 4 * Mt * N
    peak, basis = int8_peak(burst=True)
    hbm = peaks()[0]["hbm_gbs"]
    del copies
    torch.cuda.empty_cache()
    return {"workload": "single i2_s mul_mat, W 2560x2560, X 256x2560 fp32 N(0,1)", "api": "b2s_mul_mat",
            "us_per_call": round(us, 3), "TOP/s": round(ops / us / 1e6, 1),
            "GB/s_op_level": round(op_bytes / us / 1e3, 1), "frac_tensor": round(ops / us / 1e6 / peak, 4),
            "frac_hbm": round(op_bytes / us / 1e3 / hbm, 4),
            "timing": f"CUDA graph of {R} back-to-back calls over rotating weights, per-call average",
            "peak_basis": basis}


def batched_weights(dev, K, N, seed, min_bytes):
    """One i2_s tensor of R copies of a seeded weight back to back (rotated in bytes; shared scale trailer),
    R chosen so that the tensor holds more than min_bytes; row-padded when K % 128 != 0."""
    import torch
    import b2s
    from b2s import workloads as wl
    w = wl.weight(wl.rng(seed), N, K)
    base = torch.from_numpy(w.packed).to(dev)
    Kp = (K + 127) // 128 * 128
    if K % 128:
        rb = torch.empty(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device=dev)
        b2s.repack_rows(base, rb, N, K)
        torch.cuda.synchronize()
        base = rb
    wbytes = N * Kp // 4
    R = max(2, -(-min_bytes // wbytes))
    big = torch.empty(R * wbytes + 32, dtype=torch.uint8, device=dev)
    for r in range(R):
        big[r * wbytes:(r + 1) * wbytes] = torch.roll(base[:wbytes], shifts=r * 4099) if r else base[:wbytes]
    big[R * wbytes:] = base[wbytes:wbytes + 32]
    return big, b2s.i2s_tensor_batched(big, N, K, R, rowpadded=bool(K % 128)), R, wbytes


def run_sweep(local, ms_list=None, reps=5, kn_list=None, batched_only=False):
    """Config 4 on one GPU: per point TOP/s and algorithmic GB/s per launch of b2s_mul_mat_q8; for the decode
    sizes (M <= 16) also the batched form (b2s_mul_mat_q8_batched: one GEMV launch streaming R matrices of the
    shape, > 2x L2 of weights), per matrix."""
    import torch
    import b2s
    dev = torch.device("cuda", local)
    peak, basis = int8_peak(burst=True)
    hbm = peaks()[0]["hbm_gbs"]
    stream = torch.cuda.Stream(device=dev)
    rows = []
    for K, N in (kn_list or SWEEP_KN):
        copies, wbytes = rotating_weights(dev, K, N, K + N)
        R = len(copies)
        for Mt in (ms_list or SWEEP_M):
            if batched_only and Mt > 16:
                continue
            ldq = (K + 15) // 16 * 16
            q = torch.randint(-127, 128, (Mt, ldq), dtype=torch.int8, device=dev)[:, :K]
            s = torch.rand(Mt, device=dev) + 0.5
            u = q.to(torch.int32).sum(dim=1).to(torch.int32)
            y = torch.empty((Mt, N), dtype=torch.float32, device=dev)
            launches = R if Mt <= 4096 else max(2, min(R, 16))

            def seq():
                for r in range(launches):
                    b2s.mul_mat_q8(copies[r % R][1], q, s, u, y, stream=stream)
            us = time_graph(seq, stream, launches, reps) if not batched_only else float("nan")
            assert b2s.device_error() == 0
            ops = 2.0 * Mt * N * K
            byts = wbytes + Mt * K + 8 * Mt + 4 * Mt * N
            tops, gbs = ops / us / 1e6, byts / us / 1e3
            bound = "hbm" if Mt <= 16 else "tensor"
            row = {"M": Mt, "K": K, "N": N, "path": "gemv" if Mt <= 16 else "tcgen05", "us": round(us, 3),
                   "TOP/s": round(tops, 1), "GB/s": round(gbs, 1), "bound": bound,
                   "frac": round(gbs / hbm if bound == "hbm" else tops / peak, 4)}
            if Mt <= 16:
                big, Wb, Rb, _ = batched_weights(dev, K, N, K + N, 2 * 126 * 2**20 + 8 * 2**20)
                qb = torch.randint(-127, 128, (Rb, Mt, ldq), dtype=torch.int8, device=dev)[:, :, :K]
                sb = torch.rand((Rb, Mt), device=dev) + 0.5
                ub = qb.to(torch.int32).sum(dim=2).to(torch.int32)
                yb = torch.empty((Rb, Mt, N), dtype=torch.float32, device=dev)
                us_b = time_graph(lambda: b2s.mul_mat_q8_batched(Wb, qb, sb, ub, yb, stream=stream), stream, 1,
                                  reps) / Rb
                assert b2s.device_error() == 0
                row.update({"batched_matrices": Rb, "us_per_matrix_batched": round(us_b, 4),
                            "GB/s_batched": round(byts / us_b / 1e3, 1),
                            "frac_batched": round(byts / us_b / 1e3 / hbm, 4)})
                del big, qb, sb, ub, yb
            rows.append(row)
            del q, s, u, y
        del copies
        torch.cuda.empty_cache()
    return {"rows": rows, "peaks": f"HBM {hbm} GB/s; {basis}",
            "timing": "CUDA graph of back-to-back launches over rotating weight copies (> 2x L2 of weights per "
                      "pass), per-launch average; algorithmic bytes = N*Kp/4 + M*K + 8*M + 4*M*N"}


# ------------------------------------------------------------------------------------------- config 4: N-split
def run_nsplit(D, local, Mt=16384):
    """Each shape: every rank computes its output-row slice of W for all Mt tokens; compute-only writes the
    slice into a local [Mt, N] buffer, compute+gather into rank 0's buffer through b2s_peer_open (epilogue
    peer stores). Timing: max over ranks of 8 back-to-back launches. Rank 0 compares the gathered Y with its
    own single-GPU GEMM of the whole weight (bit-exact)."""
    import torch
    import b2s
    from b2s import workloads as wl
    from b2s.nsplit import PeerBuffer, nsplit_mul_mat_q8
    dev = torch.device("cuda", local)
    world, rank = D.world, D.rank
    peak, basis = int8_peak(burst=True)
    link_gbs = 770.0
    stream = torch.cuda.Stream(device=dev)
    rows = []
    launches = 8
    for K, N in SWEEP_KN:
        w = wl.weight(wl.rng(K + N), N, K)
        rp = bool(K % 128)
        full_host = w.packed
        full = torch.from_numpy(full_host).to(dev)
        if rp:  # row-padded first, then sharded by rows
            fr = torch.empty(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device=dev)
            b2s.repack_rows(full, fr, N, K)
            torch.cuda.synchronize()
            full = fr
            full_host = fr.cpu().numpy()
        n0, n1 = b2s.nsplit_range(N, world, rank)
        shard = torch.from_numpy(b2s.i2s_shard_rows(full_host, N, K, n0, n1, rowpadded=rp)).to(dev)
        W = b2s.i2s_tensor(shard, n1 - n0, K, rowpadded=rp)
        ldq = (K + 15) // 16 * 16
        gq = torch.Generator(device=dev)
        gq.manual_seed(K * 7 + N)  # same activations on every rank
        q = torch.randint(-127, 128, (Mt, ldq), dtype=torch.int8, device=dev, generator=gq)[:, :K]
        sc = torch.rand(Mt, device=dev, generator=gq) + 0.5
        u = q.to(torch.int32).sum(dim=1).to(torch.int32)
        local_y = torch.empty((Mt, N), dtype=torch.float32, device=dev)
        yb = PeerBuffer(Mt * N * 4)

        def timed(ptr):
            with torch.cuda.stream(stream):
                for _ in range(2):
                    nsplit_mul_mat_q8(b2s, W, q, sc, u, Mt, ptr, N, n0, stream=stream)
            stream.synchronize()
            D.barrier()
            e0, e1 = events()
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(launches):
                    nsplit_mul_mat_q8(b2s, W, q, sc, u, Mt, ptr, N, n0, stream=stream)
                e1.record(stream)
            stream.synchronize()
            D.barrier()
            return D.max([e0.elapsed_time(e1)])[0] * 1e3 / launches

        us_local = timed(local_y.data_ptr())
        us_gather = timed(yb.ptr)
        assert b2s.device_error() == 0
        exact = True
        if rank == 0:
            y1 = torch.empty((Mt, N), dtype=torch.float32, device=dev)
            b2s.mul_mat_q8(b2s.i2s_tensor(full, N, K, rowpadded=rp), q, sc, u, y1, path=2, stream=stream)
            stream.synchronize()
            exact = bool(torch.equal(yb.tensor((Mt, N), torch.float32), y1))
            del y1
        exact = D.max([0.0 if exact else 1.0])[0] == 0.0
        ops = 2.0 * Mt * N * K
        cross = 4.0 * Mt * (N - b2s.nsplit_range(N, world, 0)[1])  # fp32 columns stored into rank 0 by peers
        t_roof = max(ops / (peak * 1e12) * 1e6, cross / (link_gbs * 1e9) * 1e6)
        rows.append({"M": Mt, "K": K, "N": N, "gpus": world, "compute_only_us": round(us_local, 2),
                     "compute_plus_gather_us": round(us_gather, 2),
                     "TOP/s_compute_only": round(ops / us_local / 1e6, 1),
                     "TOP/s_with_gather": round(ops / us_gather / 1e6, 1), "bitexact": exact,
                     "nvlink_bytes_into_root": int(cross), "roofline_us": round(t_roof, 2),
                     "frac": round(t_roof / us_gather, 4),
                     "bound": "nvlink" if cross / (link_gbs * 1e9) > ops / (peak * 1e12) else "tensor"})
        D.barrier()
        yb.close()
        del q, sc, u, shard, local_y, full
        torch.cuda.empty_cache()
    return {"rows": rows, "all_bitexact": all(r["bitexact"] for r in rows),
            "method": "weight rows split over the GPUs (b2s_nsplit_range, b2s_i2s_shard_rows); rank 0's output "
                      "mapped into every rank (b2s_peer_export/open); each epilogue stores its column slice "
                      "straight into it (plain peer stores, no multicast, no collective)",
            "roofline": f"max(ops / {peak:.0f} TOP/s, bytes into rank 0 / {link_gbs} GB/s NVLink per direction)"}


# ------------------------------------------------------------------------------------------- drivers
def setup(world, rank, local):
    import torch
    import b2s
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    b2s.check(b2s.lib().b2s_device_check())
    return Dist(world, rank, dev), dev


def main_server(a, world, rank, local):
    D, dev = setup(world, rank, local)
    line, m_tokens = run_server(a, D, local)
    if not a.no_extras:
        line["roofline"] = gemm_roofline(dev, m_tokens)
        line["ffn_block"] = run_ffn(a, D, local, steps=2000, warmup=20)
        if world == 1:
            line["gemm_c0"] = run_gemm_c0(local)
            line["sweep"] = run_sweep(local)
        else:
            line["nsplit"] = run_nsplit(D, local)
    D.close()
    if rank != 0:
        return
    if world == 1:
        line["cpu_baseline"] = cpu_server_baseline()
        if "ffn_block" in line:
            line["ffn_block"]["cpu_baseline"] = cpu_ffn_baseline(a.cpu_seconds)
    print(json.dumps(line), flush=True)


def main_ffn(a, world, rank, local):
    D, _ = setup(world, rank, local)
    sub = run_ffn(a, D, local, steps=a.steps, warmup=a.warmup)
    D.close()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": sub.pop("value"), "unit": sub.pop("unit"), "n_gpus": world,
            "steps": sub.pop("steps"), "warmup": sub.pop("warmup"), "ms_per_step": sub.pop("ms_per_step"),
            "higher_is_better": True, "scaling": sub.pop("scaling"), "vs_baseline": None, "dtype": sub.pop("dtype"),
            "data": "synthetic (seeded random-init ternary weights, N(0,1) activations)"}
    line.update(sub)
    if world == 1:
        line["cpu_baseline"] = cpu_ffn_baseline(a.cpu_seconds)
    print(json.dumps(line), flush=True)


def main_sweep(a, world, rank, local):
    D, _ = setup(world, rank, local)
    if world > 1:
        sub = run_nsplit(D, local)
        D.close()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": round(sum(r["TOP/s_with_gather"] for r in sub["rows"]) /
                                                               len(sub["rows"]), 1),
                              "unit": "TOP/s (mean over shapes, whole job, with gather)", "n_gpus": world,
                              "steps": 8, "warmup": 2, "higher_is_better": True, "scaling": "strong",
                              "vs_baseline": None, "dtype": "int8xternary->int32", "data": "synthetic",
                              "config": {"workload": "i2s_gemm_nsplit_m16384"}, "nsplit": sub}), flush=True)
        return
    D.close()
    ms_list = [int(x) for x in a.sweep_m.split(",")] if a.sweep_m else None
    kn_list = [tuple(int(v) for v in s_.split("x")) for s_ in a.sweep_kn.split(",")] if a.sweep_kn else None
    sub = run_sweep(local, ms_list, kn_list=kn_list, batched_only=a.batched_only)
    big = [r["TOP/s"] for r in sub["rows"] if r["M"] >= 4096]
    print(json.dumps({"metric": METRIC, "value": round(sum(big) / max(1, len(big)), 1),
                      "unit": "TOP/s (mean over M >= 4096)", "n_gpus": 1, "steps": 5, "warmup": 3,
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "int8xternary->int32", "data": "synthetic (ternary P(0)=0.4, random int8 activations)",
                      "config": {"workload": "i2s_gemm_sweep"}, "sweep": sub}), flush=True)


def main_roofline(a, world, rank, local):
    D, dev = setup(world, rank, local)
    r = gemm_roofline(dev, a.obs_batch * 288)
    D.close()
    if rank == 0:
        print(json.dumps({"metric": METRIC, "value": r["achieved"], "unit": r["unit"], "n_gpus": 1, "steps": 128,
                          "warmup": 32, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "int8xternary->int32", "data": "synthetic",
                          "config": {"workload": "gemm_gate_up_m2304"}, "roofline": r}), flush=True)


def main():
    a = parse()
    world, rank, local = dist_env()
    if a.impl == "reference":
        run_reference(a, world, rank)
    elif a.workload == "roofline":
        main_roofline(a, world, rank, local)
    elif a.workload == "sweep":
        main_sweep(a, world, rank, local)
    elif a.workload == "ffn":
        main_ffn(a, world, rank, local)
    else:
        main_server(a, world, rank, local)


if __name__ == "__main__":
    main()
