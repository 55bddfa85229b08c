"""N-split i2_s GEMM on 2 GPUs with the output gather fused into the epilogue (peer stores over NVLink
into the root's buffer through CUDA IPC). Skipped on boxes with fewer than two GPUs.

Parity: at M=512 against the oracle (bit-exact); at the sweep's M=16384 the gathered result must equal
the single-GPU tensor-core GEMM bit for bit (the single-GPU path is itself parity-tested).
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        return torch.cuda.device_count()
    except Exception:
        return 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases, out_q):
    import sys
    for p in (os.path.join(ROOT, "robot.cpp_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    import b2s
    import oracle
    from b2s import workloads as wl
    from b2s.nsplit import PeerBuffer, nsplit_mul_mat_q8, row_ranges, shard_i2s_rows
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    results = []
    try:
        for (M, K, N, check) in cases:
            g = wl.rng(M + K + N)
            w = wl.weight(g, N, K)
            x = wl.activations(g, M, K)
            n0, n1 = row_ranges(N, world)[rank]
            shard = torch.from_numpy(shard_i2s_rows(w.packed, N, K, n0, n1)).cuda()
            W_local = b2s.i2s_tensor(shard, n1 - n0, K)
            xd = torch.from_numpy(x).cuda()
            ldq = (K + 15) // 16 * 16
            q = torch.empty((M, ldq), dtype=torch.int8, device="cuda")[:, :K]
            s = torch.empty(M, dtype=torch.float32, device="cuda")
            u = torch.empty(M, dtype=torch.int32, device="cuda")
            b2s.act_quant(xd, q, s, u)
            buf = PeerBuffer(M * N * 4, root=0)
            nsplit_mul_mat_q8(b2s, W_local, q, s, u, M, buf.ptr, N, n0)
            torch.cuda.synchronize()
            assert b2s.device_error() == 0
            dist.barrier()
            if rank == 0:
                y = buf.tensor((M, N), torch.float32).cpu().numpy()
                if check == "oracle":
                    ok = bool(np.array_equal(y, oracle.fast_mul_mat_i2s(w.packed, x, N, 8)))
                else:  # equal to the unsplit single-GPU GEMM
                    full = torch.from_numpy(w.packed).cuda()
                    y1 = torch.empty((M, N), dtype=torch.float32, device="cuda")
                    b2s.mul_mat_q8(b2s.i2s_tensor(full, N, K), q, s, u, y1, path=2)
                    torch.cuda.synchronize()
                    ok = bool(np.array_equal(y, y1.cpu().numpy()))
                results.append((M, K, N, ok))
            dist.barrier()
            buf.close()
        if rank == 0:
            out_q.put(results)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_nsplit_two_gpus_fused_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    cases = [(512, 2560, 2560, "oracle"), (300, 1152, 4304, "oracle"), (16384, 2560, 2560, "unsplit")]
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=10)
    assert len(res) == len(cases) and all(r[3] for r in res), res
