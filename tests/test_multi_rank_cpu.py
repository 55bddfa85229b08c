"""Multi-rank host logic on CPU (gloo, world size 2): row sharding of i2_s weights for the N-split GEMM,
the gather of the ranks' column slices, data-parallel sharding, and failure detection on the host (a rank
that never joins a collective ends the other's wait with an error instead of a hang)."""
import datetime
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_ranges_properties():
    from b2s.nsplit import row_ranges, shard_range
    for n, g in [(2560, 2), (4304, 8), (6912, 4), (7, 8), (0, 3)]:
        rr = row_ranges(n, g)
        assert len(rr) == g and rr[0][0] == 0 and rr[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rr, rr[1:]))
        sizes = [b - a for a, b in rr]
        assert max(sizes) - min(sizes) <= 1
    assert row_ranges(4304, 8)[0] == (0, 538)
    assert shard_range(64, 3, 8) == (24, 32)
    with pytest.raises(ValueError):
        row_ranges(10, 0)


def test_shard_i2s_rows_matches_oracle(orc):
    from b2s import workloads as wl
    from b2s.nsplit import row_ranges, shard_i2s_rows
    g = wl.rng(11)
    N, K = 100, 256
    t = wl.ternary(g, N, K)
    packed = orc.i2s_pack_ternary(t, 1.75)
    for n0, n1 in row_ranges(N, 3):
        sh = shard_i2s_rows(packed, N, K, n0, n1)
        ts, sc = orc.i2s_unpack_ternary(sh, n1 - n0, K)
        assert sc == np.float32(1.75) and np.array_equal(ts, t[n0:n1])
    import b2s
    with pytest.raises(b2s.B2SError):
        shard_i2s_rows(packed, N, 100, 0, 10)  # flattened rows of K % 128 != 0 are not separable
    with pytest.raises(b2s.B2SError):
        shard_i2s_rows(packed, N, K, 5, 5)


def test_shard_rowpadded_rows_matches_oracle(orc):
    """K % 128 != 0 (the ViT FFN width): shards are cut from the row-padded layout (I2_S_R)."""
    from b2s import workloads as wl
    from b2s.nsplit import row_ranges, shard_i2s_rows
    g = wl.rng(12)
    N, K = 64, 4304
    t = wl.ternary(g, N, K)
    rp = orc.i2s_to_rowpadded(orc.i2s_pack_ternary(t, 0.625), N, K)
    Kp = (K + 127) // 128 * 128
    for n0, n1 in row_ranges(N, 4):
        sh = shard_i2s_rows(rp, N, K, n0, n1, rowpadded=True)
        assert sh.size == (n1 - n0) * Kp // 4 + 32
        assert np.array_equal(sh[:-32], rp[n0 * Kp // 4: n1 * Kp // 4]) and np.array_equal(sh[-32:], rp[-32:])


def _nsplit_worker(rank, world, port, out_q):
    import sys
    for p in (os.path.join(ROOT, "robot.cpp_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import oracle
    from b2s import workloads as wl
    from b2s.nsplit import row_ranges, shard_i2s_rows
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = wl.rng(21)
        M, N, K = 9, 90, 384  # N not a multiple of the world size
        w = wl.weight(g, N, K)
        x = wl.activations(g, M, K)
        n0, n1 = row_ranges(N, world)[rank]
        shard = shard_i2s_rows(w.packed, N, K, n0, n1)
        y_local = oracle.mul_mat_i2s(shard, x, n1 - n0)        # this rank's column slice
        n_max = max(b - a for a, b in row_ranges(N, world))
        pad = torch.zeros((M, n_max), dtype=torch.float32)
        pad[:, : n1 - n0] = torch.from_numpy(y_local)
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        y = torch.cat([p[:, : b - a] for p, (a, b) in zip(parts, row_ranges(N, world))], dim=1).numpy()
        if rank == 0:
            out_q.put(bool(np.array_equal(y, oracle.mul_mat_i2s(w.packed, x, N))))
    finally:
        dist.destroy_process_group()


def _failing_worker(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            return  # this rank fails between steps: it never joins the collective
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            out_q.put("completed")
        except Exception as e:  # the bounded wait ends with an error the host can act on
            out_q.put(f"error:{type(e).__name__}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(fn, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    return q


def test_nsplit_gather_gloo():
    q = _spawn(_nsplit_worker)
    assert q.get(timeout=10) is True


def test_rank_failure_is_detected_on_host():
    q = _spawn(_failing_worker)
    msg = q.get(timeout=30)
    assert msg.startswith("error:"), msg
