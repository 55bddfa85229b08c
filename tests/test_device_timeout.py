"""Failure detection on the device, without a fault: a kernel's bounded mbarrier wait runs out.

b2s_debug_wait_timeout launches one CTA that holds tensor memory and has a bulk copy in flight, then waits on
an mbarrier that nothing arrives at, bounded by a 1 ms limit. The kernel must return on its own, the device
error word must show bit 0 (a pipeline wait gave up) and not bit 1 (its drain wait completed), and the
tensor memory must have been released: a tensor-core GEMM launched afterwards still runs and matches the
oracle bit for bit. Nothing here faults, traps or hangs the GPU; the wait is bounded by %globaltimer.
"""
import os
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from b2s import workloads as wl  # noqa: E402


def test_bounded_wait_runs_out_and_context_stays_usable(b2s, orc):
    src = torch.arange(4096, dtype=torch.int32, device="cuda").to(torch.uint8)
    torch.cuda.synchronize()
    b2s.device_error(clear=True)
    t0 = time.perf_counter()
    b2s.debug_wait_timeout(src, 1_000_000)  # 1 ms
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    bits = b2s.device_error(clear=True)
    assert bits == 1, bits  # the pipeline wait gave up; the drain of the in-flight copy completed
    assert dt < 0.5, dt     # returned on its own, well inside the one-second default bound
    assert b2s.device_error() == 0  # cleared
    # The CTA freed its tensor memory: a tcgen05 GEMM (which allocates TMEM on every SM it runs on) completes
    # and is exact.
    M, K, N = 300, 2560, 640
    g = wl.rng(901)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    buf = torch.from_numpy(w.packed).cuda()
    W = b2s.i2s_tensor(buf, N, K)
    ldq = (K + 15) // 16 * 16
    q = torch.zeros((M, ldq), dtype=torch.int8, device="cuda")[:, :K]
    s = torch.zeros(M, dtype=torch.float32, device="cuda")
    u = torch.zeros(M, dtype=torch.int32, device="cuda")
    b2s.act_quant(torch.from_numpy(x).cuda(), q, s, u)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2s.mul_mat_q8(W, q, s, u, y, path=2)
    torch.cuda.synchronize()
    assert b2s.device_error() == 0
    assert np.array_equal(y.cpu().numpy(), orc.fast_mul_mat_i2s(w.packed, x, N, os.cpu_count() or 8))


def test_wait_probe_rejects_bad_arguments(b2s):
    src = torch.zeros(64, dtype=torch.uint8, device="cuda")
    for args in ((src[:20], 1000), (src, 0), (src, 2_000_000_000)):
        with pytest.raises(b2s.B2SError):
            b2s.debug_wait_timeout(*args)
