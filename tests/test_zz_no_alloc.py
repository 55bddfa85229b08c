"""b2s_mul_mat_static: the MUL_MAT entry point for callers that cannot allocate device memory.

Such callers are an op running inside a ggml backend's compute step, which receives no allocator because
the scheduler allocated every buffer up front, and a robot control loop past start-up, which must not
call cudaMalloc since it can synchronize the device and adds latency jitter to each control period. The
entry point takes no workspace; its scratch is a library-owned static device array (4 MiB per device).

This file is named to be collected last, so a run that stops at the first failure has already run every
other test. It must pass on its own in a fresh process and after the rest of the suite.
"""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from b2s import workloads as wl  # noqa: E402

TOL = 1e-5  # max |y - y_ref| / max |y_ref|, the bar the other parity tests use (then bit-exact)


def max_abs_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


def case(b2s, seed, M, K, N):
    g = wl.rng(seed)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    buf = torch.from_numpy(w.packed).cuda()
    return buf, b2s.i2s_tensor(buf, N, K), torch.from_numpy(x).cuda(), w, x


def with_workspace(b2s, W, x, N):
    """The existing entry point, b2s_mul_mat, with a caller-owned workspace."""
    y = torch.empty((x.shape[0], N), dtype=torch.float32, device="cuda")
    ws = torch.empty(b2s.mul_mat_workspace_size(W, b2s.f32_tensor(x)), dtype=torch.uint8, device="cuda")
    b2s.mul_mat(W, x, y, ws)
    return y


def without_workspace(b2s, W, x, N):
    """The new entry point through the C ABI: no workspace argument."""
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float32, device="cuda")
    X, Y = b2s.f32_tensor(x), b2s.f32_tensor(y)
    rc = b2s.lib().b2s_mul_mat_static(C.byref(W), C.byref(X), C.byref(Y),
                                      int(torch.cuda.current_stream().cuda_stream))
    assert rc == b2s.B2S_OK, b2s.last_error()
    return y


def test_static_scratch_matches_oracle_and_workspace_entry_point(b2s, orc):
    # Shapes in a row: a prefill-size call (tensor-core GEMM; N = 640 leaves few tiles, so split-K partials use
    # the array's free room), a decode-size call (GEMV), then the first again; each reads scratch the previous
    # call left behind in the shared array. Results equal the oracle and b2s_mul_mat bit for bit (int32 sums
    # are exact and the fp32 rescale is the same operation on both paths).
    shapes = [(11, 300, 2560, 640), (12, 5, 6912, 2560), (11, 300, 2560, 640)]
    for seed, M, K, N in shapes:
        buf, W, xd, w, x = case(b2s, seed, M, K, N)
        ref = orc.fast_mul_mat_i2s(w.packed, x, N, os.cpu_count() or 8)
        for _ in range(2):  # two calls in a row through the new entry point
            y_new = without_workspace(b2s, W, xd, N)
            torch.cuda.synchronize()
            assert b2s.device_error() == 0
            a = y_new.cpu().numpy()
            assert np.isfinite(a).all()
            assert max_abs_rel(a, ref) <= TOL
            assert np.array_equal(a, ref)
        y_old = with_workspace(b2s, W, xd, N)
        torch.cuda.synchronize()
        assert torch.equal(y_new, y_old)


def test_static_scratch_rejects_oversize_calls(b2s):
    # 2048 tokens x K=2560 needs ~5.2 MB of scratch, above the 4 MiB static array: refused, nothing launched.
    buf, W, x, _, _ = case(b2s, 13, 2048, 2560, 256)
    y = torch.zeros((2048, 256), dtype=torch.float32, device="cuda")
    X, Y = b2s.f32_tensor(x), b2s.f32_tensor(y)
    rc = b2s.lib().b2s_mul_mat_static(C.byref(W), C.byref(X), C.byref(Y), None)
    assert rc == b2s.B2S_ERR_WORKSPACE
    assert "static limit" in b2s.last_error()
    torch.cuda.synchronize()
    assert not y.any()


def test_static_scratch_errors_match_workspace_entry_point(b2s):
    """Malformed operands get the same status from both entry points (and nothing is launched)."""
    buf, W, x, _, _ = case(b2s, 14, 8, 256, 128)
    y = torch.zeros((8, 128), dtype=torch.float32, device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    bad_x = b2s.f32_tensor(x)
    bad_x.type = b2s.TYPE_I32                      # X not f32 -> unsupported
    bad_w = b2s.i2s_tensor(buf, 128, 256)
    bad_w.data = int(buf.data_ptr()) + 4           # W not 16-byte aligned -> unsupported
    short_w = b2s.i2s_tensor(buf, 128, 256)
    short_w.ne[0] = 200                            # K % 16 != 0 -> unsupported
    for Wd, Xd in ((W, bad_x), (bad_w, b2s.f32_tensor(x)), (short_w, b2s.f32_tensor(x))):
        Y = b2s.f32_tensor(y)
        rc_static = b2s.lib().b2s_mul_mat_static(C.byref(Wd), C.byref(Xd), C.byref(Y), None)
        msg_static = b2s.last_error()
        rc_ws = b2s.lib().b2s_mul_mat(C.byref(Wd), C.byref(Xd), C.byref(Y), ws.data_ptr(), ws.numel(), None)
        assert rc_static == rc_ws == b2s.B2S_ERR_UNSUPPORTED, (rc_static, rc_ws, msg_static)
        assert msg_static == b2s.last_error()
    torch.cuda.synchronize()
    assert not y.any()
