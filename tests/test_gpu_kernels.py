"""Parity of the CUDA path (through the C ABI) against the oracle, on a B200.

Bars: int8 activations, scales, sums and int32 accumulators bit-exact; fp32 outputs compared with
max-abs-rel <= 1e-5 (max |y - y_ref| / max |y_ref|) and, because every fp32 step is restated with the
same IEEE operations in the same order, also checked for exact equality where stated. The softmax's exp
is the library's deterministic det_expf on both sides, so softmax is compared exactly too.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

from b2s import workloads as wl  # noqa: E402

TOL = 1e-5


def max_abs_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weight_dev(b2s, w):
    buf = dev(w.packed)
    return buf, b2s.i2s_tensor(buf, w.N, w.K)


def q8_buffers(M, K):
    ldq = (K + 15) // 16 * 16
    q = torch.zeros((M, ldq), dtype=torch.int8, device="cuda")[:, :K]
    s = torch.zeros(M, dtype=torch.float32, device="cuda")
    u = torch.zeros(M, dtype=torch.int32, device="cuda")
    return q, s, u


def sync_ok(b2s):
    torch.cuda.synchronize()
    assert b2s.device_error() == 0


# ------------------------------------------------------------------------------------------ act-quant
@pytest.mark.parametrize("M,K", [(1, 2560), (37, 2560), (5, 6912), (3, 99), (4, 4304)])
def test_act_quant_bit_exact(b2s, orc, M, K):
    g = wl.rng(100 + M + K)
    x = wl.activations(g, M, K)
    x[0, :] = 0.0                      # all-zero row: the 1e-5 amax floor
    if M > 2:
        x[1, :] *= 1e-7                # every |x| below the floor
        x[2, 3] = 127.0 * 3            # ties: amax 381 -> s = 1/3 ...
    q, s, u = q8_buffers(M, K)
    xd = dev(x)
    b2s.act_quant(xd, q, s, u)
    sync_ok(b2s)
    q_ref, s_ref, u_ref = orc.act_quant(x)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(u.cpu().numpy(), u_ref)


def test_act_quant_kat(b2s):
    import os
    kat = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat.npz"))
    x = kat["x_actq"]
    q, s, u = q8_buffers(*x.shape)
    b2s.act_quant(dev(x), q, s, u)
    sync_ok(b2s)
    assert np.array_equal(q.cpu().numpy(), kat["q_actq"])
    assert np.array_equal(s.cpu().numpy(), kat["s_actq"])
    assert np.array_equal(u.cpu().numpy(), kat["sum_actq"])


@pytest.mark.parametrize("M,K", [(3, 2560), (300, 2560), (17, 6912), (2, 1152)])
def test_rms_norm_act_quant_bit_exact(b2s, orc, M, K):
    g = wl.rng(200 + M + K)
    x = wl.activations(g, M, K) * 3.0
    w = wl.norm_weight(g, K)
    q, s, u = q8_buffers(M, K)
    b2s.rms_norm_act_quant(dev(x), dev(w), 1e-5, q, s, u)
    sync_ok(b2s)
    xn = orc.rms_norm(x, w, 1e-5)
    q_ref, s_ref, u_ref = orc.act_quant(xn)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(u.cpu().numpy(), u_ref)


# ------------------------------------------------------------------------------------------ GEMM / GEMV
def run_q8(b2s, orc, M, K, N, path, seed):
    g = wl.rng(seed)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    buf, W = weight_dev(b2s, w)
    q, s, u = q8_buffers(M, K)
    b2s.act_quant(dev(x), q, s, u)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2s.mul_mat_q8(W, q, s, u, y, path=path)
    sync_ok(b2s)
    q_ref, s_ref, _ = orc.act_quant(x)
    if M * N * K <= 64 * 1024 * 1024:
        acc = orc.gemm_i32(w.t, q_ref)
        y_ref = orc.rescale(acc, s_ref, float(w.scale))
    else:
        y_ref = orc.fast_mul_mat_i2s(w.packed, x, N, os.cpu_count() or 8)
    return y.cpu().numpy(), y_ref


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 13, 16, 21])
@pytest.mark.parametrize("K,N", [(2560, 2560), (1152, 4304), (256, 40), (6912, 2560)])
def test_gemv_path(b2s, orc, M, K, N):
    y, y_ref = run_q8(b2s, orc, M, K, N, path=1, seed=M * 7 + K + N)
    assert max_abs_rel(y, y_ref) <= TOL
    assert np.array_equal(y, y_ref)


@pytest.mark.parametrize("M", [1, 16, 37, 256, 300])
@pytest.mark.parametrize("K,N", [(128, 128), (384, 200), (2560, 2560), (1152, 4304), (6912, 2560)])
def test_tensor_core_path(b2s, orc, M, K, N):
    y, y_ref = run_q8(b2s, orc, M, K, N, path=2, seed=M * 11 + K + N)
    assert max_abs_rel(y, y_ref) <= TOL
    assert np.array_equal(y, y_ref)


@pytest.mark.parametrize("M,K,N", [(4096, 2560, 2560), (600, 2560, 6912), (513, 6912, 2560)])
def test_tensor_core_large(b2s, orc, M, K, N):
    y, y_ref = run_q8(b2s, orc, M, K, N, path=2, seed=M + K + N)
    assert max_abs_rel(y, y_ref) <= TOL
    assert np.array_equal(y, y_ref)


@pytest.mark.parametrize("M,K,N", [(16384, 2560, 2560), (16384, 2560, 6912), (16384, 6912, 2560),
                                   (16384, 1152, 4304), (4096, 1152, 4304)])
def test_persistent_gemm_sweep_sizes(b2s, orc, M, K, N):
    """The roofline sweep's large points through the automatic path (the persistent tcgen05 kernel), bit for
    bit against the oracle: every (K, N) of the sweep at M = 16384, and the K = 1152 ViT FFN shape at 4096."""
    y, y_ref = run_q8(b2s, orc, M, K, N, path=0, seed=M + 3 * K + N)
    assert max_abs_rel(y, y_ref) <= TOL
    assert np.array_equal(y, y_ref)


@pytest.mark.parametrize("M", [1, 16, 256])
def test_mul_mat_op_config0(b2s, orc, M):
    """The MUL_MAT node through ggml-style descriptors (f32 X in, f32 Y out), 2560x2560 weight."""
    K = N = 2560
    g = wl.rng(300 + M)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    buf, W = weight_dev(b2s, w)
    xd = dev(x)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    X = b2s.f32_tensor(xd)
    ws = torch.empty(b2s.mul_mat_workspace_size(W, X), dtype=torch.uint8, device="cuda")
    b2s.mul_mat(W, xd, y, ws)
    sync_ok(b2s)
    y_ref = orc.fast_mul_mat_i2s(w.packed, x, N, 8)
    assert max_abs_rel(y.cpu().numpy(), y_ref) <= TOL
    assert np.array_equal(y.cpu().numpy(), y_ref)


@pytest.mark.parametrize("M,K,N", [(300, 6912, 2560), (37, 2560, 2560), (129, 1152, 4304), (20, 2560, 640),
                                   (300, 2560, 1280), (250, 6912, 128)])
def test_mul_mat_splitk_workspace(b2s, orc, M, K, N):
    """MUL_MAT with a workspace at tile counts below the SM count: split-K over a cluster with the int32
    partial tiles exchanged through the workspace in L2 (a workspace holding stale bytes must not matter)."""
    g = wl.rng(700 + M + K + N)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    buf, W = weight_dev(b2s, w)
    xd = dev(x)
    X = b2s.f32_tensor(xd)
    ws = torch.full((b2s.mul_mat_workspace_size(W, X),), 0x5A, dtype=torch.uint8, device="cuda")  # not zero
    y_ref = orc.fast_mul_mat_i2s(w.packed, x, N, 8)
    for _ in range(2):  # the second call finds the first call's partials in the workspace
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        b2s.mul_mat(W, xd, y, ws)
        sync_ok(b2s)
        assert np.array_equal(y.cpu().numpy(), y_ref)


@pytest.mark.parametrize("M", [2, 11, 16])
def test_gemv_mma_ragged_k(b2s, orc, M):
    """The 2..16-token GEMV with K = 208 (row-padded to 256) and an activation row stride of 212 bytes (not a
    multiple of 16: byte-wise staging), at token counts that leave part of the last 8-token MMA tile empty."""
    K, N = 208, 64
    g = wl.rng(450 + M)
    w = wl.weight(g, N, K)
    src = dev(w.packed)
    dst = torch.zeros(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device="cuda")
    b2s.repack_rows(src, dst, N, K)
    W = b2s.i2s_tensor(dst, N, K, rowpadded=True)
    x = wl.activations(g, M, K)
    q = torch.zeros((M, K + 4), dtype=torch.int8, device="cuda")[:, :K]
    s = torch.zeros(M, dtype=torch.float32, device="cuda")
    u = torch.zeros(M, dtype=torch.int32, device="cuda")
    b2s.act_quant(dev(x), q, s, u)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2s.mul_mat_q8(W, q, s, u, y, path=1)
    sync_ok(b2s)
    assert np.array_equal(y.cpu().numpy(), orc.mul_mat_i2s(w.packed, x, N))


def test_repack_rows_and_mul_mat(b2s, orc):
    """K % 128 != 0 (ViT FFN down 4304 -> 1152 shape, fewer rows): flattened i2_s -> row-padded."""
    K, N, M = 4304, 64, 20
    g = wl.rng(400)
    w = wl.weight(g, N, K)
    src = dev(w.packed)
    dst = torch.zeros(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device="cuda")
    b2s.repack_rows(src, dst, N, K)
    sync_ok(b2s)
    assert np.array_equal(dst.cpu().numpy(), orc.i2s_to_rowpadded(w.packed, N, K))
    W = b2s.i2s_tensor(dst, N, K, rowpadded=True)
    x = wl.activations(g, M, K)
    for path in (1, 2):
        q, s, u = q8_buffers(M, K)
        b2s.act_quant(dev(x), q, s, u)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        b2s.mul_mat_q8(W, q, s, u, y, path=path)
        sync_ok(b2s)
        assert np.array_equal(y.cpu().numpy(), orc.mul_mat_i2s(w.packed, x, N))


# ------------------------------------------------------------------------------------------ FFN
def test_gate_up_sqrelu(b2s, orc):
    M, H, F = 45, 2560, 640
    g = wl.rng(500)
    wg, wu = wl.weight(g, F, H), wl.weight(g, F, H)
    x = wl.activations(g, M, H)
    bg, Wg = weight_dev(b2s, wg)
    bu, Wu = weight_dev(b2s, wu)
    q, s, u = q8_buffers(M, H)
    b2s.act_quant(dev(x), q, s, u)
    p = torch.empty((M, F), dtype=torch.float32, device="cuda")
    b2s.ffn_gate_up_sqrelu_q8(Wg, Wu, q, s, u, p)
    sync_ok(b2s)
    p_ref = orc.sqrelu_mul(orc.mul_mat_i2s(wg.packed, x, F), orc.mul_mat_i2s(wu.packed, x, F))
    assert np.array_equal(p.cpu().numpy(), p_ref)


@pytest.mark.parametrize("M,F,pad", [(300, 6912, 0), (203, 6880, 0), (300, 6912, 3), (17, 6912, 0)])
def test_gate_up_sqrelu_tiles(b2s, orc, M, F, pad):
    """Gate/up at tile counts that fill the GPU without split-K: the staged epilogue (shared-memory tile,
    TMA stores that drop rows past M and columns past F), and with a row stride that is not a multiple of
    16 bytes (pad=3) the direct-store epilogue."""
    H = 2560
    g = wl.rng(510 + M + pad)
    wg, wu = wl.weight(g, F, H), wl.weight(g, F, H)
    x = wl.activations(g, M, H)
    bg, Wg = weight_dev(b2s, wg)
    bu, Wu = weight_dev(b2s, wu)
    q, s, u = q8_buffers(M, H)
    b2s.act_quant(dev(x), q, s, u)
    full = torch.full((M, F + pad), 7.0, dtype=torch.float32, device="cuda")
    p = full[:, :F]
    b2s.ffn_gate_up_sqrelu_q8(Wg, Wu, q, s, u, p)
    sync_ok(b2s)
    p_ref = orc.sqrelu_mul(orc.fast_mul_mat_i2s(wg.packed, x, F, 8), orc.fast_mul_mat_i2s(wu.packed, x, F, 8))
    assert np.array_equal(p.cpu().numpy(), p_ref)
    assert bool(full[:, F:].eq(7.0).all())  # nothing written past the F columns of a row


@pytest.mark.parametrize("M", [300, 7])
def test_ffn_block_config1(b2s, orc, M):
    """BitNet-b1.58-2B FFN block (H=2560, F=6912), prefill M=300 and a decode-size M."""
    f = wl.ffn_block(seed=600 + M, M=M)
    bufs = [weight_dev(b2s, w) for w in (f.w_gate, f.w_up, f.w_down)]
    y = torch.empty((M, f.H), dtype=torch.float32, device="cuda")
    ws = torch.empty(b2s.ffn_block_workspace_size(M, f.H, f.F), dtype=torch.uint8, device="cuda")
    b2s.ffn_block(dev(f.x), dev(f.g1), dev(f.g2), f.eps, bufs[0][1], bufs[1][1], bufs[2][1], y, ws)
    sync_ok(b2s)
    y_ref = orc.fast_ffn_block(f.x, f.g1, f.g2, f.eps, f.w_gate.packed, f.w_up.packed, f.w_down.packed, f.H, f.F, 8)
    assert max_abs_rel(y.cpu().numpy(), y_ref) <= TOL
    assert np.array_equal(y.cpu().numpy(), y_ref)


def test_ffn_tiny_golden(b2s):
    import os
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "ffn_tiny.npz"))
    M, H = d["x"].shape
    F = d["g2"].shape[0]
    Ws = []
    for k, (n, kk) in (("w_gate", (F, H)), ("w_up", (F, H)), ("w_down", (H, F))):
        buf = dev(d[k])
        Ws.append((buf, b2s.i2s_tensor(buf, n, kk)))
    y = torch.empty((M, H), dtype=torch.float32, device="cuda")
    ws = torch.empty(b2s.ffn_block_workspace_size(M, H, F), dtype=torch.uint8, device="cuda")
    b2s.ffn_block(dev(d["x"]), dev(d["g1"]), dev(d["g2"]), float(d["eps"]), Ws[0][1], Ws[1][1], Ws[2][1], y, ws)
    sync_ok(b2s)
    assert np.array_equal(y.cpu().numpy(), d["y"])


# ------------------------------------------------------------------------------------------ softmax
@pytest.mark.parametrize("M,N,masked", [(16 * 256, 256, False), (20 * 288, 288, True), (7, 1000, True)])
def test_soft_max_ext(b2s, orc, M, N, masked):
    g = wl.rng(700 + N)
    x = (g.standard_normal((M, N)) * 4).astype(np.float32)
    mask = None
    if masked:  # causal mask rows, as in a decoder prefill
        r = min(M, N)
        mask = np.triu(np.full((r, N), -np.inf, np.float32), k=1)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    b2s.soft_max_ext(dev(x), None if mask is None else dev(mask), 0.125, y)
    sync_ok(b2s)
    y_ref = orc.soft_max_ext(x, mask, 0.125)
    yy = y.cpu().numpy()
    assert np.max(np.abs(yy - y_ref)) <= 2e-6
    assert np.array_equal(yy, y_ref)
    if masked:
        assert np.all(yy[np.isneginf(np.broadcast_to(mask[np.arange(M) % mask.shape[0]], (M, N)))] == 0.0)


# ------------------------------------------------------------------------------------------ errors
def test_errors_before_launch(b2s):
    K, N = 4304, 64
    buf = torch.zeros(b2s.i2s_nbytes(N, K), dtype=torch.uint8, device="cuda")
    W = b2s.i2s_tensor(buf, N, K)  # flattened i2_s with K % 128 != 0 needs a repack
    x = torch.zeros((4, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((4, N), dtype=torch.float32, device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(b2s.B2SError) as e:
        b2s.mul_mat(W, x, y, ws)
    assert e.value.status == b2s.B2S_ERR_UNSUPPORTED
    K = N = 256
    buf = torch.zeros(b2s.i2s_nbytes(N, K), dtype=torch.uint8, device="cuda")
    W = b2s.i2s_tensor(buf, N, K)
    x = torch.zeros((4, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((4, N), dtype=torch.float32, device="cuda")
    with pytest.raises(b2s.B2SError) as e:
        b2s.mul_mat(W, x, y, ws[:16])
    assert e.value.status == b2s.B2S_ERR_WORKSPACE
    with pytest.raises(b2s.B2SError) as e:
        b2s.mul_mat(W, torch.zeros((4, K + 16), dtype=torch.float32, device="cuda"), y, ws)
    assert e.value.status == b2s.B2S_ERR_INVALID_ARG
    sync_ok(b2s)


# ------------------------------------------------------------------------------------------ batched (ggml ne[2])
@pytest.mark.parametrize("M", [1, 5, 16, 40])
@pytest.mark.parametrize("K,N,B", [(2560, 2560, 3), (1152, 4304, 2), (256, 40, 5), (208, 64, 3),
                                   (256, 2560, 15), (384, 2600, 16), (3008, 2600, 15)])
def test_mul_mat_q8_batched(b2s, orc, M, K, N, B):
    """B independent problems in one call (one GEMV launch for M <= 16, a GEMM per matrix above): problem b
    equals the oracle's mul_mat of matrix b alone, bit for bit. The last three shapes have enough row groups
    (N/16 x B >= 2368) for the streaming GEMV kernels (TMA-fed for one token); 2600 rows leave a partial last
    row group, and K = 3008
    (row-padded to 3072) streams each row in two K chunks."""
    g = wl.rng(900 + M + K + N + B)
    ws = [wl.weight(g, N, K) for _ in range(B)]
    # One tensor: the B matrices' codes back to back, then the shared 32-byte scale trailer (all matrices
    # carry the first matrix's scale).
    sc = np.float32(ws[0].scale)
    packed = [orc.i2s_pack_ternary(w.t, float(sc)) for w in ws]
    body = np.concatenate([p[:-32] for p in packed] + [packed[0][-32:]])
    rp = K % 128 != 0
    buf = dev(body)
    if rp:  # row-pad every matrix (the flattened layout of B*N rows) on the device
        rbuf = torch.zeros(b2s.i2s_r_nbytes(B * N, K), dtype=torch.uint8, device="cuda")
        b2s.repack_rows(buf, rbuf, B * N, K)
        buf = rbuf
    W = b2s.i2s_tensor_batched(buf, N, K, B, rowpadded=rp)
    xs = [wl.activations(g, M, K) for _ in range(B)]
    ldq = (K + 15) // 16 * 16
    q = torch.zeros((B, M, ldq), dtype=torch.int8, device="cuda")[:, :, :K]
    s = torch.zeros((B, M), dtype=torch.float32, device="cuda")
    u = torch.zeros((B, M), dtype=torch.int32, device="cuda")
    for b in range(B):
        b2s.act_quant(dev(xs[b]), q[b], s[b], u[b])
    y = torch.full((B, M, N), float("nan"), dtype=torch.float32, device="cuda")
    b2s.mul_mat_q8_batched(W, q, s, u, y)
    sync_ok(b2s)
    got = y.cpu().numpy()
    for b in range(B):
        ref = orc.mul_mat_i2s(packed[b], xs[b], N) if M * N * K <= 64 * 1024 * 1024 else \
            orc.fast_mul_mat_i2s(packed[b], xs[b], N, os.cpu_count() or 8)
        assert np.array_equal(got[b], ref), b


def test_mul_mat_batched_ne2(b2s, orc):
    """b2s_mul_mat with ne[2] = 4 (fp32 X in, act-quant of all 4x7 tokens in one launch)."""
    B, M, K, N = 4, 7, 2560, 640
    g = wl.rng(950)
    ws = [wl.weight(g, N, K) for _ in range(B)]
    sc = float(ws[0].scale)
    packed = [orc.i2s_pack_ternary(w.t, sc) for w in ws]
    buf = dev(np.concatenate([p[:-32] for p in packed] + [packed[0][-32:]]))
    W = b2s.i2s_tensor_batched(buf, N, K, B)
    x = np.stack([wl.activations(g, M, K) for _ in range(B)])
    xd = dev(x.reshape(B * M, K))
    y = torch.full((B * M, N), float("nan"), dtype=torch.float32, device="cuda")
    X, Y = b2s.f32_tensor(xd), b2s.f32_tensor(y)
    for T_, rows in ((X, M), (Y, M)):
        T_.ne[1], T_.ne[2] = rows, B
        T_.nb[2] = T_.nb[1] * rows
        T_.nb[3] = T_.nb[2] * B
    ws_buf = torch.empty(b2s.mul_mat_workspace_size(W, X), dtype=torch.uint8, device="cuda")
    import ctypes as C
    b2s.check(b2s.lib().b2s_mul_mat(C.byref(W), C.byref(X), C.byref(Y), ws_buf.data_ptr(), ws_buf.numel(), None))
    sync_ok(b2s)
    got = y.cpu().numpy().reshape(B, M, N)
    for b in range(B):
        assert np.array_equal(got[b], orc.mul_mat_i2s(packed[b], x[b], N)), b
