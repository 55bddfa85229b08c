"""The non-i2_s operators of the BitVLA-shape forward (through the C ABI) against the oracle, on a B200.

Every operator repeats the oracle's IEEE operation sequence (fused multiply-adds in a fixed order for the
attention and patch-embedding products, the deterministic exp/tanh for softmax and GELU, RoPE angles in
double rounded once), so all comparisons are exact; max-abs-rel <= 1e-5 is asserted first so that a
failure shows its size.
"""
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


def sync_ok(b2s):
    torch.cuda.synchronize()
    assert b2s.device_error() == 0


def q8_buffers(M, K):
    ldq = (K + 15) // 16 * 16
    q = torch.zeros((M, ldq), dtype=torch.int8, device="cuda")[:, :K]
    s = torch.zeros(M, dtype=torch.float32, device="cuda")
    u = torch.zeros(M, dtype=torch.int32, device="cuda")
    return q, s, u


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("M,K", [(1, 1152), (256, 1152), (7, 2560), (3, 4304), (2, 100)])
def test_norm_fp32_bit_exact(b2s, orc, kind, M, K):
    g = wl.rng(10 * M + K + kind)
    x = wl.activations(g, M, K) * 2.0 + 0.5
    w = wl.norm_weight(g, K)
    b = (0.02 * g.standard_normal(K)).astype(np.float32)
    y = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    bb = None if kind == 0 else dev(b)
    b2s.norm(dev(x), dev(w), bb, 1e-6, kind, y)
    sync_ok(b2s)
    ref = orc.rms_norm(x, w, 1e-6) if kind == 0 else orc.layer_norm(x, w, b, 1e-6)
    assert np.array_equal(y.cpu().numpy(), ref)


@pytest.mark.parametrize("M,K", [(256, 1152), (5, 4304), (300, 2560)])
def test_layer_norm_act_quant_bit_exact(b2s, orc, M, K):
    g = wl.rng(M + K)
    x = wl.activations(g, M, K) * 3.0
    w = wl.norm_weight(g, K)
    b = (0.02 * g.standard_normal(K)).astype(np.float32)
    q, s, u = q8_buffers(M, K)
    b2s.norm_act_quant(dev(x), dev(w), dev(b), 1e-6, 1, q, s, u)
    sync_ok(b2s)
    q_ref, s_ref, u_ref = orc.act_quant(orc.layer_norm(x, w, b, 1e-6))
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(u.cpu().numpy(), u_ref)


@pytest.mark.parametrize("M,heads,hd,pos0", [(288, 25, 128, 0), (5, 3, 72, 1000), (1, 1, 2, 7)])
def test_rope_neox_bit_exact(b2s, orc, M, heads, hd, pos0):
    g = wl.rng(M * heads + hd)
    ld = heads * hd + 16
    x = wl.activations(g, M, ld)
    xd = dev(x)
    b2s.rope_neox(xd[:, : heads * hd], heads, hd, 500000.0, pos0)
    sync_ok(b2s)
    ref = orc.rope_neox(x[:, : heads * hd], heads, hd, 500000.0, pos0)
    got = xd.cpu().numpy()
    assert np.array_equal(got[:, : heads * hd], ref)
    assert np.array_equal(got[:, heads * hd:], x[:, heads * hd:])  # columns past the heads untouched


@pytest.mark.parametrize("M,heads,kv,hd,causal", [(256, 16, 16, 72, False), (288, 20, 5, 128, True),
                                                  (200, 8, 2, 128, False), (130, 4, 4, 128, True),
                                                  (77, 6, 3, 72, True), (100, 4, 2, 128, True),
                                                  (33, 4, 2, 64, True), (1, 2, 1, 8, True)])
def test_attention(b2s, orc, M, heads, kv, hd, causal):
    """Head dims 128 and 72 run the wide-tile kernel, others the 256-thread one; both repeat the oracle's
    operation order, so the result is bit-exact. Ragged sizes leave partial query blocks and key chunks; a
    last block of at most 32 rows with an even number of query heads per K/V head is computed for two heads
    in one tile (288, 200 and 77 tokens), a 36-row one is not (100 tokens)."""
    g = wl.rng(M + heads + hd)
    H, KV = heads * hd, kv * hd
    qkv = wl.activations(g, M, H + 2 * KV)
    scale = 1.0 / np.sqrt(hd)
    qkvd = dev(qkv)
    o = torch.full((M, H), float("nan"), dtype=torch.float32, device="cuda")
    b2s.attention(qkvd[:, :H], qkvd[:, H:H + KV], qkvd[:, H + KV:], heads, kv, hd, float(scale), causal, o)
    sync_ok(b2s)
    ref = orc.attention(qkv, 0, H, H + KV, 1, heads, kv, hd, M, causal, float(scale))
    got = o.cpu().numpy()
    assert max_abs_rel(got, ref) <= TOL
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("M,heads,kv,hd,causal", [(256, 16, 16, 72, False), (288, 20, 5, 128, True),
                                                  (33, 4, 2, 64, True), (1, 2, 1, 8, True), (300, 8, 8, 32, False),
                                                  (384, 4, 4, 128, False), (100, 32, 4, 16, True),
                                                  (77, 6, 3, 40, False)])
def test_attention_tensor_cores(b2s, orc, M, heads, kv, hd, causal):
    """b2s_attention_tc (3xTF32 tcgen05 products, exact-max softmax) against the oracle's fp32 attention and a
    float64 evaluation: within the 1e-5 per-operator bar (max |o - ref| / max |ref|)."""
    g = wl.rng(3 * M + heads + hd)
    H, KV = heads * hd, kv * hd
    qkv = wl.activations(g, M, H + 2 * KV) * 2.0
    scale = 1.0 / np.sqrt(hd)
    qkvd = dev(qkv)
    o = torch.full((M, H), float("nan"), dtype=torch.float32, device="cuda")
    b2s.attention_tc(qkvd[:, :H], qkvd[:, H:H + KV], qkvd[:, H + KV:], heads, kv, hd, float(scale), causal, o)
    sync_ok(b2s)
    got = o.cpu().numpy()
    ref = orc.attention(qkv, 0, H, H + KV, 1, heads, kv, hd, M, causal, float(scale))
    q64 = qkv[:, :H].astype(np.float64).reshape(M, heads, hd)
    k64 = qkv[:, H:H + KV].astype(np.float64).reshape(M, kv, hd)
    v64 = qkv[:, H + KV:].astype(np.float64).reshape(M, kv, hd)
    rep = heads // kv
    s64 = np.einsum("mhd,nhd->hmn", q64, np.repeat(k64, rep, axis=1)) * scale
    if causal:
        s64 = np.where(np.tril(np.ones((M, M), bool))[None], s64, -np.inf)
    p64 = np.exp(s64 - s64.max(axis=2, keepdims=True))
    p64 /= p64.sum(axis=2, keepdims=True)
    o64 = np.einsum("hmn,nhd->mhd", p64, np.repeat(v64, rep, axis=1)).reshape(M, H)
    assert np.isfinite(got).all()
    assert max_abs_rel(got, o64) <= TOL, max_abs_rel(got, o64)
    assert max_abs_rel(got, ref) <= TOL, max_abs_rel(got, ref)


def test_attention_tensor_cores_unsupported(b2s):
    qkv = torch.zeros((400, 3 * 64), dtype=torch.float32, device="cuda")
    o = torch.zeros((400, 64), dtype=torch.float32, device="cuda")
    with pytest.raises(b2s.B2SError):  # 400 keys visible to one query block (no causal mask): above 384
        b2s.attention_tc(qkv[:, :64], qkv[:, 64:128], qkv[:, 128:], 1, 1, 64, 0.125, False, o)
    with pytest.raises(b2s.B2SError):  # 3 query heads per K/V head does not divide the 128 MMA rows
        q3 = torch.zeros((8, 3 * 64), dtype=torch.float32, device="cuda")
        b2s.attention_tc(q3, qkv[:8, :64], qkv[:8, 64:128], 3, 1, 64, 0.125, True, o[:8].repeat(1, 3))


def test_attention_unsupported(b2s):
    qkv = torch.zeros((8, 3 * 36), dtype=torch.float32, device="cuda")
    o = torch.zeros((8, 36), dtype=torch.float32, device="cuda")
    with pytest.raises(b2s.B2SError):  # head_dim 36 is not a multiple of 8
        b2s.attention(qkv[:, :36], qkv[:, 36:72], qkv[:, 72:], 1, 1, 36, 1.0, False, o)
    assert b2s.last_error()


def test_patch_embed(b2s):
    g = wl.rng(5)
    C, S, P, D = 3, 224, 14, 1152
    img = g.random((C, S, S), dtype=np.float32)
    w = (g.standard_normal((D, C * P * P)) * 0.04).astype(np.float32)
    bias = (0.02 * g.standard_normal(D)).astype(np.float32)
    pos = (0.02 * g.standard_normal(((S // P) ** 2, D))).astype(np.float32)
    y = torch.zeros(((S // P) ** 2, D), dtype=torch.float32, device="cuda")
    b2s.patch_embed(dev(img), P, dev(w), dev(bias), dev(pos), y)
    sync_ok(b2s)
    G = S // P
    cols = img.reshape(C, G, P, G, P).transpose(1, 3, 0, 2, 4).reshape(G * G, C * P * P).astype(np.float64)
    ref64 = cols @ w.astype(np.float64).T + (bias[None, :] + pos).astype(np.float64)
    got = y.cpu().numpy()
    assert max_abs_rel(got, ref64) <= TOL
    # the fixed order: acc = fma(col[k], w[d][k], acc), k ascending; y = (bias + pos) + acc
    colsf = cols.astype(np.float32)
    for r, d in [(0, 0), (5, 17), (255, 1151), (100, 600)]:
        acc = np.float32(0.0)
        for k in range(colsf.shape[1]):
            acc = np.float32(np.float64(colsf[r, k]) * np.float64(w[d, k]) + np.float64(acc))  # exact fma in double
        assert got[r, d] == np.float32(bias[d] + pos[r, d]) + acc


def test_embed_tokens_hash_bit_exact(b2s, orc):
    toks = np.array([0, 1, 128255, 42, 42, 99999], np.int32)
    D, seed = 2560, 1234
    y = torch.zeros((len(toks), D), dtype=torch.float32, device="cuda")
    b2s.embed_tokens_hash(dev(toks), D, seed, y)
    sync_ok(b2s)
    got = y.cpu().numpy()
    ref = np.zeros_like(got)
    for i, t in enumerate(toks):
        bits = np.array([orc.bv_param_bits(seed, 0x80000000 | int(t), c) for c in range(D)], np.uint64)
        u = (bits >> 8).astype(np.float32) * np.float32(1.0 / 16777216.0)
        ref[i] = np.float32(-0.02) + np.float32(0.04) * u
    assert np.array_equal(got, ref)
    assert np.array_equal(got[3], got[4])


@pytest.mark.parametrize("M,K,N", [(256, 1152, 3456), (7, 2560, 640), (300, 4304, 1152)])
@pytest.mark.parametrize("act", [0, 1])
def test_mul_mat_epilogue(b2s, orc, M, K, N, act):
    """y = residual + act(W q + bias), in place on the residual; GEMV (M <= 16) and tensor cores."""
    g = wl.rng(M + K + N + act)
    w = wl.weight(g, N, K)
    x = wl.activations(g, M, K)
    bias = (0.1 * g.standard_normal(N)).astype(np.float32)
    res = wl.activations(g, M, N)
    buf = dev(w.packed)
    W = b2s.i2s_tensor(buf, N, K)
    if K % 128:
        Kp = (K + 127) // 128 * 128
        rbuf = torch.zeros(b2s.i2s_r_nbytes(N, K), dtype=torch.uint8, device="cuda")
        b2s.repack_rows(buf, rbuf, N, K)
        W = b2s.i2s_tensor(rbuf, N, K, rowpadded=True)
        buf = rbuf
        assert Kp > K
    q, s, u = q8_buffers(M, K)
    b2s.act_quant(dev(x), q, s, u)
    y = dev(res)
    b2s.mul_mat_q8_epi(W, q, s, u, y, bias=dev(bias), residual=y, act=act)
    sync_ok(b2s)
    q_ref, s_ref, _ = orc.act_quant(x)
    v = orc.rescale(orc.gemm_i32(w.t, q_ref), s_ref, float(w.scale)) + bias[None, :]
    if act == 1:
        v = orc.gelu_tanh(v)
    ref = res + v
    got = y.cpu().numpy()
    assert max_abs_rel(got, ref) <= TOL
    assert np.array_equal(got, ref)
