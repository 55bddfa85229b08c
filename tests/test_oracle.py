"""The oracle pinned against the golden fixtures (tests/golden, see make_golden.py) -- CPU only.

The reference holds no i2_s vectors, so the pins are hand-derived known answers, an independent
pure-Python restatement, and a third-party cross-check of the act-quant formula. The threaded SIMD
variant (the timed CPU baseline) must agree with the scalar oracle bit for bit.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_layout_kat(orc):
    k = load("kat.npz")
    assert np.array_equal(orc.i2s_pack_ternary(k["t_kat"], 1.5), k["kat_bytes"])
    # byte 0 carries positions 0, 32, 64, 96 at shifts 6, 4, 2, 0
    assert k["kat_bytes"][0] == (0 << 6) | (2 << 4) | (1 << 2) | 0
    assert np.array_equal(orc.i2s_pack_ternary(k["t_two"], 0.75), k["two_bytes"])
    t, s = orc.i2s_unpack_ternary(k["two_bytes"], 2, 64)
    assert np.array_equal(t, k["t_two"]) and s == np.float32(0.75)


def test_act_quant_kat(orc):
    k = load("kat.npz")
    q, s, u = orc.act_quant(k["x_actq"])
    assert np.array_equal(q, k["q_actq"])
    assert np.array_equal(s, k["s_actq"])
    assert np.array_equal(u, k["sum_actq"])
    # ties round half away from zero; the all-zero row keeps the 1e-5 floor
    assert q[0, 1] == 3 and q[0, 2] == -3 and s[1] == np.float32(12700000.0) and not q[1].any()


def test_act_quant_third_party_xcheck(orc):
    d = load("actquant_xcheck.npz")
    q, s, _ = orc.act_quant(d["x"])
    assert np.array_equal(q, d["q"]) and np.array_equal(s, d["s"])


def test_random_small_cases(orc):
    d = load("random_small.npz")
    for i in range(int(d["ncases"])):
        t, ws, packed, x = d[f"c{i}_t"], float(d[f"c{i}_ws"]), d[f"c{i}_packed"], d[f"c{i}_x"]
        N, K = t.shape
        assert np.array_equal(orc.i2s_pack_ternary(t, ws), packed)
        q, s, u = orc.act_quant(x)
        assert np.array_equal(q, d[f"c{i}_q"]) and np.array_equal(s, d[f"c{i}_s"])
        assert np.array_equal(u, d[f"c{i}_sums"])
        acc = orc.gemm_i32(t, q)
        assert np.array_equal(acc, d[f"c{i}_acc"])
        assert np.array_equal(orc.rescale(acc, s, ws), d[f"c{i}_y"])
        assert np.array_equal(orc.mul_mat_i2s(packed, x, N), d[f"c{i}_y"])
        assert np.array_equal(orc.fast_mul_mat_i2s(packed, x, N, 4), d[f"c{i}_y"])


def test_ffn_tiny(orc):
    d = load("ffn_tiny.npz")
    M, H = d["x"].shape
    F = d["g2"].shape[0]
    y, p = orc.ffn_block(d["x"], d["g1"], d["g2"], float(d["eps"]), d["w_gate"], d["w_up"], d["w_down"], H, F,
                         want_p=True)
    assert np.array_equal(p, d["p"])
    assert np.array_equal(y, d["y"])
    yf = orc.fast_ffn_block(d["x"], d["g1"], d["g2"], float(d["eps"]), d["w_gate"], d["w_up"], d["w_down"], H, F, 3)
    assert np.array_equal(yf, d["y"])


@pytest.mark.parametrize("M,N,K", [(1, 8, 128), (9, 40, 2560), (33, 32, 4304), (5, 128, 6912), (17, 16, 1152)])
def test_fast_equals_scalar(orc, M, N, K):
    g = np.random.default_rng(M + N + K)
    t = g.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    packed = orc.i2s_pack_ternary(t, float(np.float32(g.uniform(0.5, 2))))
    x = g.standard_normal((M, K)).astype(np.float32)
    assert np.array_equal(orc.fast_mul_mat_i2s(packed, x, N, 8), orc.mul_mat_i2s(packed, x, N))


def test_rowpadded_roundtrip(orc):
    g = np.random.default_rng(5)
    N, K = 32, 4304
    t = g.choice(np.array([-1, 0, 1], np.int8), size=(N, K))
    packed = orc.i2s_pack_ternary(t, 1.25)
    rp = orc.i2s_to_rowpadded(packed, N, K)
    Kp = 4352
    assert rp.size == N * Kp // 4 + 32
    # decode the row-padded rows: each row is its own sequence of 128-weight blocks
    tp, s = orc.i2s_unpack_ternary(rp, N, Kp)
    assert s == np.float32(1.25)
    assert np.array_equal(tp[:, :K], t) and not tp[:, K:].any()


def test_quantize_from_float(orc):
    g = np.random.default_rng(6)
    t = g.choice(np.array([-1, 0, 1], np.int8), size=(4, 256))
    w = t.astype(np.float32) * np.float32(0.8125)
    w[0, 0] = 5e-7  # below the 1e-6 zero threshold
    t_exp = t.copy()
    t_exp[0, 0] = 0
    packed = orc.i2s_quantize(w)
    t2, s = orc.i2s_unpack_ternary(packed, 4, 256)
    assert np.array_equal(t2, t_exp) and s == np.float32(0.8125)
    assert np.array_equal(orc.i2s_dequantize(packed, 4, 256), t_exp.astype(np.float32) * np.float32(0.8125))
    with pytest.raises(ValueError):
        orc.i2s_quantize(np.ones((3, 10), np.float32))


def test_planted_mistake_is_caught(orc):
    """Flipping one weight code in the packed bytes must change the oracle output (the checks are live)."""
    d = load("random_small.npz")
    packed = d["c1_packed"].copy()
    packed[0] ^= 0b11000000  # position 0: code 0 <-> 3 / 1 <-> 2 ...
    N = d["c1_t"].shape[0]
    assert not np.array_equal(orc.mul_mat_i2s(packed, d["c1_x"], N), d["c1_y"])


def test_softmax_oracle(orc):
    g = np.random.default_rng(7)
    x = g.standard_normal((5, 33)).astype(np.float32)
    mask = np.triu(np.full((5, 33), -np.inf, np.float32), k=1)
    y = orc.soft_max_ext(x, mask, 0.5)
    assert np.allclose(y.sum(1), 1.0, atol=1e-6)
    assert np.all(y[np.isneginf(mask)] == 0)
    z = x * 0.5 + mask
    e = np.exp(z - z.max(1, keepdims=True))
    assert np.allclose(y, e / e.sum(1, keepdims=True), atol=1e-6)


def test_bitvla_model_resident_weights_equal_forward(orc):
    """The CPU baseline's model (weights generated once, several forwards) gives the one-shot forward's bytes."""
    cfg = orc.bitvla_config(vit_layers=1, dec_layers=1)
    g = np.random.Generator(np.random.PCG64(5))
    img = g.random((2, 3, cfg.image_size, cfg.image_size), dtype=np.float32)
    tok = g.integers(0, cfg.vocab, (2, cfg.n_text)).astype(np.int32)
    h_ref, a_ref = orc.bitvla_forward(cfg, 77, img, tok)
    m = orc.BitVLAModel(cfg, 77)
    for _ in range(2):
        h, a = m.forward(img, tok, want_hidden=True)
        assert np.array_equal(h, h_ref) and np.array_equal(a, a_ref)
    m.close()


def test_forward_amplifies_rounding_differences(orc):
    """Why the end-to-end bar is met bit for bit and not by a tolerance: the per-token int8 act-quant between
    layers turns a rounding-level change into flipped int8 codes that grow layer by layer. Scaling every
    pixel by (1 + 2^-22) -- two ulps -- moves the oracle's own hidden states and actions by percents after
    two ViT and two decoder layers, far above 1e-3; any implementation that does not repeat the oracle's
    fp32 operation order (a reordered reduction, tensor-core products) lands at that distance."""
    cfg = orc.bitvla_config(vit_layers=2, dec_layers=2)
    g = np.random.Generator(np.random.PCG64(22))
    img = g.random((1, 3, cfg.image_size, cfg.image_size), dtype=np.float32)
    tok = g.integers(0, cfg.vocab, (1, cfg.n_text)).astype(np.int32)
    m = orc.BitVLAModel(cfg, 9)
    h0, a0 = m.forward(img, tok, want_hidden=True)
    h1, a1 = m.forward(img * np.float32(1 + 2.0 ** -22), tok, want_hidden=True)
    m.close()
    rel = float(np.max(np.abs(h1.astype(np.float64) - h0)) / np.max(np.abs(h0)))
    assert rel > 1e-2, rel


def test_det_recipf_accuracy(orc):
    """The reciprocal inside tanh (bit-pattern seed, three Newton-Raphson steps) is within 2^-22 of 1/d over
    the whole range tanh feeds it (e^{2|u|} + 1 in [2, e^19 + 1]) and beyond, powers of two included."""
    g = np.random.default_rng(7)
    d = np.concatenate([np.exp(g.uniform(0, 19, 4000)) + 1, g.uniform(1, 2, 2000) * 2.0 ** g.integers(-20, 60, 2000),
                        2.0 ** np.arange(-20, 60), np.nextafter(np.float32(2.0) ** np.arange(-20, 60), 0)])
    d = d.astype(np.float32)
    y = orc.det_recipf(d).astype(np.float64)
    assert np.max(np.abs(y * d.astype(np.float64) - 1.0)) <= 2.0 ** -22


def test_gelu_tanh_accuracy(orc):
    """GELU (tanh form) with the oracle's exp and reciprocal stays within 1e-6 x max(1, |x|) of the float64
    evaluation of the same formula, across the saturating tails."""
    x = np.concatenate([np.linspace(-12, 12, 24001), np.random.default_rng(8).standard_normal(4000) * 3]).astype(
        np.float32)
    got = orc.gelu_tanh(x).astype(np.float64)
    x64 = x.astype(np.float64)
    ref = 0.5 * x64 * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x64 + 0.044715 * x64 ** 3)))
    assert np.all(np.abs(got - ref) <= 1e-6 * np.maximum(1.0, np.abs(x64)))

