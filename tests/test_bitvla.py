"""The BitVLA-shape engine (C ABI include/b2s_bitvla.h) against the oracle's forward, on a B200.

The engine regenerates the random-init model on the device from the seed; the oracle regenerates the
same parameters on the host with its own copy of the generator. Two attention modes:
  * the default (attention_tc=0): every operator of the forward repeats the oracle's IEEE operation sequence (ternary
    GEMMs exact in int32, fixed-order fused multiply-adds in attention and patch embedding, the deterministic
    exp/tanh), so hidden states and actions are compared bit for bit, after the max-abs-rel bars
    (max |y - ref| / max |ref|) of 1e-5 per operator and 1e-3 end to end through all 57 layers;
  * attention_tc=1: attention on the tensor cores (3xTF32 products, within 1e-5 per operator of the oracle).
    The int8 act-quant between layers turns any rounding difference into code flips that grow layer by
    layer (tests/test_oracle.py shows a 2^-22 relative input change moving the oracle's own output by
    several percent), so this mode is checked for batch independence and for staying within a few percent
    of the oracle, not against the 1e-3 end-to-end bar.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def max_abs_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


def inputs(cfg, batch, seed):
    g = np.random.Generator(np.random.PCG64(seed))
    img = g.random((batch, 3, cfg.image_size, cfg.image_size), dtype=np.float32)
    tok = g.integers(0, cfg.vocab, (batch, cfg.n_text)).astype(np.int32)
    return img, tok


def run_engine(cfg_over, seed, batch, img, tok, max_batch=None):
    from b2s import bitvla, device_error
    cfg = bitvla.default_config(**cfg_over)
    m = bitvla.Model(cfg, seed, max_batch=max_batch or batch)
    seq = m.seq_len
    hidden = torch.full((batch * seq, cfg.dec_hidden), float("nan"), dtype=torch.float32, device="cuda")
    actions = torch.full((batch, cfg.action_chunk * cfg.action_dim), float("nan"), dtype=torch.float32,
                         device="cuda")
    m.forward(torch.from_numpy(img).cuda(), torch.from_numpy(tok).cuda(), hidden, actions)
    torch.cuda.synchronize()
    assert device_error() == 0
    out = hidden.cpu().numpy(), actions.cpu().numpy()
    m.close()
    return out


def run_oracle(orc, cfg_over, seed, img, tok):
    return orc.bitvla_forward(orc.bitvla_config(**cfg_over), seed, img, tok)


@pytest.mark.parametrize("over,tol", [
    (dict(vit_layers=0, dec_layers=0), 1e-5),             # patch embed -> post-LN -> connector -> final norm
    (dict(vit_layers=0, dec_layers=0, n_text=0), 1e-5),   # no text tokens
])
def test_connector_path(b2s, orc, over, tol):
    img, tok = inputs(orc.bitvla_config(**over), 1, 11)
    h, a = run_engine(over, 5, 1, img, tok)
    h_ref, a_ref = run_oracle(orc, over, 5, img, tok)
    assert max_abs_rel(h, h_ref) <= tol and max_abs_rel(a, a_ref) <= tol
    assert np.array_equal(h, h_ref) and np.array_equal(a, a_ref)


@pytest.mark.parametrize("batch", [1, 3])
def test_reduced_depth(b2s, orc, batch):
    over = dict(vit_layers=2, dec_layers=2)
    img, tok = inputs(orc.bitvla_config(**over), batch, 21)
    h, a = run_engine(over, 9, batch, img, tok)
    h_ref, a_ref = run_oracle(orc, over, 9, img, tok)
    assert np.isfinite(h).all() and np.isfinite(a).all()
    assert max_abs_rel(h, h_ref) <= 1e-5 and max_abs_rel(a, a_ref) <= 1e-5
    assert np.array_equal(h, h_ref) and np.array_equal(a, a_ref)


@pytest.mark.parametrize("batch", [1, 3])
def test_reduced_depth_tensor_core_attention(b2s, orc, batch):
    over = dict(vit_layers=2, dec_layers=2, attention_tc=1)
    img, tok = inputs(orc.bitvla_config(**over), batch, 22)
    h, a = run_engine(over, 9, batch, img, tok)
    h_ref, a_ref = run_oracle(orc, over, 9, img, tok)
    assert np.isfinite(h).all() and np.isfinite(a).all()
    assert max_abs_rel(h, h_ref) <= 0.2 and max_abs_rel(a, a_ref) <= 0.2
    if batch > 1:  # observations do not mix: each row block equals that observation run alone
        h1, a1 = run_engine(over, 9, 1, img[1:2], tok[1:2])
        seq = h1.shape[0]
        assert np.array_equal(h[seq:2 * seq], h1) and np.array_equal(a[1:2], a1)


def test_batch_rows_independent(b2s, orc):
    """Observation b of a batched forward equals the same observation run alone."""
    over = dict(vit_layers=1, dec_layers=1)
    img, tok = inputs(orc.bitvla_config(**over), 2, 31)
    h2, a2 = run_engine(over, 3, 2, img, tok)
    h1, a1 = run_engine(over, 3, 1, img[1:], tok[1:])
    seq = h1.shape[0]
    assert np.array_equal(h2[seq:], h1)
    assert np.array_equal(a2[1:], a1)


def test_full_depth_end_to_end(b2s, orc):
    """The BitVLA shape (27 ViT + 30 decoder layers), one observation: 1e-3 end to end, then bit for bit."""
    over = {}
    img, tok = inputs(orc.bitvla_config(), 1, 41)
    h, a = run_engine(over, 2024, 1, img, tok)
    h_ref, a_ref = run_oracle(orc, over, 2024, img, tok)
    assert max_abs_rel(h, h_ref) <= 1e-3 and max_abs_rel(a, a_ref) <= 1e-3
    assert np.array_equal(h, h_ref) and np.array_equal(a, a_ref)


def test_full_depth_tensor_core_attention(b2s, orc):
    """Tensor-core attention through all 57 layers: finite and within a few percent of the oracle."""
    over = dict(attention_tc=1)
    img, tok = inputs(orc.bitvla_config(), 1, 42)
    h, a = run_engine(over, 2025, 1, img, tok)
    h_ref, a_ref = run_oracle(orc, over, 2025, img, tok)
    assert np.isfinite(h).all() and np.isfinite(a).all()
    assert max_abs_rel(h, h_ref) <= 0.25 and max_abs_rel(a, a_ref) <= 0.25


def test_full_depth_batch8_rows(b2s, orc):
    """The benched configuration: a full-depth forward of 8 observations equals each observation run alone
    (batch 1, bit for bit: no kernel mixes observations), and one of them equals the oracle's forward (1e-3
    end to end, then bit for bit)."""
    from b2s import bitvla, device_error
    cfg = bitvla.default_config()
    img, tok = inputs(orc.bitvla_config(), 8, 51)
    m = bitvla.Model(cfg, 1234, max_batch=8)
    seq = m.seq_len
    h8 = torch.full((8 * seq, cfg.dec_hidden), float("nan"), dtype=torch.float32, device="cuda")
    a8 = torch.full((8, cfg.action_chunk * cfg.action_dim), float("nan"), dtype=torch.float32, device="cuda")
    m.forward(torch.from_numpy(img).cuda(), torch.from_numpy(tok).cuda(), h8, a8)
    h1 = torch.full((seq, cfg.dec_hidden), float("nan"), dtype=torch.float32, device="cuda")
    a1 = torch.full((1, cfg.action_chunk * cfg.action_dim), float("nan"), dtype=torch.float32, device="cuda")
    for b in range(8):
        m.forward(torch.from_numpy(img[b:b + 1]).cuda(), torch.from_numpy(tok[b:b + 1]).cuda(), h1, a1)
        torch.cuda.synchronize()
        assert torch.equal(h8[b * seq:(b + 1) * seq], h1), b
        assert torch.equal(a8[b], a1[0]), b
    assert device_error() == 0
    h8n, a8n = h8.cpu().numpy(), a8.cpu().numpy()
    m.close()
    om = orc.BitVLAModel(orc.bitvla_config(), 1234)
    h_ref, a_ref = om.forward(img[5:6], tok[5:6], want_hidden=True)
    om.close()
    assert max_abs_rel(h8n[5 * seq:6 * seq], h_ref) <= 1e-3 and max_abs_rel(a8n[5:6], a_ref) <= 1e-3
    assert np.array_equal(h8n[5 * seq:6 * seq], h_ref) and np.array_equal(a8n[5:6], a_ref)


def test_predict_host_path(b2s):
    """predict() (uint8 HWC host images -> host actions) equals forward() on value/255 images."""
    from b2s import bitvla
    over = dict(vit_layers=1, dec_layers=1)
    cfg = bitvla.default_config(**over)
    g = np.random.Generator(np.random.PCG64(77))
    u8 = g.integers(0, 256, (2, cfg.image_size, cfg.image_size, 3)).astype(np.uint8)
    tok = g.integers(0, cfg.vocab, (2, cfg.n_text)).astype(np.int32)
    m = bitvla.Model(cfg, 17, max_batch=2)
    act = np.zeros((2, cfg.action_chunk * cfg.action_dim), np.float32)
    m.predict(u8, tok, act)
    img = (u8.astype(np.float32).transpose(0, 3, 1, 2) / np.float32(255.0)).astype(np.float32)
    a_dev = torch.zeros((2, act.shape[1]), dtype=torch.float32, device="cuda")
    m.forward(torch.from_numpy(np.ascontiguousarray(img)).cuda(), torch.from_numpy(tok).cuda(), None, a_dev)
    torch.cuda.synchronize()
    assert np.array_equal(act, a_dev.cpu().numpy())
    # replaying the captured graph gives the same answer
    act2 = np.zeros_like(act)
    m.predict(u8, tok, act2)
    assert np.array_equal(act, act2)
    m.close()


def test_create_errors(b2s):
    from b2s import bitvla
    with pytest.raises(b2s.B2SError):
        bitvla.Model(bitvla.default_config(vit_hidden=1000), 1)
    m = bitvla.Model(bitvla.default_config(vit_layers=0, dec_layers=0), 1, max_batch=1)
    img = torch.zeros((2, 3, 224, 224), dtype=torch.float32, device="cuda")
    tok = torch.zeros((2, 32), dtype=torch.int32, device="cuda")
    with pytest.raises(b2s.B2SError):
        m.forward(img, tok)  # batch 2 > max_batch 1
    m.close()
