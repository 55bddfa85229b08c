"""GGUF files with i2_s tensors (b2s/gguf.py writer and reader, b2s_bitvla_create_from_gguf loader).

CPU: the writer's parameter generator equals the oracle's; a written file reads back with the expected
metadata, shapes and I2_S bytes (dequantized codes x scale == the generated ternary weights).
GPU: a model loaded from the file gives the same hidden states and actions, bit for bit, as the model
generated from the same seed; malformed files are rejected with an error status.
"""
import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def small_gguf(tmp_path_factory, b2s):
    from b2s import bitvla, gguf
    cfg = bitvla.default_config(vit_layers=1, dec_layers=1)
    path = str(tmp_path_factory.mktemp("gguf") / "bitvla_small.gguf")
    gguf.write_bitvla(path, cfg, 4321)
    return path, cfg


def test_generator_matches_oracle(b2s, orc):
    from b2s import gguf
    for seed, tid, rows, K in [(7, 0x102, 3, 1152), (1234, 0x10037, 2, 2560), (5, 0x10E, 2, 4304)]:
        t = gguf.ternary(seed, tid, rows, K)
        Kp = (K + 127) // 128 * 128
        rp = orc.bv_ternary_rowpadded(rows, K, seed, tid).reshape(rows, Kp // 4)
        codes = np.zeros((rows, Kp), np.int8)
        for j in range(Kp // 4):
            for g in range(4):
                codes[:, 128 * (j // 32) + 32 * g + j % 32] = ((rp[:, j] >> (6 - 2 * g)) & 3).astype(np.int8) - 1
        assert np.array_equal(codes[:, :K], t)
        assert gguf.ternary_scale(seed, tid, K) == np.float32(orc.bv_ternary_scale(seed, tid, K))
    for seed, tid, n, lo, hi in [(3, 1, 1000, -0.041, 0.041), (9, 0x10000, 77, 0.9, 1.1)]:
        assert np.array_equal(gguf.uniform(seed, tid, n, lo, hi), orc.bv_uniform(n, seed, tid, lo, hi))


def test_file_round_trip(small_gguf, b2s):
    from b2s import gguf
    path, cfg = small_gguf
    g = gguf.GgufFile(path)
    assert g.kv["general.architecture"] == "bitvla"
    assert g.kv["bitvla.block_count"] == 1 and g.kv["bitvla.vision.block_count"] == 1
    assert g.kv["bitvla.token_embd.seed"] == 4321
    assert len(g.tensors) == 3 + 16 + 2 + 4 + 11 + 1 + 2
    t = g.tensors["blk.0.ffn_down.weight"]
    assert t["type"] == gguf.GGML_I2_S and t["ne"] == [cfg.dec_ffn, cfg.dec_hidden]
    for name, tid, rows, K in [("blk.0.ffn_down.weight", gguf.dec_id(0, 10), cfg.dec_hidden, cfg.dec_ffn),
                               ("v.blk.0.ffn_down.weight", gguf.vit_id(0, 14), cfg.vit_hidden, cfg.vit_ffn)]:
        raw = g.data(name)
        w = b2s.i2s_dequantize_host(raw, rows, K)
        ref = gguf.ternary(4321, tid, rows, K).astype(np.float32) * gguf.ternary_scale(4321, tid, K)
        assert np.array_equal(w, ref)
    assert np.array_equal(g.f32("blk.0.attn_norm.weight"), gguf.uniform(4321, gguf.dec_id(0, 0), cfg.dec_hidden,
                                                                         0.9, 1.1))
    with open(path, "rb") as f:
        assert f.read(4) == b"GGUF"


@pytest.mark.gpu
def test_gguf_model_equals_seeded_model(small_gguf, b2s):
    torch = pytest.importorskip("torch")
    from b2s import bitvla
    path, cfg = small_gguf
    g = np.random.Generator(np.random.PCG64(8))
    img = torch.from_numpy(g.random((2, 3, 224, 224), dtype=np.float32)).cuda()
    tok = torch.from_numpy(g.integers(0, cfg.vocab, (2, cfg.n_text)).astype(np.int32)).cuda()
    outs = []
    for kw in (dict(cfg=cfg, seed=4321), dict(cfg=None, seed=0, gguf_path=path)):
        m = bitvla.Model(kw["cfg"], kw["seed"], max_batch=2, gguf_path=kw.get("gguf_path"))
        assert m.ternary_bytes() > 0
        h = torch.zeros((2 * m.seq_len, cfg.dec_hidden), device="cuda")
        a = torch.zeros((2, cfg.action_chunk * cfg.action_dim), device="cuda")
        m.forward(img, tok, h, a)
        torch.cuda.synchronize()
        outs.append((h.cpu().numpy(), a.cpu().numpy()))
        m.close()
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


@pytest.mark.gpu
def test_gguf_errors(tmp_path, b2s):
    from b2s import bitvla
    with pytest.raises(b2s.B2SError):
        bitvla.Model(None, 0, gguf_path=str(tmp_path / "missing.gguf"))
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 60)
    with pytest.raises(b2s.B2SError):
        bitvla.Model(None, 0, gguf_path=str(bad))
    assert b2s.last_error()
