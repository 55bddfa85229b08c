"""The C ABI library without a GPU: it loads, exports every symbol include/b2s.h, include/b2s_bitvla.h and
include/b2s_server.h declare, its host type traits agree with the oracle byte for byte, and device entry points fail cleanly
(no compute calls)."""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols(header="b2s.h"):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2s_\w+)\s*\(", src)))


def test_exports_every_declared_symbol(b2s):
    import ctypes
    lib = ctypes.CDLL(b2s.LIB_PATH)
    decl = declared_symbols()
    assert decl, "no declarations parsed"
    missing = [s for s in decl if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    assert sorted(b2s.EXPORTED) == decl


def test_exports_bitvla_symbols(b2s):
    import ctypes
    from b2s import bitvla
    lib = ctypes.CDLL(b2s.LIB_PATH)
    decl = declared_symbols("b2s_bitvla.h")
    assert decl and not [s for s in decl if not hasattr(lib, s)]
    assert sorted(bitvla.EXPORTED) == decl


def test_exports_server_symbols(b2s):
    import ctypes
    from b2s import server
    lib = ctypes.CDLL(b2s.LIB_PATH)
    decl = declared_symbols("b2s_server.h")
    assert decl and not [s for s in decl if not hasattr(lib, s)]
    assert sorted(server.EXPORTED) == decl


def test_bitvla_host_traits(b2s, orc):
    """Host-side engine traits: the parameter generator matches the oracle's; shapes and op counts."""
    from b2s import bitvla
    for seed, tensor, idx in [(0, 0, 0), (7, 0x100, 12345), (0xFFFFFFFF, 0x10000 + 16 * 29 + 10, 2**31 + 5),
                              (123, 0x80000000 | 128255, 2559)]:
        assert bitvla.param_bits(seed, tensor, idx) == orc.bv_param_bits(seed, tensor, idx)
    cfg = bitvla.default_config()
    assert bitvla.seq_len(cfg) == 288 == orc.bitvla_seq_len(orc.bitvla_config())
    ops = bitvla.ternary_ops(cfg)
    # ViT 0.210 T + decoder 1.200 T + connector (1152x2560 and 2560x2560 over 256 tokens)
    vit = 2 * 256 * 27 * (4 * 1152 * 1152 + 2 * 1152 * 4304)
    dec = 2 * 288 * 30 * (2 * 2560 * 2560 + 2 * 2560 * 640 + 3 * 2560 * 6912)
    conn = 2 * 256 * (1152 * 2560 + 2560 * 2560)
    assert ops == vit + dec + conn
    assert abs(vit / 1e12 - 0.210) < 0.001 and abs(dec / 1e12 - 1.200) < 0.001
    bad = bitvla.default_config(patch=15)
    import ctypes
    h = ctypes.c_void_p()
    assert bitvla._bind().b2s_bitvla_create(ctypes.byref(bad), 1, 1, ctypes.byref(h)) != 0
    assert not h.value


def test_nbytes(b2s, orc):
    for N, K in [(2560, 2560), (6912, 2560), (1152, 4304), (3, 128)]:
        assert b2s.i2s_nbytes(N, K) == orc.i2s_nbytes(N, K) == N * K // 4 + 32
        assert b2s.i2s_r_nbytes(N, K) == N * ((K + 127) // 128 * 128) // 4 + 32


@pytest.mark.parametrize("N,K", [(8, 128), (40, 2560), (32, 4304), (3, 1152)])
def test_host_quantize_matches_oracle(b2s, orc, N, K):
    g = np.random.default_rng(N * K)
    t = g.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
    w = t.astype(np.float32) * np.float32(g.uniform(0.5, 2))
    mine = b2s.i2s_quantize_host(w)
    assert np.array_equal(mine, orc.i2s_quantize(w))
    assert np.array_equal(b2s.i2s_dequantize_host(mine, N, K), orc.i2s_dequantize(mine, N, K))


def test_host_trait_errors(b2s):
    with pytest.raises(b2s.B2SError):
        b2s.i2s_quantize_host(np.ones((3, 10), np.float32))
    assert "multiple of 128" in b2s.last_error()
    assert b2s.lib().b2s_i2s_dequantize(None, None, 1, 128) == b2s.B2S_ERR_INVALID_ARG


def test_device_entry_points_fail_cleanly_without_gpu(b2s):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    rc = b2s.lib().b2s_device_check()
    assert rc in (b2s.B2S_ERR_CUDA, b2s.B2S_ERR_DEVICE)
    assert b2s.last_error()
    W = b2s.Tensor()
    rc = b2s.lib().b2s_mul_mat(W, W, W, None, 0, None)
    assert rc != b2s.B2S_OK


def test_workspace_sizes(b2s):
    W = b2s.Tensor()
    W.ne[:] = [2560, 2560, 1, 1]
    X = b2s.Tensor()
    X.ne[:] = [2560, 300, 1, 1]
    ws = b2s.mul_mat_workspace_size(W, X)
    assert ws >= 300 * 2560 + 300 * 8 and ws % 256 == 0
    f = b2s.ffn_block_workspace_size(300, 2560, 6912)
    assert f >= 300 * 2560 + 300 * 6912 * 4 + 300 * 6912
