"""ctypes wrapper over the oracle library (TEST INFRASTRUCTURE).

The oracle is the CPU restatement of the i2_s mul_mat path (algorithm, provenance and byte layout in
``i2s_oracle.h``). Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
may import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.orc_i2s_nbytes.restype = C.c_size_t
        L.orc_i2s_nbytes.argtypes = [_i64, _i64]
        L.orc_i2s_r_nbytes.restype = C.c_size_t
        L.orc_i2s_r_nbytes.argtypes = [_i64, _i64]
        L.orc_i2s_quantize.restype = C.c_size_t
        L.orc_i2s_quantize.argtypes = [_f32p, _u8p, _i64, _i64]
        L.orc_i2s_pack_ternary.restype = C.c_size_t
        L.orc_i2s_pack_ternary.argtypes = [_i8p, C.c_float, _u8p, _i64, _i64]
        L.orc_i2s_unpack_ternary.restype = C.c_float
        L.orc_i2s_unpack_ternary.argtypes = [_u8p, _i8p, _i64, _i64]
        L.orc_i2s_dequantize.restype = None
        L.orc_i2s_dequantize.argtypes = [_u8p, _f32p, _i64, _i64]
        L.orc_i2s_to_rowpadded.restype = C.c_size_t
        L.orc_i2s_to_rowpadded.argtypes = [_u8p, _u8p, _i64, _i64]
        L.orc_act_quant.restype = None
        L.orc_act_quant.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _i32p]
        L.orc_gemm_i32.restype = None
        L.orc_gemm_i32.argtypes = [_i8p, _i8p, _i64, _i64, _i64, _i32p]
        L.orc_rescale.restype = None
        L.orc_rescale.argtypes = [_i32p, _f32p, C.c_float, _i64, _i64, _f32p]
        L.orc_mul_mat_i2s.restype = None
        L.orc_mul_mat_i2s.argtypes = [_u8p, _f32p, _i64, _i64, _i64, _f32p]
        L.orc_rms_norm.restype = None
        L.orc_rms_norm.argtypes = [_f32p, C.c_void_p, _i64, _i64, C.c_float, _f32p]
        L.orc_sqrelu_mul.restype = None
        L.orc_sqrelu_mul.argtypes = [_f32p, _f32p, _i64, _f32p]
        L.orc_soft_max_ext.restype = None
        L.orc_soft_max_ext.argtypes = [_f32p, C.c_void_p, _i64, _i64, _i64, C.c_float, _f32p]
        L.orc_ffn_block.restype = None
        L.orc_ffn_block.argtypes = [_f32p, _i64, _i64, _i64, _f32p, _f32p, C.c_float,
                                    _u8p, _u8p, _u8p, _f32p, C.c_void_p]
        L.orc_fast_mul_mat_i2s.restype = None
        L.orc_fast_mul_mat_i2s.argtypes = [_u8p, _f32p, _i64, _i64, _i64, _f32p, C.c_int]
        L.orc_fast_ffn_block.restype = None
        L.orc_fast_ffn_block.argtypes = [_f32p, _i64, _i64, _i64, _f32p, _f32p, C.c_float,
                                         _u8p, _u8p, _u8p, _f32p, C.c_int]
        L.orc_fast_isa.restype = C.c_int
        L.orc_fast_isa.argtypes = []
        L.orc_bv_param_bits.restype = C.c_uint32
        L.orc_bv_param_bits.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_bv_ternary_scale.restype = C.c_float
        L.orc_bv_ternary_scale.argtypes = [C.c_uint32, C.c_uint32, _i64]
        L.orc_bv_gen_ternary.restype = None
        L.orc_bv_gen_ternary.argtypes = [_u8p, _i64, _i64, C.c_uint32, C.c_uint32, C.c_int]
        L.orc_bv_gen_uniform.restype = None
        L.orc_bv_gen_uniform.argtypes = [_f32p, _i64, C.c_uint32, C.c_uint32, C.c_float, C.c_float]
        L.orc_layer_norm.restype = None
        L.orc_layer_norm.argtypes = [_f32p, C.c_void_p, C.c_void_p, _i64, _i64, C.c_float, _f32p]
        L.orc_gelu_tanh.restype = C.c_float
        L.orc_gelu_tanh.argtypes = [C.c_float]
        L.orc_det_recipf.restype = C.c_float
        L.orc_det_recipf.argtypes = [C.c_float]
        L.orc_rope_table.restype = None
        L.orc_rope_table.argtypes = [C.c_float, C.c_int, C.c_int, _f32p]
        L.orc_rope_neox.restype = None
        L.orc_rope_neox.argtypes = [_f32p, _i64, C.c_int, C.c_int, _i64, _f32p, C.c_int, C.c_int]
        L.orc_attention.restype = None
        L.orc_attention.argtypes = [_f32p, _i64, _i64, _i64, _i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_float, _f32p, _i64, C.c_int]
        L.orc_bitvla_create.restype = C.c_void_p
        L.orc_bitvla_create.argtypes = [C.c_void_p, C.c_uint32, C.c_int]
        L.orc_bitvla_free.restype = None
        L.orc_bitvla_free.argtypes = [C.c_void_p]
        L.orc_bitvla_run.restype = C.c_int
        L.orc_bitvla_run.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.orc_bitvla_forward.restype = C.c_int
        L.orc_bitvla_forward.argtypes = [C.c_void_p, C.c_uint32, C.c_int, _f32p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_int]
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def i2s_nbytes(N: int, K: int) -> int:
    return int(lib().orc_i2s_nbytes(N, K))


def i2s_quantize(w: np.ndarray) -> np.ndarray:
    """Pack float weights [N, K] (ternary times a scale) into i2_s bytes."""
    w = _c(w, np.float32)
    N, K = w.shape
    out = np.zeros(i2s_nbytes(N, K), np.uint8)
    if lib().orc_i2s_quantize(w, out, N, K) == 0:
        raise ValueError("i2_s needs N*K to be a multiple of 128")
    return out


def i2s_pack_ternary(t: np.ndarray, scale: float) -> np.ndarray:
    t = _c(t, np.int8)
    N, K = t.shape
    out = np.zeros(i2s_nbytes(N, K), np.uint8)
    if lib().orc_i2s_pack_ternary(t, float(scale), out, N, K) == 0:
        raise ValueError("i2_s needs N*K to be a multiple of 128")
    return out


def i2s_unpack_ternary(packed: np.ndarray, N: int, K: int):
    t = np.zeros((N, K), np.int8)
    s = lib().orc_i2s_unpack_ternary(_c(packed, np.uint8), t, N, K)
    return t, float(s)


def i2s_dequantize(packed: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.zeros((N, K), np.float32)
    lib().orc_i2s_dequantize(_c(packed, np.uint8), out, N, K)
    return out


def i2s_to_rowpadded(packed: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.zeros(int(lib().orc_i2s_r_nbytes(N, K)), np.uint8)
    lib().orc_i2s_to_rowpadded(_c(packed, np.uint8), out, N, K)
    return out


def act_quant(x: np.ndarray):
    x = _c(x, np.float32)
    M, K = x.shape
    q = np.zeros((M, K), np.int8)
    s = np.zeros(M, np.float32)
    sums = np.zeros(M, np.int32)
    lib().orc_act_quant(x, M, K, q, s, sums)
    return q, s, sums


def gemm_i32(t: np.ndarray, q: np.ndarray) -> np.ndarray:
    t = _c(t, np.int8)
    q = _c(q, np.int8)
    N, K = t.shape
    M = q.shape[0]
    acc = np.zeros((M, N), np.int32)
    lib().orc_gemm_i32(t, q, M, N, K, acc)
    return acc


def rescale(acc: np.ndarray, s: np.ndarray, w_scale: float) -> np.ndarray:
    acc = _c(acc, np.int32)
    M, N = acc.shape
    y = np.zeros((M, N), np.float32)
    lib().orc_rescale(acc, _c(s, np.float32), float(w_scale), M, N, y)
    return y


def mul_mat_i2s(packed: np.ndarray, x: np.ndarray, N: int) -> np.ndarray:
    x = _c(x, np.float32)
    M, K = x.shape
    y = np.zeros((M, N), np.float32)
    lib().orc_mul_mat_i2s(_c(packed, np.uint8), x, M, N, K, y)
    return y


def rms_norm(x: np.ndarray, g, eps: float) -> np.ndarray:
    x = _c(x, np.float32)
    M, K = x.shape
    g = None if g is None else _c(g, np.float32)
    y = np.zeros((M, K), np.float32)
    lib().orc_rms_norm(x, _ptr(g), M, K, float(eps), y)
    return y


def sqrelu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = _c(g, np.float32)
    u = _c(u, np.float32)
    p = np.zeros_like(g)
    lib().orc_sqrelu_mul(g.reshape(-1), u.reshape(-1), g.size, p.reshape(-1))
    return p


def soft_max_ext(x: np.ndarray, mask, scale: float) -> np.ndarray:
    x = _c(x, np.float32)
    M, N = x.shape
    mask = None if mask is None else _c(mask, np.float32)
    mrows = 1 if mask is None else mask.shape[0]
    y = np.zeros((M, N), np.float32)
    lib().orc_soft_max_ext(x, _ptr(mask), mrows, M, N, float(scale), y)
    return y


def ffn_block(x, g1, g2, eps, w_gate, w_up, w_down, H, F, want_p=False):
    x = _c(x, np.float32)
    M = x.shape[0]
    y = np.zeros((M, H), np.float32)
    p = np.zeros((M, F), np.float32) if want_p else None
    lib().orc_ffn_block(x, M, H, F, _c(g1, np.float32), _c(g2, np.float32), float(eps),
                        _c(w_gate, np.uint8), _c(w_up, np.uint8), _c(w_down, np.uint8), y, _ptr(p))
    return (y, p) if want_p else y


def fast_mul_mat_i2s(packed, x, N, nthreads):
    x = _c(x, np.float32)
    M, K = x.shape
    y = np.zeros((M, N), np.float32)
    lib().orc_fast_mul_mat_i2s(_c(packed, np.uint8), x, M, N, K, y, int(nthreads))
    return y


def fast_ffn_block(x, g1, g2, eps, w_gate, w_up, w_down, H, F, nthreads):
    x = _c(x, np.float32)
    M = x.shape[0]
    y = np.zeros((M, H), np.float32)
    lib().orc_fast_ffn_block(x, M, H, F, _c(g1, np.float32), _c(g2, np.float32), float(eps),
                             _c(w_gate, np.uint8), _c(w_up, np.uint8), _c(w_down, np.uint8), y,
                             int(nthreads))
    return y


def fast_isa() -> int:
    return int(lib().orc_fast_isa())


# ------------------------------------------------------------------------------ BitVLA-shape forward
class BitVLAConfig(C.Structure):
    """Field-for-field mirror of b2s_bitvla_config (include/b2s_bitvla.h)."""
    _fields_ = [("image_size", C.c_int), ("patch", C.c_int), ("vit_layers", C.c_int), ("vit_hidden", C.c_int),
                ("vit_ffn", C.c_int), ("vit_heads", C.c_int), ("vit_eps", C.c_float), ("conn_hidden", C.c_int),
                ("dec_layers", C.c_int), ("dec_hidden", C.c_int), ("dec_ffn", C.c_int), ("dec_heads", C.c_int),
                ("dec_kv_heads", C.c_int), ("head_dim", C.c_int), ("rope_theta", C.c_float), ("dec_eps", C.c_float),
                ("vocab", C.c_int), ("n_text", C.c_int), ("action_chunk", C.c_int), ("action_dim", C.c_int),
                ("attention_tc", C.c_int)]


def bitvla_config(**over) -> BitVLAConfig:
    """The BitVLA shape (224px/14 ViT 27x1152/4304/16h, connector 2560, decoder 30x2560/6912, 20/5 heads)."""
    d = dict(image_size=224, patch=14, vit_layers=27, vit_hidden=1152, vit_ffn=4304, vit_heads=16, vit_eps=1e-6,
             conn_hidden=2560, dec_layers=30, dec_hidden=2560, dec_ffn=6912, dec_heads=20, dec_kv_heads=5,
             head_dim=128, rope_theta=500000.0, dec_eps=1e-5, vocab=128256, n_text=32, action_chunk=8,
             action_dim=7)
    d.update(over)
    return BitVLAConfig(**d)


def bitvla_seq_len(cfg: BitVLAConfig) -> int:
    g = cfg.image_size // cfg.patch
    return g * g + cfg.n_text


def bitvla_forward(cfg: BitVLAConfig, seed: int, images: np.ndarray, tokens: np.ndarray, nthreads: int = 0):
    """(hidden [B*seq, dec_hidden], actions [B, chunk*dim]) of the oracle forward."""
    images = _c(images, np.float32)
    tokens = _c(tokens, np.int32)
    B = images.shape[0]
    seq = bitvla_seq_len(cfg)
    hidden = np.zeros((B * seq, cfg.dec_hidden), np.float32)
    actions = np.zeros((B, cfg.action_chunk * cfg.action_dim), np.float32)
    nth = nthreads or (os.cpu_count() or 1)
    rc = lib().orc_bitvla_forward(C.byref(cfg), seed & 0xFFFFFFFF, B, images, tokens.ctypes.data_as(C.c_void_p),
                                  hidden.ctypes.data_as(C.c_void_p), actions.ctypes.data_as(C.c_void_p), nth)
    assert rc == 0
    return hidden, actions


class BitVLAModel:
    """The oracle's BitVLA-shape model with every weight generated once (host memory), for repeated
    forwards (the timed CPU baseline); bitvla_forward regenerates the weights on each call."""

    def __init__(self, cfg: BitVLAConfig, seed: int, nthreads: int = 0):
        self.cfg = cfg
        self.nth = nthreads or (os.cpu_count() or 1)
        self._h = lib().orc_bitvla_create(C.byref(cfg), seed & 0xFFFFFFFF, self.nth)
        if not self._h:
            raise MemoryError("orc_bitvla_create failed")

    def forward(self, images: np.ndarray, tokens: np.ndarray, want_hidden: bool = False):
        images = _c(images, np.float32)
        tokens = _c(tokens, np.int32)
        B = images.shape[0]
        cfg = self.cfg
        hidden = np.zeros((B * bitvla_seq_len(cfg), cfg.dec_hidden), np.float32) if want_hidden else None
        actions = np.zeros((B, cfg.action_chunk * cfg.action_dim), np.float32)
        rc = lib().orc_bitvla_run(self._h, B, images, tokens.ctypes.data_as(C.c_void_p),
                                  hidden.ctypes.data_as(C.c_void_p) if hidden is not None else None,
                                  actions.ctypes.data_as(C.c_void_p), self.nth)
        assert rc == 0
        return hidden, actions

    def close(self):
        if self._h:
            lib().orc_bitvla_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def bv_param_bits(seed: int, tensor: int, idx: int) -> int:
    return int(lib().orc_bv_param_bits(seed & 0xFFFFFFFF, tensor & 0xFFFFFFFF, idx & 0xFFFFFFFF))


def bv_ternary_rowpadded(rows: int, K: int, seed: int, tensor: int) -> np.ndarray:
    Kp = (K + 127) // 128 * 128
    out = np.zeros(rows * Kp // 4, np.uint8)
    lib().orc_bv_gen_ternary(out, rows, K, seed, tensor, os.cpu_count() or 1)
    return out


def bv_uniform(n: int, seed: int, tensor: int, lo: float, hi: float) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().orc_bv_gen_uniform(out, n, seed, tensor, float(lo), float(hi))
    return out


def bv_ternary_scale(seed: int, tensor: int, K: int) -> float:
    return float(lib().orc_bv_ternary_scale(seed, tensor, K))


def layer_norm(x, g, b, eps: float) -> np.ndarray:
    x = _c(x, np.float32)
    M, K = x.shape
    g = None if g is None else _c(g, np.float32)
    b = None if b is None else _c(b, np.float32)
    y = np.zeros((M, K), np.float32)
    lib().orc_layer_norm(x, _ptr(g), _ptr(b), M, K, float(eps), y)
    return y


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    f = lib().orc_gelu_tanh
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).reshape(-1)], np.float32).reshape(np.shape(x))


def det_recipf(d: np.ndarray) -> np.ndarray:
    """1/d by the device's seed-and-Newton sequence (i2s_oracle.c: orc_det_recipf)."""
    f = lib().orc_det_recipf
    return np.array([f(float(v)) for v in np.asarray(d, np.float32).reshape(-1)], np.float32).reshape(np.shape(d))


def rope_table(base: float, hd: int, n_pos: int) -> np.ndarray:
    cs = np.zeros((n_pos, hd // 2, 2), np.float32)
    lib().orc_rope_table(float(base), hd, n_pos, cs)
    return cs


def rope_neox(x: np.ndarray, n_heads: int, hd: int, base: float, pos0: int = 0, period: int = 0) -> np.ndarray:
    x = _c(x, np.float32).copy()
    M = x.shape[0]
    npos = pos0 + (period if period > 0 else M)
    cs = rope_table(base, hd, npos)
    lib().orc_rope_neox(x, M, n_heads, hd, x.shape[1], cs, period, pos0)
    return x


def attention(qkv: np.ndarray, q_off: int, k_off: int, v_off: int, batch: int, heads: int, kv_heads: int, hd: int,
              T: int, causal: bool, scale: float) -> np.ndarray:
    qkv = _c(qkv, np.float32)
    o = np.zeros((batch * T, heads * hd), np.float32)
    lib().orc_attention(qkv, qkv.shape[1], q_off, k_off, v_off, batch, heads, kv_heads, hd, T, int(causal),
                        float(scale), o, heads * hd, os.cpu_count() or 1)
    return o
