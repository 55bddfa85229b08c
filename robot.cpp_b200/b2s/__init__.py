"""Python binding of libb2s.so, the B200 ternary i2_s mul_mat library (C ABI in include/b2s.h).

This is the ctypes path a Python caller of the reference uses for native ggml code (the quant tool binds
libggml-base the same way, tools/quant/quantize-vla-gguf.py:47-53). Device buffers and streams come from
torch (plumbing only); every op runs the library's own CUDA kernels. There is no fallback: if the shared
library is missing or fails to load, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb2s.so")

B2S_OK = 0
B2S_ERR_INVALID_ARG = -1
B2S_ERR_UNSUPPORTED = -2
B2S_ERR_WORKSPACE = -3
B2S_ERR_CUDA = -4
B2S_ERR_DEVICE = -5
B2S_ERR_DEVICE_TIMEOUT = -6

TYPE_F32 = 0
TYPE_I8 = 24
TYPE_I32 = 26
TYPE_I2_S = 36
TYPE_I2_S_R = 1036

# Every symbol include/b2s.h declares (checked by the CPU test suite against the built library).
EXPORTED = [
    "b2s_version", "b2s_last_error", "b2s_device_check", "b2s_device_error",
    "b2s_i2s_nbytes", "b2s_i2s_r_nbytes", "b2s_i2s_quantize", "b2s_i2s_dequantize",
    "b2s_i2s_repack_rows", "b2s_act_quant", "b2s_rms_norm_act_quant", "b2s_mul_mat_workspace_size",
    "b2s_mul_mat", "b2s_mul_mat_q8", "b2s_mul_mat_q8_ex", "b2s_ffn_gate_up_sqrelu_q8",
    "b2s_ffn_block_workspace_size", "b2s_ffn_block", "b2s_soft_max_ext", "b2s_mul_mat_static",
    "b2s_mul_mat_q8_epi", "b2s_norm", "b2s_norm_act_quant", "b2s_rope_neox", "b2s_attention",
    "b2s_patch_embed", "b2s_embed_tokens_hash", "b2s_nsplit_range", "b2s_i2s_shard_rows", "b2s_peer_export",
    "b2s_peer_open", "b2s_peer_close", "b2s_debug_wait_timeout", "b2s_attention_tc", "b2s_mul_mat_q8_batched",
]
PEER_HANDLE_BYTES = 72


class B2SError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"b2s status {status}: {msg}")
        self.status = status


class Tensor(C.Structure):
    """Mirror of ``b2s_tensor`` (= the ggml_tensor fields an op reads)."""
    _fields_ = [("type", C.c_int32), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4), ("data", C.c_void_p)]


_lib = None
_vp = C.c_void_p
_i64 = C.c_int64
_TP = C.POINTER(Tensor)


def lib():
    """Load libb2s.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C robot.cpp_b200/csrc` "
                               "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        sig = {
            "b2s_version": (C.c_char_p, []),
            "b2s_last_error": (C.c_char_p, []),
            "b2s_device_check": (C.c_int, []),
            "b2s_device_error": (C.c_int, [C.POINTER(C.c_uint32), C.c_int]),
            "b2s_i2s_nbytes": (C.c_size_t, [_i64, _i64]),
            "b2s_i2s_r_nbytes": (C.c_size_t, [_i64, _i64]),
            "b2s_i2s_quantize": (C.c_size_t, [_vp, _vp, _i64, _i64]),
            "b2s_i2s_dequantize": (C.c_int, [_vp, _vp, _i64, _i64]),
            "b2s_i2s_repack_rows": (C.c_int, [_vp, _vp, _i64, _i64, _vp]),
            "b2s_act_quant": (C.c_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
            "b2s_rms_norm_act_quant": (C.c_int, [_vp, _vp, _i64, _i64, _i64, C.c_float, _vp, _i64, _vp, _vp, _vp]),
            "b2s_mul_mat_workspace_size": (C.c_size_t, [_TP, _TP]),
            "b2s_mul_mat": (C.c_int, [_TP, _TP, _TP, _vp, C.c_size_t, _vp]),
            "b2s_mul_mat_q8": (C.c_int, [_TP, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _vp]),
            "b2s_mul_mat_q8_ex": (C.c_int, [_TP, _vp, _i64, _vp, _vp, _i64, _vp, _i64, C.c_int, _vp]),
            "b2s_ffn_gate_up_sqrelu_q8": (C.c_int, [_TP, _TP, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _vp]),
            "b2s_ffn_block_workspace_size": (C.c_size_t, [_i64, _i64, _i64]),
            "b2s_ffn_block": (C.c_int, [_vp, _i64, _vp, _vp, C.c_float, _TP, _TP, _TP, _vp, _vp, C.c_size_t, _vp]),
            "b2s_soft_max_ext": (C.c_int, [_vp, _vp, _i64, _i64, _i64, C.c_float, _vp, _vp]),
            "b2s_mul_mat_static": (C.c_int, [_TP, _TP, _TP, _vp]),
            "b2s_mul_mat_q8_epi": (C.c_int, [_TP, _vp, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _i64, C.c_int,
                                             _vp]),
            "b2s_norm": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, C.c_float, C.c_int, _vp, _i64, _vp]),
            "b2s_norm_act_quant": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, C.c_float, C.c_int, _vp, _i64, _vp,
                                             _vp, _vp]),
            "b2s_rope_neox": (C.c_int, [_vp, _i64, C.c_int, C.c_int, _i64, C.c_float, C.c_int, _vp]),
            "b2s_attention": (C.c_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, C.c_int, C.c_int, C.c_int, C.c_float,
                                        C.c_int, _vp, _i64, _vp]),
            "b2s_mul_mat_q8_batched": (C.c_int, [_TP, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp]),
            "b2s_attention_tc": (C.c_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, C.c_int, C.c_int, C.c_int,
                                           C.c_float, C.c_int, _vp, _i64, _vp]),
            "b2s_patch_embed": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _i64,
                                          _vp]),
            "b2s_embed_tokens_hash": (C.c_int, [_vp, C.c_int, C.c_int, C.c_uint32, _vp, _i64, _vp]),
            "b2s_nsplit_range": (C.c_int, [_i64, C.c_int, C.c_int, C.POINTER(_i64), C.POINTER(_i64)]),
            "b2s_i2s_shard_rows": (C.c_size_t, [_vp, C.c_int32, _i64, _i64, _i64, _i64, _vp]),
            "b2s_peer_export": (C.c_int, [_vp, _vp, C.c_size_t]),
            "b2s_peer_open": (C.c_int, [_vp, C.c_size_t, C.POINTER(_vp)]),
            "b2s_peer_close": (C.c_int, [_vp]),
            "b2s_debug_wait_timeout": (C.c_int, [_vp, C.c_size_t, C.c_uint64, _vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().b2s_last_error().decode()


def check(status: int) -> None:
    if status != B2S_OK:
        raise B2SError(status, last_error())


def version() -> str:
    return lib().b2s_version().decode()


def debug_wait_timeout(src, wait_limit_ns: int, stream=None) -> None:
    """Runs the bounded-wait failure path once (b2s_debug_wait_timeout) on a device byte buffer `src`."""
    check(lib().b2s_debug_wait_timeout(_ptr(src), src.numel() * src.element_size(), int(wait_limit_ns),
                                       _stream(stream)))


def device_error(clear: bool = True) -> int:
    v = C.c_uint32(0)
    check(lib().b2s_device_error(C.byref(v), int(clear)))
    return int(v.value)


# ---------------------------------------------------------------------------------------------- tensors
def _ptr(t) -> int | None:
    if t is None:
        return None
    return int(t.data_ptr())


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return int(torch.cuda.current_stream().cuda_stream)
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


def i2s_tensor(buf, N: int, K: int, rowpadded: bool = False) -> Tensor:
    """Descriptor of an i2_s weight (ne=[K,N]) stored in the device byte buffer ``buf``."""
    t = Tensor()
    t.type = TYPE_I2_S_R if rowpadded else TYPE_I2_S
    t.ne[:] = [K, N, 1, 1]
    rb = (((K + 127) // 128) * 128 // 4) if rowpadded else K // 4
    t.nb[:] = [1, rb, rb * N, rb * N]
    t.data = _ptr(buf)
    return t


def f32_tensor(x) -> Tensor:
    """Descriptor of a 2-D float32 torch tensor [rows, cols] as ggml ne=[cols, rows]."""
    assert x.dtype.is_floating_point and x.element_size() == 4 and x.dim() == 2 and x.stride(1) == 1
    t = Tensor()
    t.type = TYPE_F32
    t.ne[:] = [x.shape[1], x.shape[0], 1, 1]
    t.nb[:] = [4, x.stride(0) * 4, x.stride(0) * 4 * x.shape[0], x.stride(0) * 4 * x.shape[0]]
    t.data = _ptr(x)
    return t


def i2s_nbytes(N: int, K: int) -> int:
    return int(lib().b2s_i2s_nbytes(N, K))


def i2s_r_nbytes(N: int, K: int) -> int:
    return int(lib().b2s_i2s_r_nbytes(N, K))


def i2s_quantize_host(w):
    """from_float on the host: numpy float32 [N, K] -> numpy uint8 i2_s bytes."""
    import numpy as np
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.zeros(i2s_nbytes(N, K), np.uint8)
    n = lib().b2s_i2s_quantize(w.ctypes.data, out.ctypes.data, N, K)
    if n == 0:
        raise B2SError(B2S_ERR_UNSUPPORTED, last_error())
    return out


def i2s_dequantize_host(buf, N: int, K: int):
    import numpy as np
    buf = np.ascontiguousarray(buf, dtype=np.uint8)
    out = np.zeros((N, K), np.float32)
    check(lib().b2s_i2s_dequantize(buf.ctypes.data, out.ctypes.data, N, K))
    return out


# ---------------------------------------------------------------------------------------------- device ops
def repack_rows(src, dst, N: int, K: int, stream=None) -> None:
    check(lib().b2s_i2s_repack_rows(_ptr(src), _ptr(dst), N, K, _stream(stream)))


def act_quant(x, q, s, sums=None, stream=None) -> None:
    M, K = x.shape
    check(lib().b2s_act_quant(_ptr(x), M, K, x.stride(0), _ptr(q), q.stride(0), _ptr(s), _ptr(sums), _stream(stream)))


def rms_norm_act_quant(x, g, eps: float, q, s, sums=None, stream=None) -> None:
    M, K = x.shape
    check(lib().b2s_rms_norm_act_quant(_ptr(x), _ptr(g), M, K, x.stride(0), float(eps), _ptr(q), q.stride(0),
                                       _ptr(s), _ptr(sums), _stream(stream)))


def mul_mat_workspace_size(W: Tensor, X: Tensor) -> int:
    return int(lib().b2s_mul_mat_workspace_size(C.byref(W), C.byref(X)))


def mul_mat(W: Tensor, x, y, workspace, stream=None) -> None:
    X = f32_tensor(x)
    Y = f32_tensor(y)
    check(lib().b2s_mul_mat(C.byref(W), C.byref(X), C.byref(Y), _ptr(workspace),
                            workspace.numel() * workspace.element_size(), _stream(stream)))


def mul_mat_static(W: Tensor, x, y, stream=None) -> None:
    """MUL_MAT without a workspace: for callers that may not allocate (the library's 4 MiB static scratch)."""
    X = f32_tensor(x)
    Y = f32_tensor(y)
    check(lib().b2s_mul_mat_static(C.byref(W), C.byref(X), C.byref(Y), _stream(stream)))


def mul_mat_q8(W: Tensor, q, s, sums, y, path: int = 0, stream=None) -> None:
    M = q.shape[0]
    check(lib().b2s_mul_mat_q8_ex(C.byref(W), _ptr(q), q.stride(0), _ptr(s), _ptr(sums), M, _ptr(y), y.stride(0),
                                  int(path), _stream(stream)))


def i2s_tensor_batched(buf, N: int, K: int, B: int, rowpadded: bool = False) -> Tensor:
    """Descriptor of B i2_s matrices (ne=[K,N,B]) stored back to back in ``buf`` with one trailing scale."""
    t = i2s_tensor(buf, N, K, rowpadded)
    t.ne[:] = [K, N, B, 1]
    t.nb[3] = t.nb[2] * B
    return t


def mul_mat_q8_batched(W: Tensor, q, s, sums, y, stream=None) -> None:
    """q [B, M, ldq] int8 (a strided view), s/sums [B, M], y [B, M, N] f32: y[b] = mul_mat(W[b], q[b])."""
    B, M = q.shape[0], q.shape[1]
    check(lib().b2s_mul_mat_q8_batched(C.byref(W), _ptr(q), q.stride(1), q.stride(0), _ptr(s), _ptr(sums), s.stride(0),
                                       M, _ptr(y), y.stride(1), y.stride(0), _stream(stream)))


def ffn_gate_up_sqrelu_q8(Wg: Tensor, Wu: Tensor, q, s, sums, p, stream=None) -> None:
    M = q.shape[0]
    check(lib().b2s_ffn_gate_up_sqrelu_q8(C.byref(Wg), C.byref(Wu), _ptr(q), q.stride(0), _ptr(s), _ptr(sums), M,
                                          _ptr(p), p.stride(0), _stream(stream)))


def ffn_block_workspace_size(M: int, H: int, F: int) -> int:
    return int(lib().b2s_ffn_block_workspace_size(M, H, F))


def ffn_block(x, g1, g2, eps: float, Wg: Tensor, Wu: Tensor, Wd: Tensor, y, workspace, stream=None) -> None:
    M = x.shape[0]
    check(lib().b2s_ffn_block(_ptr(x), M, _ptr(g1), _ptr(g2), float(eps), C.byref(Wg), C.byref(Wu), C.byref(Wd),
                              _ptr(y), _ptr(workspace), workspace.numel() * workspace.element_size(),
                              _stream(stream)))


def soft_max_ext(x, mask, scale: float, y, stream=None) -> None:
    M, N = x.shape
    mrows = 1 if mask is None else mask.shape[0]
    check(lib().b2s_soft_max_ext(_ptr(x), _ptr(mask), mrows, M, N, float(scale), _ptr(y), _stream(stream)))


def mul_mat_q8_epi(W: Tensor, q, s, sums, y, bias=None, residual=None, act: int = 0, stream=None) -> None:
    """y = W*q then + bias, GELU (act=1), + residual (residual may be y itself)."""
    M = q.shape[0]
    ld_res = residual.stride(0) if residual is not None else 0
    check(lib().b2s_mul_mat_q8_epi(C.byref(W), _ptr(q), q.stride(0), _ptr(s), _ptr(sums), M, _ptr(y), y.stride(0),
                                   _ptr(bias), _ptr(residual), ld_res, int(act), _stream(stream)))


NORM_RMS = 0
NORM_LAYER = 1


def norm(x, g, b, eps: float, kind: int, y, stream=None) -> None:
    M, K = x.shape
    check(lib().b2s_norm(_ptr(x), _ptr(g), _ptr(b), M, K, x.stride(0), float(eps), int(kind), _ptr(y), y.stride(0),
                         _stream(stream)))


def norm_act_quant(x, g, b, eps: float, kind: int, q, s, sums, stream=None) -> None:
    M, K = x.shape
    check(lib().b2s_norm_act_quant(_ptr(x), _ptr(g), _ptr(b), M, K, x.stride(0), float(eps), int(kind), _ptr(q),
                                   q.stride(0), _ptr(s), _ptr(sums), _stream(stream)))


def rope_neox(x, n_heads: int, head_dim: int, theta_base: float, pos0: int = 0, stream=None) -> None:
    M = x.shape[0]
    check(lib().b2s_rope_neox(_ptr(x), M, int(n_heads), int(head_dim), x.stride(0), float(theta_base), int(pos0),
                              _stream(stream)))


def attention(q, k, v, n_heads: int, n_kv_heads: int, head_dim: int, scale: float, causal: bool, o,
              stream=None) -> None:
    M = q.shape[0]
    check(lib().b2s_attention(_ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0), M, int(n_heads),
                              int(n_kv_heads), int(head_dim), float(scale), int(bool(causal)), _ptr(o), o.stride(0),
                              _stream(stream)))


def attention_tc(q, k, v, n_heads: int, n_kv_heads: int, head_dim: int, scale: float, causal: bool, o,
                 stream=None) -> None:
    """Tensor-core attention (3xTF32 products, exact-max softmax); same operands as attention()."""
    M = q.shape[0]
    check(lib().b2s_attention_tc(_ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0), M, int(n_heads),
                                 int(n_kv_heads), int(head_dim), float(scale), int(bool(causal)), _ptr(o), o.stride(0),
                                 _stream(stream)))


def patch_embed(img, P: int, w, bias, pos, y, stream=None) -> None:
    C_, H, W = img.shape
    D = w.shape[0]
    check(lib().b2s_patch_embed(_ptr(img), C_, H, W, int(P), _ptr(w), _ptr(bias), _ptr(pos), D, _ptr(y), y.stride(0),
                                _stream(stream)))


def embed_tokens_hash(tokens, dim: int, seed: int, y, stream=None) -> None:
    n = tokens.shape[0]
    check(lib().b2s_embed_tokens_hash(_ptr(tokens), n, int(dim), int(seed) & 0xFFFFFFFF, _ptr(y), y.stride(0),
                                      _stream(stream)))


# ---------------------------------------------------------------------------------------------- N-split host side
def nsplit_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [n0, n1) of an n_rows-row weight owned by `rank` of `world` (balanced, contiguous)."""
    n0, n1 = _i64(0), _i64(0)
    check(lib().b2s_nsplit_range(int(n_rows), int(world), int(rank), C.byref(n0), C.byref(n1)))
    return int(n0.value), int(n1.value)


def i2s_shard_rows(packed, N: int, K: int, r0: int, r1: int, rowpadded: bool = False):
    """Host: rows [r0, r1) of an i2_s tensor (numpy uint8 bytes) as a standalone tensor of the same type."""
    import numpy as np
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    rb = ((K + 127) // 128 * 128 // 4) if rowpadded else K // 4
    out = np.zeros(max(r1 - r0, 0) * rb + 32, np.uint8)
    n = lib().b2s_i2s_shard_rows(packed.ctypes.data, TYPE_I2_S_R if rowpadded else TYPE_I2_S, int(N), int(K),
                                 int(r0), int(r1), out.ctypes.data)
    if n == 0:
        raise B2SError(B2S_ERR_INVALID_ARG, last_error())
    return out


def peer_export(dev_ptr: int) -> bytes:
    """Peer handle (72 bytes: the enclosing allocation's CUDA IPC handle and the offset) of a device buffer."""
    h = (C.c_uint8 * PEER_HANDLE_BYTES)()
    check(lib().b2s_peer_export(int(dev_ptr), h, PEER_HANDLE_BYTES))
    return bytes(h)


def peer_open(handle: bytes) -> int:
    """Device address (in this process, current device) of a peer's exported allocation."""
    h = (C.c_uint8 * PEER_HANDLE_BYTES).from_buffer_copy(handle)
    p = _vp()
    check(lib().b2s_peer_open(h, PEER_HANDLE_BYTES, C.byref(p)))
    return int(p.value)


def peer_close(dev_ptr: int) -> None:
    check(lib().b2s_peer_close(int(dev_ptr)))
