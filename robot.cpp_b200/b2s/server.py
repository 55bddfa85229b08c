"""Python binding of the batched data-parallel server in libb2s.so (C ABI in include/b2s_server.h).

``Server.bitvla(devices, ...)`` builds one BitVLA-shape engine per GPU; ``Server(engines, ...)`` serves
caller-provided engines (Python callables, e.g. fakes in tests). ``submit`` queues one observation and
returns a request id; ``wait`` returns its actions or raises B2SError with the engine's status. This is the
call a robot.cpp session makes in place of ``policy.predict`` under the global predict mutex
(robot_server/session.cpp:124).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import B2SError, check, last_error, lib as _lib
from .bitvla import Config

ERR_BUSY = -7
ERR_UNAVAILABLE = -8
ERR_TIMEOUT = -9

SETUP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)
PREDICT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_uint8), C.POINTER(C.c_int32),
                         C.POINTER(C.c_float))
DESTROY_FN = C.CFUNCTYPE(None, C.c_void_p)


class EngineOps(C.Structure):
    _fields_ = [("setup", SETUP_FN), ("predict", PREDICT_FN), ("destroy", DESTROY_FN)]


class Shape(C.Structure):
    _fields_ = [("image_bytes", C.c_int), ("n_text", C.c_int), ("action_floats", C.c_int)]


EXPORTED = ["b2s_server_create", "b2s_server_create_bitvla", "b2s_server_submit", "b2s_server_wait",
            "b2s_server_engines", "b2s_server_engine_status", "b2s_server_free", "b2s_server_engine_error"]

_bound = False


def _bind():
    global _bound
    L = _lib()
    if _bound:
        return L
    vp, i64 = C.c_void_p, C.c_int64
    sig = {
        "b2s_server_create": (C.c_int, [C.POINTER(EngineOps), C.POINTER(vp), C.c_int, C.POINTER(Shape), C.c_int,
                                        C.c_int, C.POINTER(vp)]),
        "b2s_server_create_bitvla": (C.c_int, [C.POINTER(C.c_int), C.c_int, C.POINTER(Config), C.c_uint32,
                                               C.c_char_p, C.c_int, C.c_int, C.POINTER(vp)]),
        "b2s_server_submit": (i64, [vp, vp, vp]),
        "b2s_server_wait": (C.c_int, [vp, i64, vp, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_int)]),
        "b2s_server_engines": (C.c_int, [vp]),
        "b2s_server_engine_status": (C.c_int, [vp, C.c_int, C.POINTER(C.c_int), C.POINTER(i64), C.POINTER(i64)]),
        "b2s_server_free": (None, [vp]),
        "b2s_server_engine_error": (C.c_int, [C.c_int, C.c_char_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _bound = True
    return L


class Server:
    """Batched data-parallel serving over several engines (one worker thread per engine)."""

    def __init__(self, engines=None, image_bytes=0, n_text=0, action_floats=0, max_batch=8, queue_capacity=256,
                 _handle=None, _shape=None):
        L = _bind()
        self._keep = []
        if _handle is not None:
            self._h, self.shape = _handle, _shape
            return
        # Python engines: each is an object with predict(images [B, image_bytes] uint8, tokens [B, n_text]
        # int32) -> actions [B, action_floats] float32, raising B2SError to fail.
        self.shape = (int(image_bytes), int(n_text), int(action_floats))
        py_engines = list(engines)

        def predict(ctx, batch, images, tokens, actions):
            try:
                eng = py_engines[int(ctx) - 1]
                img = np.ctypeslib.as_array(images, (batch, self.shape[0]))
                tok = np.ctypeslib.as_array(tokens, (batch, max(self.shape[1], 1)))[:, :self.shape[1]]
                out = np.asarray(eng.predict(img.copy(), tok.copy()), np.float32).reshape(batch, self.shape[2])
                np.ctypeslib.as_array(actions, (batch, self.shape[2]))[:] = out
                return 0
            except B2SError as e:
                return _bind().b2s_server_engine_error(e.status, str(e).encode())
            except Exception as e:  # any other failure is an engine failure (B2S_ERR_CUDA)
                return _bind().b2s_server_engine_error(-4, f"engine raised {e!r}".encode())

        ops = EngineOps(SETUP_FN(0), PREDICT_FN(predict), DESTROY_FN(0))
        self._keep += [ops, predict]
        ctxs = (C.c_void_p * len(py_engines))(*[i + 1 for i in range(len(py_engines))])
        sh = Shape(*self.shape)
        h = C.c_void_p()
        check(L.b2s_server_create(C.byref(ops), ctxs, len(py_engines), C.byref(sh), int(max_batch),
                                  int(queue_capacity), C.byref(h)))
        self._h = h

    @classmethod
    def bitvla(cls, devices, cfg: Config, seed: int, max_batch=8, queue_capacity=256, gguf_path=None) -> "Server":
        L = _bind()
        devs = (C.c_int * len(devices))(*devices)
        h = C.c_void_p()
        check(L.b2s_server_create_bitvla(devs, len(devices), C.byref(cfg), seed & 0xFFFFFFFF,
                                         gguf_path.encode() if gguf_path else None, int(max_batch),
                                         int(queue_capacity), C.byref(h)))
        shape = (3 * cfg.image_size ** 2, cfg.n_text, cfg.action_chunk * cfg.action_dim)
        return cls(_handle=h, _shape=shape)

    def submit(self, image_hwc: np.ndarray, tokens: np.ndarray) -> int:
        img = np.ascontiguousarray(image_hwc, np.uint8)
        tok = np.ascontiguousarray(tokens, np.int32)
        assert img.size == self.shape[0] and tok.size == self.shape[1]
        rid = _bind().b2s_server_submit(self._h, img.ctypes.data, tok.ctypes.data)
        if rid < 0:
            raise B2SError(int(rid), last_error())
        return int(rid)

    def wait(self, rid: int, timeout_ms: int = -1):
        """(actions [action_floats], latency_ms, engine) of request `rid`; raises B2SError on failure."""
        act = np.zeros(self.shape[2], np.float32)
        lat, eng = C.c_double(0.0), C.c_int(-1)
        rc = _bind().b2s_server_wait(self._h, int(rid), act.ctypes.data, int(timeout_ms), C.byref(lat), C.byref(eng))
        if rc != 0:
            err = B2SError(rc, last_error())
            err.engine = int(eng.value)
            raise err
        return act, float(lat.value), int(eng.value)

    def engine_status(self):
        L = _bind()
        out = []
        for i in range(L.b2s_server_engines(self._h)):
            ok, done, nb = C.c_int(0), C.c_int64(0), C.c_int64(0)
            check(L.b2s_server_engine_status(self._h, i, C.byref(ok), C.byref(done), C.byref(nb)))
            out.append({"healthy": bool(ok.value), "completed": int(done.value), "batches": int(nb.value)})
        return out

    def close(self):
        if getattr(self, "_h", None):
            _bind().b2s_server_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

