"""Python binding of the BitVLA-shape engine in libb2s.so (C ABI in include/b2s_bitvla.h).

A ``Model`` owns a random-init BitVLA-shape network on one GPU (weights generated on the device from a
seed) and runs whole-observation forwards through the library's CUDA graph. ``predict`` mirrors
``robotcpp::Model::predict`` (src/models/model.h:65-71): host images and tokens in, host actions out.
"""
from __future__ import annotations

import ctypes as C

from . import check, lib as _lib, _ptr, _stream


class Config(C.Structure):
    """Mirror of b2s_bitvla_config."""
    _fields_ = [("image_size", C.c_int), ("patch", C.c_int), ("vit_layers", C.c_int), ("vit_hidden", C.c_int),
                ("vit_ffn", C.c_int), ("vit_heads", C.c_int), ("vit_eps", C.c_float), ("conn_hidden", C.c_int),
                ("dec_layers", C.c_int), ("dec_hidden", C.c_int), ("dec_ffn", C.c_int), ("dec_heads", C.c_int),
                ("dec_kv_heads", C.c_int), ("head_dim", C.c_int), ("rope_theta", C.c_float), ("dec_eps", C.c_float),
                ("vocab", C.c_int), ("n_text", C.c_int), ("action_chunk", C.c_int), ("action_dim", C.c_int),
                ("attention_tc", C.c_int)]


_bound = False


def _bind():
    global _bound
    L = _lib()
    if _bound:
        return L
    vp, i64 = C.c_void_p, C.c_int64
    P = C.POINTER(Config)
    sig = {
        "b2s_bitvla_default_config": (None, [P]),
        "b2s_bitvla_seq_len": (C.c_int, [P]),
        "b2s_bitvla_ternary_ops": (C.c_double, [P]),
        "b2s_bitvla_param_bits": (C.c_uint32, [C.c_uint32, C.c_uint32, C.c_uint32]),
        "b2s_bitvla_create": (C.c_int, [P, C.c_uint32, C.c_int, C.POINTER(vp)]),
        "b2s_bitvla_free": (None, [vp]),
        "b2s_bitvla_ternary_bytes": (C.c_size_t, [vp]),
        "b2s_bitvla_weight_bytes": (C.c_size_t, [vp]),
        "b2s_bitvla_activation_bytes": (C.c_size_t, [vp]),
        "b2s_bitvla_forward": (C.c_int, [vp, C.c_int, vp, vp, vp, vp, vp]),
        "b2s_bitvla_predict": (C.c_int, [vp, C.c_int, vp, vp, vp, vp]),
        "b2s_bitvla_create_from_gguf": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(vp)]),
        "b2s_bitvla_get_config": (C.c_int, [vp, P]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _bound = True
    return L


EXPORTED = ["b2s_bitvla_default_config", "b2s_bitvla_seq_len", "b2s_bitvla_ternary_ops", "b2s_bitvla_param_bits",
            "b2s_bitvla_create", "b2s_bitvla_free", "b2s_bitvla_ternary_bytes", "b2s_bitvla_weight_bytes",
            "b2s_bitvla_activation_bytes", "b2s_bitvla_forward", "b2s_bitvla_predict", "b2s_bitvla_create_from_gguf",
            "b2s_bitvla_get_config"]


def default_config(**over) -> Config:
    c = Config()
    _bind().b2s_bitvla_default_config(C.byref(c))
    for k, v in over.items():
        setattr(c, k, v)
    return c


def seq_len(cfg: Config) -> int:
    return int(_bind().b2s_bitvla_seq_len(C.byref(cfg)))


def ternary_ops(cfg: Config) -> float:
    return float(_bind().b2s_bitvla_ternary_ops(C.byref(cfg)))


def param_bits(seed: int, tensor: int, idx: int) -> int:
    return int(_bind().b2s_bitvla_param_bits(seed & 0xFFFFFFFF, tensor & 0xFFFFFFFF, idx & 0xFFFFFFFF))


class Model:
    """A BitVLA-shape model on the current CUDA device."""

    def __init__(self, cfg: Config, seed: int, max_batch: int = 1, gguf_path: str | None = None):
        """Random-init model from `seed`, or (gguf_path) the model stored in a GGUF file; for a file the
        shape comes from its metadata and `cfg`/`seed` are only recorded."""
        L = _bind()
        self.max_batch = max_batch
        h = C.c_void_p()
        if gguf_path is not None:
            check(L.b2s_bitvla_create_from_gguf(gguf_path.encode(), max_batch, C.byref(h)))
            from .gguf import GgufFile
            cfg = Config()
            check(L.b2s_bitvla_get_config(h, C.byref(cfg)))
            seed = GgufFile(gguf_path).kv["bitvla.token_embd.seed"]
        else:
            check(L.b2s_bitvla_create(C.byref(cfg), seed & 0xFFFFFFFF, max_batch, C.byref(h)))
        self.cfg = cfg
        self.seed = seed
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            _bind().b2s_bitvla_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def seq_len(self) -> int:
        return seq_len(self.cfg)

    def ternary_bytes(self) -> int:
        return int(_bind().b2s_bitvla_ternary_bytes(self._h))

    def weight_bytes(self) -> int:
        return int(_bind().b2s_bitvla_weight_bytes(self._h))

    def activation_bytes(self) -> int:
        return int(_bind().b2s_bitvla_activation_bytes(self._h))

    def forward(self, images, tokens, hidden=None, actions=None, stream=None) -> None:
        """Device tensors: images [B,3,S,S] f32, tokens [B,n_text] i32 -> hidden [B*seq, H], actions [B, A]."""
        B = images.shape[0]
        check(_bind().b2s_bitvla_forward(self._h, B, _ptr(images), _ptr(tokens), _ptr(hidden), _ptr(actions),
                                         _stream(stream)))

    def predict(self, images_hwc, tokens, actions, stream=None) -> None:
        """Host numpy arrays: images [B,S,S,3] uint8, tokens [B,n_text] int32 -> actions [B, A] float32."""
        B = images_hwc.shape[0]
        check(_bind().b2s_bitvla_predict(self._h, B, images_hwc.ctypes.data, tokens.ctypes.data,
                                         actions.ctypes.data, _stream(stream)))


def _main(argv=None) -> None:
    """Times forwards of the BitVLA shape on cuda:0; with --profile-range the timed forwards are bracketed
    by cudaProfilerStart/Stop (for `ncu --profile-from-start off`).

        PYTHONPATH=robot.cpp_b200 python -m b2s.bitvla --batch 8 --iters 1 --profile-range
    """
    import argparse
    import torch

    p = argparse.ArgumentParser(description=_main.__doc__)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--profile-range", action="store_true")
    p.add_argument("--attention-tc", action="store_true",
                   help="tensor-core attention (opt-in; not bit-identical to the fixed-order fp32 kernel)")
    a = p.parse_args(argv)
    cfg = default_config()
    cfg.attention_tc = 1 if a.attention_tc else 0
    m = Model(cfg, a.seed, max_batch=a.batch)
    img = torch.rand((a.batch, 3, cfg.image_size, cfg.image_size), device="cuda")
    tok = torch.randint(0, cfg.vocab, (a.batch, cfg.n_text), dtype=torch.int32, device="cuda")
    act = torch.zeros((a.batch, cfg.action_chunk * cfg.action_dim), device="cuda")
    for _ in range(3):  # the first call captures the graph
        m.forward(img, tok, None, act)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.profile_range:
        torch.cuda.cudart().cudaProfilerStart()
    e0.record()
    for _ in range(a.iters):
        m.forward(img, tok, None, act)
    e1.record()
    torch.cuda.synchronize()
    if a.profile_range:
        torch.cuda.cudart().cudaProfilerStop()
    ms = e0.elapsed_time(e1) / a.iters
    print(f"batch {a.batch}: {ms:.3f} ms per forward, {a.batch / ms * 1e3:.1f} obs/s, "
          f"{ternary_ops(cfg) * a.batch / ms / 1e9:.1f} ternary TOP/s")
    m.close()


if __name__ == "__main__":
    _main()
