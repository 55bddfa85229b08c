"""GGUF files with i2_s tensors for the BitVLA-shape model: writer, reader and command line.

There is no BitVLA checkpoint (and no BitVLA converter in the reference: its converters emit
f32/f16/bf16 only, tools/hf2gguf/pi0/gguf_writer.py:82-91). This module writes the random-init model of
b2s_bitvla_create(seed) as a GGUF v3 file that b2s_bitvla_create_from_gguf loads back into the identical
model, so the GGUF path of the i2_s op (raw tensor bytes to the device, gguf_loader.cpp:115-137) is
exercised end to end.

Format: "GGUF", version 3, tensor count, kv count, kv pairs, tensor infos (name, n_dims, ne[] in ggml
order, ggml type, data offset), padding to general.alignment (32), tensor data at 32-byte aligned
offsets. Ternary weights are I2_S (ggml type 36 of the BitNet fork): the flattened x86 i2_s bytes (n/4
bytes of 2-bit codes in 128-weight blocks) followed by a 32-byte trailer whose first 4 bytes are the fp32
tensor scale -- packed by the library's own host trait b2s_i2s_quantize. Everything else is F32.
The gguf package (0.19) in this environment has no I2_S type, so this is a small self-contained writer.

Command line:
    PYTHONPATH=robot.cpp_b200 python -m b2s.gguf write model.gguf --seed 1234 [--vit-layers N --dec-layers N]
    PYTHONPATH=robot.cpp_b200 python -m b2s.gguf info model.gguf
"""
from __future__ import annotations

import struct

import numpy as np

GGML_F32 = 0
GGML_I2_S = 36
ALIGN = 32

_KV_U32, _KV_F32, _KV_STRING = 4, 6, 8

# Tensor ids of the parameter generator (include/b2s_bitvla.h); globals, then 16 slots per layer.
ID_PATCH_W, ID_PATCH_B, ID_POS, ID_POST_W, ID_POST_B, ID_CONN1, ID_CONN1_B, ID_CONN2, ID_CONN2_B, \
    ID_FINAL_NORM, ID_ACT_W, ID_ACT_B = range(1, 13)


def vit_id(l: int, slot: int) -> int:
    return 0x100 + 16 * l + slot


def dec_id(l: int, slot: int) -> int:
    return 0x10000 + 16 * l + slot


# --------------------------------------------------------------------------------------------- generator
def _mix(h):
    h = h ^ (h >> np.uint32(16))
    h = h * np.uint32(0x85EBCA6B)
    h = h ^ (h >> np.uint32(13))
    h = h * np.uint32(0xC2B2AE35)
    h = h ^ (h >> np.uint32(16))
    return h


def param_bits(seed: int, tensor: int, idx) -> np.ndarray:
    """b2s_bitvla_param_bits over an index array (uint32 arithmetic modulo 2^32)."""
    with np.errstate(over="ignore"):
        t = _mix(np.uint32(seed & 0xFFFFFFFF) ^ _mix(np.uint32(tensor & 0xFFFFFFFF) * np.uint32(0x9E3779B1)
                                                     + np.uint32(0x7F4A7C15)))
        i = np.asarray(idx, dtype=np.uint32)
        return _mix(t ^ (i * np.uint32(0x85EBCA77) + np.uint32(0x165667B1)))


def ternary(seed: int, tensor: int, rows: int, K: int) -> np.ndarray:
    """int8 [rows, K] in {-1, 0, +1}: u = bits >> 8; u < 5033165 -> -1, u < 11744051 -> 0, else +1."""
    idx = np.arange(rows * K, dtype=np.uint64).astype(np.uint32)
    u = param_bits(seed, tensor, idx) >> np.uint32(8)
    t = np.where(u < 5033165, -1, np.where(u < 11744051, 0, 1)).astype(np.int8)
    return t.reshape(rows, K)


def ternary_scale(seed: int, tensor: int, K: int) -> np.float32:
    """(0.5 + 1.5 u) / sqrt(0.6 K) in fp32, u from element 0xFFFFFFFF."""
    u = np.float32(int(param_bits(seed, tensor, 0xFFFFFFFF)) >> 8) * np.float32(1.0 / 16777216.0)
    a = np.float32(0.5) + np.float32(1.5) * u
    return np.float32(a / np.sqrt(np.float32(0.6) * np.float32(K)))


def uniform(seed: int, tensor: int, n: int, lo: float, hi: float) -> np.ndarray:
    lo32, width = np.float32(lo), np.float32(np.float32(hi) - np.float32(lo))
    u = (param_bits(seed, tensor, np.arange(n, dtype=np.uint64).astype(np.uint32)) >> np.uint32(8)).astype(
        np.float32) * np.float32(1.0 / 16777216.0)
    return (lo32 + width * u).astype(np.float32)


# --------------------------------------------------------------------------------------------- writer
def _kv_bytes(key: str, value) -> bytes:
    kb = key.encode()
    out = struct.pack("<Q", len(kb)) + kb
    if isinstance(value, str):
        vb = value.encode()
        return out + struct.pack("<IQ", _KV_STRING, len(vb)) + vb
    if isinstance(value, float):
        return out + struct.pack("<If", _KV_F32, value)
    return out + struct.pack("<II", _KV_U32, int(value))


def write_gguf(path: str, kv: dict, tensors: list) -> None:
    """tensors: list of (name, ggml_type, ne (ggml order), bytes)."""
    infos, offset = [], 0
    for name, typ, ne, data in tensors:
        nb = name.encode()
        infos.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(ne)) +
                     b"".join(struct.pack("<Q", int(d)) for d in ne) + struct.pack("<IQ", typ, offset))
        offset += (len(data) + ALIGN - 1) // ALIGN * ALIGN
    header = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kv))
    header += b"".join(_kv_bytes(k, v) for k, v in kv.items()) + b"".join(infos)
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * ((ALIGN - len(header) % ALIGN) % ALIGN))
        for _, _, _, data in tensors:
            f.write(data)
            f.write(b"\0" * ((ALIGN - len(data) % ALIGN) % ALIGN))


def _i2s_bytes(t: np.ndarray, scale: np.float32) -> bytes:
    from . import i2s_quantize_host
    return i2s_quantize_host(t.astype(np.float32) * scale).tobytes()


def bitvla_tensors(cfg, seed: int):
    """Yields (name, ggml_type, ne, bytes) of every tensor of the random-init model from `seed`."""
    D, F, P = cfg.vit_hidden, cfg.vit_ffn, cfg.patch
    H, FF, KV = cfg.dec_hidden, cfg.dec_ffn, cfg.dec_kv_heads * cfg.head_dim
    kdim = 3 * P * P
    np_ = (cfg.image_size // P) ** 2

    def f32(name, n, tid, lo, hi, ne):
        return name, GGML_F32, ne, uniform(seed, tid, n, lo, hi).tobytes()

    def tern(name, rows, K, tid):
        return name, GGML_I2_S, [K, rows], _i2s_bytes(ternary(seed, tid, rows, K), ternary_scale(seed, tid, K))

    pa = np.float32(1.0) / np.sqrt(np.float32(kdim))
    yield "v.patch_embd.weight", GGML_F32, [kdim, D], uniform(seed, ID_PATCH_W, D * kdim, -pa, pa).tobytes()
    yield f32("v.patch_embd.bias", D, ID_PATCH_B, -0.02, 0.02, [D])
    yield f32("v.position_embd.weight", np_ * D, ID_POS, -0.02, 0.02, [D, np_])
    for l in range(cfg.vit_layers):
        v = f"v.blk.{l}."
        yield f32(v + "ln1.weight", D, vit_id(l, 0), 0.9, 1.1, [D])
        yield f32(v + "ln1.bias", D, vit_id(l, 1), -0.02, 0.02, [D])
        for j, nm in enumerate(("attn_q", "attn_k", "attn_v")):
            yield tern(v + nm + ".weight", D, D, vit_id(l, 2 + j))
            yield f32(v + nm + ".bias", D, vit_id(l, 5 + j), -0.02, 0.02, [D])
        yield tern(v + "attn_out.weight", D, D, vit_id(l, 8))
        yield f32(v + "attn_out.bias", D, vit_id(l, 9), -0.02, 0.02, [D])
        yield f32(v + "ln2.weight", D, vit_id(l, 10), 0.9, 1.1, [D])
        yield f32(v + "ln2.bias", D, vit_id(l, 11), -0.02, 0.02, [D])
        yield tern(v + "ffn_up.weight", F, D, vit_id(l, 12))
        yield f32(v + "ffn_up.bias", F, vit_id(l, 13), -0.02, 0.02, [F])
        yield tern(v + "ffn_down.weight", D, F, vit_id(l, 14))
        yield f32(v + "ffn_down.bias", D, vit_id(l, 15), -0.02, 0.02, [D])
    yield f32("v.post_ln.weight", D, ID_POST_W, 0.9, 1.1, [D])
    yield f32("v.post_ln.bias", D, ID_POST_B, -0.02, 0.02, [D])
    yield tern("mm.0.weight", cfg.conn_hidden, D, ID_CONN1)
    yield f32("mm.0.bias", cfg.conn_hidden, ID_CONN1_B, -0.02, 0.02, [cfg.conn_hidden])
    yield tern("mm.2.weight", H, cfg.conn_hidden, ID_CONN2)
    yield f32("mm.2.bias", H, ID_CONN2_B, -0.02, 0.02, [H])
    for l in range(cfg.dec_layers):
        b = f"blk.{l}."
        yield f32(b + "attn_norm.weight", H, dec_id(l, 0), 0.9, 1.1, [H])
        yield tern(b + "attn_q.weight", H, H, dec_id(l, 1))
        yield tern(b + "attn_k.weight", KV, H, dec_id(l, 2))
        yield tern(b + "attn_v.weight", KV, H, dec_id(l, 3))
        yield f32(b + "attn_sub_norm.weight", H, dec_id(l, 4), 0.9, 1.1, [H])
        yield tern(b + "attn_output.weight", H, H, dec_id(l, 5))
        yield f32(b + "ffn_norm.weight", H, dec_id(l, 6), 0.9, 1.1, [H])
        yield tern(b + "ffn_gate.weight", FF, H, dec_id(l, 7))
        yield tern(b + "ffn_up.weight", FF, H, dec_id(l, 8))
        yield f32(b + "ffn_sub_norm.weight", FF, dec_id(l, 9), 0.9, 1.1, [FF])
        yield tern(b + "ffn_down.weight", H, FF, dec_id(l, 10))
    yield f32("output_norm.weight", H, ID_FINAL_NORM, 0.9, 1.1, [H])
    na = cfg.action_chunk * cfg.action_dim
    aa = np.float32(1.0) / np.sqrt(np.float32(H))
    yield "action_head.weight", GGML_F32, [H, na], uniform(seed, ID_ACT_W, na * H, -aa, aa).tobytes()
    yield f32("action_head.bias", na, ID_ACT_B, -0.02, 0.02, [na])


def bitvla_kv(cfg, seed: int) -> dict:
    return {
        "general.architecture": "bitvla", "general.name": f"bitvla random-init seed {seed}",
        "general.alignment": ALIGN,
        "bitvla.image_size": cfg.image_size, "bitvla.patch_size": cfg.patch,
        "bitvla.vision.block_count": cfg.vit_layers, "bitvla.vision.embedding_length": cfg.vit_hidden,
        "bitvla.vision.feed_forward_length": cfg.vit_ffn, "bitvla.vision.attention.head_count": cfg.vit_heads,
        "bitvla.vision.attention.layer_norm_epsilon": float(cfg.vit_eps),
        "bitvla.connector.embedding_length": cfg.conn_hidden, "bitvla.block_count": cfg.dec_layers,
        "bitvla.embedding_length": cfg.dec_hidden, "bitvla.feed_forward_length": cfg.dec_ffn,
        "bitvla.attention.head_count": cfg.dec_heads, "bitvla.attention.head_count_kv": cfg.dec_kv_heads,
        "bitvla.attention.key_length": cfg.head_dim, "bitvla.rope.freq_base": float(cfg.rope_theta),
        "bitvla.attention.layer_norm_rms_epsilon": float(cfg.dec_eps), "bitvla.vocab_size": cfg.vocab,
        "bitvla.text_tokens": cfg.n_text, "bitvla.action.chunk_size": cfg.action_chunk,
        "bitvla.action.dim": cfg.action_dim, "bitvla.token_embd.seed": seed & 0xFFFFFFFF,
    }


def write_bitvla(path: str, cfg, seed: int) -> None:
    write_gguf(path, bitvla_kv(cfg, seed), list(bitvla_tensors(cfg, seed)))


# --------------------------------------------------------------------------------------------- reader
class GgufFile:
    """Minimal GGUF v2/v3 reader: metadata dict, tensor infos, memory-mapped tensor bytes."""

    def __init__(self, path: str):
        self.path = path
        self.kv, self.tensors = {}, {}
        with open(path, "rb") as f:
            buf = f.read()
        self._buf = memoryview(buf)
        p = 0

        def take(fmt):
            nonlocal p
            v = struct.unpack_from(fmt, buf, p)
            p += struct.calcsize(fmt)
            return v if len(v) > 1 else v[0]

        def string():
            nonlocal p
            n = take("<Q")
            s = bytes(buf[p:p + n]).decode()
            p += n
            return s

        scal = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                12: "<d"}
        magic, version, n_t, n_kv = take("<IIQQ")
        if magic != 0x46554747 or version not in (2, 3):
            raise ValueError("not a GGUF v2/v3 file")
        for _ in range(n_kv):
            key, typ = string(), take("<I")
            if typ == 8:
                self.kv[key] = string()
            elif typ == 9:
                at, n = take("<IQ")
                self.kv[key] = [string() if at == 8 else take(scal[at]) for _ in range(n)]
            else:
                self.kv[key] = take(scal[typ])
        infos = []
        for _ in range(n_t):
            name = string()
            nd = take("<I")
            ne = [take("<Q") for _ in range(nd)]
            typ, off = take("<IQ")
            infos.append((name, ne, typ, off))
        align = int(self.kv.get("general.alignment", ALIGN))
        data0 = (p + align - 1) // align * align
        for name, ne, typ, off in infos:
            n = int(np.prod(ne))
            nbytes = n * 4 if typ == GGML_F32 else (n // 4 + 32 if typ == GGML_I2_S else 0)
            self.tensors[name] = {"ne": ne, "type": typ, "offset": data0 + off, "nbytes": nbytes}

    def data(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return np.frombuffer(self._buf[t["offset"]:t["offset"] + t["nbytes"]], dtype=np.uint8)

    def f32(self, name: str) -> np.ndarray:
        return self.data(name).view(np.float32)


def _main(argv=None) -> None:
    import argparse
    from . import bitvla
    p = argparse.ArgumentParser(description="BitVLA-shape GGUF files with i2_s tensors")
    sub = p.add_subparsers(dest="cmd", required=True)
    w = sub.add_parser("write")
    w.add_argument("path")
    w.add_argument("--seed", type=int, default=1234)
    w.add_argument("--vit-layers", type=int, default=None)
    w.add_argument("--dec-layers", type=int, default=None)
    i = sub.add_parser("info")
    i.add_argument("path")
    a = p.parse_args(argv)
    if a.cmd == "write":
        over = {}
        if a.vit_layers is not None:
            over["vit_layers"] = a.vit_layers
        if a.dec_layers is not None:
            over["dec_layers"] = a.dec_layers
        cfg = bitvla.default_config(**over)
        write_bitvla(a.path, cfg, a.seed)
        print(f"wrote {a.path}")
    else:
        g = GgufFile(a.path)
        n_i2s = sum(1 for t in g.tensors.values() if t["type"] == GGML_I2_S)
        size = sum(t["nbytes"] for t in g.tensors.values())
        print(f"{a.path}: {len(g.tensors)} tensors ({n_i2s} I2_S), {size / 1e6:.1f} MB of tensor data")
        for k, v in g.kv.items():
            print(f"  {k} = {v}")


if __name__ == "__main__":
    _main()
