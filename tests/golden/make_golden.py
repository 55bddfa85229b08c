"""Generates the golden fixtures in this directory (run from the repo root: python tests/golden/make_golden.py).

The reference tree holds no i2_s code, tests or vectors (its ggml submodule is empty), so these fixtures
pin the oracle's restatement of the BitNet fork's i2_s path with:
  1. hand-derived known answers (byte layout, rounding ties, the 1e-5 amax floor, saturation);
  2. an independent pure-Python/numpy restatement (loops over scalars, float32 ops one at a time),
     written without reference to the C oracle;
  3. a cross-check of the per-token act-quant against the third-party formula in
     transformers/integrations/bitnet.py (ActQuant.forward: scale = 127/max|x|.clamp(1e-5),
     round().clamp(-128,127)), on inputs that contain no exact .5 ties (transformers rounds half to
     even, the fork's C code half away from zero; the tie KAT pins the latter).
Outputs: kat.npz, random_small.npz, ffn_tiny.npz, actquant_xcheck.npz.
"""
from __future__ import annotations

import math
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def pack_py(t: np.ndarray, scale: float) -> np.ndarray:
    """Independent restatement of the flattened x86 I2_S layout: block of 128 -> 32 bytes,
    byte j%32 holds position j at shift 6-2*(j//32); code = t+1; scale after the codes."""
    flat = t.reshape(-1).astype(np.int64)
    n = flat.size
    assert n % 128 == 0
    out = bytearray(n // 4 + 32)
    for g in range(n):
        blk, j = divmod(g, 128)
        out[32 * blk + (j % 32)] |= (int(flat[g]) + 1) << (6 - 2 * (j // 32))
    out[n // 4:n // 4 + 4] = struct.pack("<f", scale)
    return np.frombuffer(bytes(out), np.uint8).copy()


def round_half_away(v: float) -> float:
    return math.floor(v + 0.5) if v >= 0 else -math.floor(-v + 0.5)


def act_quant_py(x: np.ndarray):
    M, K = x.shape
    q = np.zeros((M, K), np.int8)
    s = np.zeros(M, f32)
    sums = np.zeros(M, np.int32)
    for m in range(M):
        amax = 1e-5
        for k in range(K):
            amax = max(amax, abs(float(x[m, k])))
        sc = f32(127.0 / amax)  # double quotient rounded to float
        tot = 0
        for k in range(K):
            prod = float(f32(x[m, k]) * sc)  # fp32 product
            r = round_half_away(prod)
            r = min(127, max(-128, r))
            q[m, k] = r
            tot += r
        s[m] = sc
        sums[m] = tot
    return q, s, sums


def mul_mat_py(t: np.ndarray, ws: float, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    q, s, _ = act_quant_py(x)
    acc = (q.astype(np.int64) @ t.astype(np.int64).T).astype(np.int32)
    M, N = acc.shape
    y = np.zeros((M, N), f32)
    for m in range(M):
        r = f32(f32(ws) / s[m])
        for n in range(N):
            y[m, n] = f32(acc[m, n]) * r
    return acc, y


def rms_norm_py(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    M, K = x.shape
    y = np.zeros_like(x)
    for m in range(M):
        tot = 0.0
        for k in range(K):
            tot += float(f32(x[m, k]) * f32(x[m, k]))
        mean = f32(tot / K)
        scale = f32(f32(1.0) / f32(math.sqrt(float(f32(mean + f32(eps))))))
        for k in range(K):
            y[m, k] = f32(f32(x[m, k]) * scale) * f32(g[k])
    return y


def main() -> None:
    rng = np.random.Generator(np.random.PCG64(20261201))

    # ---------------------------------------------------------------- 1. known answers
    # Layout KAT: one block, position j carries t = (j % 3) - 1.
    t_kat = (np.arange(128) % 3 - 1).astype(np.int8).reshape(1, 128)
    kat_bytes = pack_py(t_kat, 1.5)
    # byte 0 holds positions 0,32,64,96 -> t = -1, +1 (32%3=2), 0 (64%3=1), -1 (96%3=0)
    assert kat_bytes[0] == (0 << 6) | (2 << 4) | (1 << 2) | (0 << 0)
    # Two-row tensor with K=64: rows share the first block (flattened interleave).
    t_two = rng.choice(np.array([-1, 0, 1], np.int8), size=(2, 64))
    two_bytes = pack_py(t_two, 0.75)

    # Act-quant KATs: row 0 ties (amax 127 -> s = 1 exactly; 2.5 -> 3, -2.5 -> -3, 0.5 -> 1);
    # row 1 all zeros (amax floor 1e-5 -> s = 12700000, q = 0); row 2 tiny values below the floor;
    # row 3 a single dominant value (q = +-127 at the max).
    xk = np.zeros((4, 16), f32)
    xk[0, :6] = [127.0, 2.5, -2.5, 0.5, -0.5, 1.5]
    xk[2, :3] = [5e-6, -3e-6, 9.9e-6]
    xk[3, :] = rng.standard_normal(16).astype(f32)
    xk[3, 7] = 40.0
    qk, sk, uk = act_quant_py(xk)
    assert qk[0, 1] == 3 and qk[0, 2] == -3 and qk[0, 3] == 1 and qk[0, 4] == -1 and qk[0, 5] == 2
    assert sk[1] == f32(12700000.0)
    np.savez(os.path.join(HERE, "kat.npz"), t_kat=t_kat, kat_bytes=kat_bytes, t_two=t_two, two_bytes=two_bytes,
             x_actq=xk, q_actq=qk, s_actq=sk, sum_actq=uk)

    # ---------------------------------------------------------------- 2. random small mul_mat cases
    cases = {}
    for i, (M, N, K) in enumerate([(1, 8, 128), (5, 16, 256), (17, 24, 384), (3, 32, 1152)]):
        t = rng.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])
        ws = float(f32(rng.uniform(0.5, 2.0)))
        x = rng.standard_normal((M, K)).astype(f32)
        acc, y = mul_mat_py(t, ws, x)
        q, s, sums = act_quant_py(x)
        cases.update({f"c{i}_t": t, f"c{i}_ws": np.array(ws, f32), f"c{i}_packed": pack_py(t, ws), f"c{i}_x": x,
                      f"c{i}_q": q, f"c{i}_s": s, f"c{i}_sums": sums, f"c{i}_acc": acc, f"c{i}_y": y})
    np.savez(os.path.join(HERE, "random_small.npz"), ncases=np.array(4), **cases)

    # ---------------------------------------------------------------- 3. tiny FFN block
    M, H, F, eps = 3, 128, 256, 1e-5
    x = rng.standard_normal((M, H)).astype(f32)
    g1 = (1 + 0.1 * rng.standard_normal(H)).astype(f32)
    g2 = (1 + 0.1 * rng.standard_normal(F)).astype(f32)
    tw = {k: rng.choice(np.array([-1, 0, 1], np.int8), size=sh, p=[0.3, 0.4, 0.3])
          for k, sh in (("gate", (F, H)), ("up", (F, H)), ("down", (H, F)))}
    sw = {k: float(f32(rng.uniform(0.5, 2.0))) for k in tw}
    xn = rms_norm_py(x, g1, eps)
    _, gt = mul_mat_py(tw["gate"], sw["gate"], xn)
    _, up = mul_mat_py(tw["up"], sw["up"], xn)
    r = np.where(gt > 0, gt, f32(0)).astype(f32)
    p = ((r * r).astype(f32) * up).astype(f32)
    pn = rms_norm_py(p, g2, eps)
    _, y = mul_mat_py(tw["down"], sw["down"], pn)
    np.savez(os.path.join(HERE, "ffn_tiny.npz"), x=x, g1=g1, g2=g2, eps=np.array(eps, f32),
             **{f"w_{k}": pack_py(v, sw[k]) for k, v in tw.items()}, p=p, y=y)

    # ---------------------------------------------------------------- 4. third-party act-quant cross-check
    os.environ["TORCHDYNAMO_DISABLE"] = "1"  # run ActQuant's torch.compile'd forward eagerly
    import torch
    from transformers.integrations.bitnet import ActQuant

    xc = rng.standard_normal((8, 512)).astype(f32)
    q_py, s_py, _ = act_quant_py(xc)
    with torch.no_grad():
        xt = torch.from_numpy(xc)
        deq = ActQuant.apply(xt).numpy()  # round(x*s).clamp(-128,127)/s with s = 127/max|x|
        s_tf = (127.0 / xt.abs().max(dim=-1, keepdim=True).values.clamp(min=1e-5)).numpy().reshape(-1)
    q_tf = np.rint(deq * s_tf[:, None]).astype(np.int32)
    prods = xc * s_py[:, None]
    ties = np.abs(prods - np.trunc(prods)) == 0.5
    assert not ties.any(), "regenerate with another seed: exact .5 ties differ between the two roundings"
    # torch evaluates `127 / tensor` on the CPU as a reciprocal times 127, which can land 1 ulp away from
    # the correctly rounded quotient the fork's C code produces; the int8 codes must still agree exactly.
    ulp = np.abs(s_tf.astype(f32).view(np.int32) - s_py.view(np.int32))
    assert ulp.max() <= 1 and np.array_equal(q_tf, q_py.astype(np.int32))
    np.savez(os.path.join(HERE, "actquant_xcheck.npz"), x=xc, q=q_py, s=s_py)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
