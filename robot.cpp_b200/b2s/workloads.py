"""Seeded synthetic inputs with the shapes and value distributions of the i2_s workloads.

There are no BitVLA checkpoints or datasets here; every workload is random-init with these generators
(numpy PCG64, fixed seeds), created on the host so that the CUDA path and the oracle see identical bytes:
  * ternary weights: P(0)=0.4, P(-1)=P(+1)=0.3, one fp32 scale per matrix drawn U(0.5, 2);
  * activations: fp32 N(0, 1);
  * RMSNorm weights: N(1, 0.1).
Packing uses the library's own host from_float trait (b2s_i2s_quantize).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import i2s_quantize_host

# The five workload families (sizes as published for the path).
FFN_BLOCK = dict(M=300, H=2560, F=6912, eps=1e-5)         # BitNet-b1.58-2B-shape FFN block, prefill 300 tokens
SINGLE_GEMM = dict(M=256, K=2560, N=2560)                  # one i2_s mul_mat
SWEEP_M = (1, 16, 256, 4096, 16384)
SWEEP_KN = ((2560, 2560), (2560, 6912), (6912, 2560), (1152, 4304))


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def ternary(g: np.random.Generator, N: int, K: int) -> np.ndarray:
    return g.choice(np.array([-1, 0, 1], np.int8), size=(N, K), p=[0.3, 0.4, 0.3])


@dataclass
class I2sWeightHost:
    t: np.ndarray        # int8 ternary [N, K]
    scale: np.float32
    packed: np.ndarray   # uint8 i2_s bytes (flattened layout)
    N: int
    K: int


def weight(g: np.random.Generator, N: int, K: int) -> I2sWeightHost:
    t = ternary(g, N, K)
    sc = np.float32(g.uniform(0.5, 2.0))
    packed = i2s_quantize_host(t.astype(np.float32) * sc)
    return I2sWeightHost(t=t, scale=sc, packed=packed, N=N, K=K)


def activations(g: np.random.Generator, M: int, K: int) -> np.ndarray:
    return g.standard_normal((M, K), dtype=np.float32)


def norm_weight(g: np.random.Generator, K: int) -> np.ndarray:
    return (1.0 + 0.1 * g.standard_normal(K)).astype(np.float32)


@dataclass
class FfnHost:
    x: np.ndarray
    g1: np.ndarray
    g2: np.ndarray
    w_gate: I2sWeightHost
    w_up: I2sWeightHost
    w_down: I2sWeightHost
    eps: float
    M: int
    H: int
    F: int


def ffn_block(seed: int, M: int = 300, H: int = 2560, F: int = 6912, eps: float = 1e-5) -> FfnHost:
    g = rng(seed)
    return FfnHost(x=activations(g, M, H), g1=norm_weight(g, H), g2=norm_weight(g, F), w_gate=weight(g, F, H),
                   w_up=weight(g, F, H), w_down=weight(g, H, F), eps=eps, M=M, H=H, F=F)
