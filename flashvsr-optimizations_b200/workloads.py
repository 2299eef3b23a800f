"""Seeded synthetic inputs with the shapes and value distributions of the
reference's FFN workloads (Wan-1.3B FFN: d_model 1536, d_ff 8960).

The reference measures on real video activations and downloaded weights
(fetch_assets.py), which are not available here; these generators stand in
for them.  numpy generators are deterministic across machines, so a CPU
oracle and a GPU run see identical bf16 bit patterns.
"""
from __future__ import annotations

import numpy as np

D_MODEL = 1536
D_FF = 8960
LAYERS = 30
FLOP_PER_TOKEN = 2 * D_MODEL * D_FF * 2  # two GEMMs per FFN layer: 55,050,240

# benchmark workloads (token counts)
M_CPU_CASE = 1024          # reference torch emulation on CPU, seed 0
M_ONE_LAYER = 7680         # one layer on one GPU (2 latent frames of 48x80), seed 1
M_STACK = 15360            # 30-layer stack (4 frames of 48x80), seed 3
M_4K = 64800               # 30-layer stack, 4K stream (2 frames of 135x240), seed 4
QUANT_SWEEP_M = (1024, 4096, 16384, 65536)
QUANT_SWEEP_K = (D_MODEL, D_FF)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def gaussian(m: int, k: int, seed: int, std: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32) * np.float32(std))


def student_t(m: int, k: int, seed: int, nu: float = 4.0, scale: float = 0.5) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits((rng.standard_t(nu, size=(m, k)) * scale).astype(np.float32))


def with_outliers(m: int, k: int, seed: int, frac: float = 0.001, mult: float = 50.0) -> np.ndarray:
    """N(0,1) with a seeded 0.1% of the elements multiplied by 50 (quantize sweep)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    n_out = max(1, int(round(frac * m * k)))
    idx = rng.choice(m * k, size=n_out, replace=False)
    x.reshape(-1)[idx] *= np.float32(mult)
    return f32_to_bf16_bits(x)


def linear_params(out_f: int, in_f: int, seed: int, w_std: float = 0.02, b_std: float | None = None):
    """(weight bits [out, in], bias bits [out] or zeros) for one nn.Linear."""
    rng = np.random.default_rng(seed)
    w = f32_to_bf16_bits(rng.standard_normal((out_f, in_f), dtype=np.float32) * np.float32(w_std))
    if b_std is None:
        b = np.zeros(out_f, dtype=np.uint16)
    else:
        b = f32_to_bf16_bits(rng.standard_normal(out_f, dtype=np.float32) * np.float32(b_std))
    return w, b


def edge_case_tensor(m: int = 130, k: int = 256, seed: int = 5) -> np.ndarray:
    """Rows exercising the quantizer's corner cases (bf16 bits):

    all-zero blocks, blocks of negative zeros, blocks whose maximum is a bf16
    subnormal, blocks far below the tensor maximum (scale underflows to 0 or
    to E4M3 subnormals), values on E2M1 rounding ties, a block at the tensor
    maximum (scale 448), mixed signs, and a ragged row count (130).
    """
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[0, :16] = 0.0
    x[0, 16:32] = -0.0
    x[1, :16] = np.float32(2.0 ** -130) * np.arange(16, dtype=np.float32)   # bf16 subnormals
    x[1, 16:32] = np.float32(1e-30)
    x[1, 32:48] = np.float32(1e-6) * rng.standard_normal(16).astype(np.float32)
    x[1, 48:64] = np.float32(3e-4) * rng.standard_normal(16).astype(np.float32)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0], dtype=np.float32)
    x[2, :16] = np.concatenate([ties, -ties])
    x[3, :16] = np.float32(1000.0) * np.sign(rng.standard_normal(16)).astype(np.float32)
    x[3, 5] = np.float32(1024.0)                                              # tensor maximum
    x[4, :] = np.float32(0.0)                                                 # whole zero row
    x[5, ::2] *= np.float32(-1.0)
    x[5, 3] = np.float32(0.0)                                                 # zeros inside
    x[6, 17] = np.float32(-0.0)                                               # non-zero blocks
    return f32_to_bf16_bits(x)


def stack_layer_params(layer: int):
    """Weights of layer `layer` (0-based) of the 30-layer stack workloads (15360 and 64800
    tokens): distinct per layer, W ~ N(0, 0.02), bias ~ N(0, 0.01) for both linears.
    Returns (w1, b1, w2, b2) as bf16 bits: w1 [d_ff, d_model], w2 [d_model, d_ff]."""
    w1, b1 = linear_params(D_FF, D_MODEL, seed=300 + 2 * layer, b_std=0.01)
    w2, b2 = linear_params(D_MODEL, D_FF, seed=301 + 2 * layer, b_std=0.01)
    return w1, b1, w2, b2


# Per-rank row counts of the stack workloads on 1/2/4/8 GPUs (contiguous row blocks).
STACK_SHARD_ROWS = {M_STACK: (15360, 7680, 3840, 1920), M_4K: (64800, 32400, 16200, 8100)}
