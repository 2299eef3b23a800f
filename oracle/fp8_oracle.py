"""CPU oracle for the FP8 (E4M3, W8A8) paths (TEST INFRASTRUCTURE ONLY).

This module is a test oracle, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The CUDA extension never calls into it.

It restates, in numpy, the arithmetic of the reference's FP8 mode:

* ``row_quant``  -- ffn_quantization.py:6-13 (Triton ``_row_quant``) and
  :22-26, applied to weights (:44-45) and activations (:58):

      scale[r] = max(max_k |x[r, k]| / 448, 1e-12)        (fp32)
      q[r, k]  = e4m3_rn_satfinite(x[r, k] / scale[r])

* ``quantize_activation`` -- decoder_fp8.py:9-24 (and lq_fp8.py:24-31, the
  same steps): the amax of ``_partial_amax`` (ffn_quantization.py:15-19),
  ``scale = max(amax / 448, 1e-12)`` computed by torch (IEEE division), then
  ``q = e4m3_rn(min(max(x / scale, -448), 448))``.

* ``scaled_mm`` -- ffn_quantization.py:58-60, ``torch._scaled_mm`` with
  row-wise scales: ``bf16(acc * scale_a[m] * scale_w[n])``; products of E4M3
  values are exact in fp32, the sum is formed in float64 and rounded once
  (the GPU accumulates in fp32 in its own order, so agreement is to within
  accumulation rounding).  Then the bias add (:68-69, a bf16 add that rounds
  twice), GELU-tanh in fp32 rounded to bf16 (the upstream ``ffn[1]``).

The ``/`` in both Triton kernels is Triton's fp32 division, which its NVIDIA
backend emits as ``div.full.f32``: an approximation with at most 2 ulp of
error, whose exact results a CPU cannot derive from documentation.  The
functions here take a divider ``div``: ``None`` divides with IEEE rounding; a
:class:`DivTable` adds quotients measured on a GPU for the (dividend,
divisor) pairs where that instruction's result differs from the IEEE one (the
golden fixtures carry such tables, and with them the oracle is bit-exact); any
other callable ``div(a, b)`` is used as is (on a GPU: the instruction itself,
through libfvq's probe).

torch's ``tensor / 448.`` on a CUDA tensor multiplies by the fp32 reciprocal
of the Python scalar, so the per-tensor scale is ``amax * fl(1/448)`` (two
IEEE roundings), not ``amax / 448``.

Parity status: pinned against the reference's own steps run on a B200 --
its Triton row and tensor quantizers restated step for step in Triton and
``torch._scaled_mm`` (``tests/golden/make_golden_fp8.py``).
"""
from __future__ import annotations

import numpy as np

from .nvfp4_oracle import (F32, bf16_bits_to_f32, bias_add_bf16, e4m3_to_f32, f32_to_bf16_bits,
                           f32_to_e4m3, gelu_tanh_bf16, round_bf16)

E4M3_MAX = F32(448.0)
SCALE_FLOOR = F32(1e-12)       # tl.maximum(..., 1.e-12) and clamp_min(1e-12)


class DivTable:
    """Measured ``div.full.f32`` results for the pairs where they differ from IEEE division.

    Built from three equal-length uint32 arrays: dividend bits, divisor bits and
    quotient bits.  Lookup is vectorised over a combined 64-bit key.
    """

    def __init__(self, a_bits=(), b_bits=(), q_bits=()):
        a = np.asarray(a_bits, dtype=np.uint64)
        b = np.asarray(b_bits, dtype=np.uint64)
        keys = (a << np.uint64(32)) | b
        order = np.argsort(keys, kind="stable")
        self.keys = keys[order]
        self.vals = np.asarray(q_bits, dtype=np.uint32)[order]

    def __len__(self) -> int:
        return int(self.keys.size)

    def __call__(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        return self.apply(a, b, ieee_div(a, b))

    def apply(self, a: np.ndarray, b: np.ndarray, q: np.ndarray) -> np.ndarray:
        if self.keys.size == 0:
            return q
        a_u = np.ascontiguousarray(a, dtype=F32).view(np.uint32).astype(np.uint64)
        b_u = np.ascontiguousarray(np.broadcast_to(b, np.shape(a)), dtype=F32).view(np.uint32)
        keys = (a_u << np.uint64(32)) | b_u.astype(np.uint64)
        pos = np.searchsorted(self.keys, keys)
        pos = np.minimum(pos, self.keys.size - 1)
        hit = self.keys[pos] == keys
        out = np.array(q, dtype=F32, copy=True).view(np.uint32)
        out[hit] = self.vals[pos[hit]]
        return out.view(F32)


def ieee_div(a, b) -> np.ndarray:
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore", under="ignore"):
        return (a / b).astype(F32)


def div_f32(a, b, div=None) -> np.ndarray:
    """fp32 a / b through the divider ``div`` (None: IEEE rounded)."""
    a = np.asarray(a, dtype=F32)
    b = np.broadcast_to(np.asarray(b, dtype=F32), np.broadcast_shapes(np.shape(a), np.shape(b)))
    a = np.broadcast_to(a, b.shape)
    if div is None:
        return ieee_div(a, b)
    return np.asarray(div(np.ascontiguousarray(a), np.ascontiguousarray(b)), dtype=F32).reshape(b.shape)


def row_scales(x_bits: np.ndarray, div=None) -> np.ndarray:
    """max(max_k |x[r]| / 448, 1e-12) per row of a bf16 [M, K] tensor -> fp32 [M]."""
    xf = bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16))
    amax = np.abs(xf).max(axis=1) if xf.shape[1] else np.zeros(xf.shape[0], F32)
    return np.maximum(div_f32(amax.astype(F32), E4M3_MAX, div), SCALE_FLOOR).astype(F32)


def row_quant(x_bits: np.ndarray, div=None):
    """bf16 [M, K] (uint16 bits) -> (E4M3 bytes [M, K], fp32 scales [M])."""
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    s = row_scales(x_bits, div)
    xf = bf16_bits_to_f32(x_bits)
    return f32_to_e4m3(div_f32(xf, s[:, None], div)), s


INV_448 = F32(F32(1.0) / E4M3_MAX)   # torch's reciprocal of the scalar divisor


def tensor_scale(x_bits: np.ndarray) -> F32:
    """``(amax / 448.).clamp_min(1e-12)`` as torch evaluates it: amax * fl(1/448)."""
    a = np.abs(bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16))).max()
    return F32(max(F32(F32(a) * INV_448), SCALE_FLOOR))


def quantize_activation(x_bits: np.ndarray, div=None):
    """Any-shape bf16 tensor (uint16 bits, memory order) -> (E4M3 bytes, fp32 scale)."""
    x_bits = np.asarray(x_bits, dtype=np.uint16)
    s = tensor_scale(x_bits)
    q = div_f32(bf16_bits_to_f32(x_bits), s, div)
    q = np.minimum(np.maximum(q, -E4M3_MAX), E4M3_MAX).astype(F32)
    return f32_to_e4m3(q), s


def scale_division_pairs(x_bits: np.ndarray):
    """(dividends, divisors) of the per-row ``max|x| / 448`` divisions of ``row_quant``."""
    xf = bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16))
    amax = np.abs(xf).max(axis=1).astype(F32)
    return amax, np.full(amax.shape, E4M3_MAX, F32)


def element_division_pairs(x_bits: np.ndarray, scales: np.ndarray):
    """(dividends, divisors) of the per-element ``x / scale[row]`` divisions of ``row_quant``."""
    xf = bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16))
    s = np.asarray(scales, dtype=F32).reshape(-1, 1)
    return xf.ravel().astype(F32), np.broadcast_to(s, xf.shape).ravel().astype(F32)


def merge_tables(*tables: DivTable) -> DivTable:
    keys = np.concatenate([t.keys for t in tables])
    vals = np.concatenate([t.vals for t in tables])
    return DivTable((keys >> np.uint64(32)).astype(np.uint32),
                    (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32), vals)


def scaled_mm(qa: np.ndarray, sa: np.ndarray, qw: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """bf16((A @ W^T) * sa[m] * sw[n]) over E4M3 operands -> float32 holding bf16 values."""
    a = e4m3_to_f32(np.asarray(qa, dtype=np.uint8)).astype(np.float64)
    w = e4m3_to_f32(np.asarray(qw, dtype=np.uint8)).astype(np.float64)
    acc = (a @ w.T).astype(F32)
    sa = np.asarray(sa, dtype=F32).reshape(-1, 1)
    sw = np.asarray(sw, dtype=F32).reshape(1, -1)
    return round_bf16((acc * sa).astype(F32) * sw)


class OracleFp8Linear:
    """Weight-side state of ``QuantLinear(linear, 'fp8')`` (ffn_quantization.py:36-46)."""

    def __init__(self, weight_bits: np.ndarray, bias_bits: np.ndarray | None, div=None):
        weight_bits = np.asarray(weight_bits, dtype=np.uint16)
        self.out_features, self.in_features = weight_bits.shape
        self.qweight, self.scale = row_quant(weight_bits, div)
        self.bias = None if bias_bits is None else np.asarray(bias_bits, dtype=np.uint16)

    def forward_bits(self, x_bits: np.ndarray, div=None, fp32_matmul: bool = False) -> np.ndarray:
        """QuantLinear.forward (ffn_quantization.py:54-60, :68-70) -> float32 of bf16 values.

        ``fp32_matmul=True`` is the CPU-baseline variant: the dequantised weight
        is cached and the product is a float32 BLAS matmul.
        """
        q, s = row_quant(x_bits, div)
        if fp32_matmul:
            if getattr(self, "_w_deq", None) is None:
                self._w_deq = e4m3_to_f32(self.qweight)
            acc = e4m3_to_f32(q) @ self._w_deq.T
            out = round_bf16((acc.astype(F32) * s[:, None]).astype(F32) * self.scale[None, :])
        else:
            out = scaled_mm(q, s, self.qweight, self.scale)
        return bias_add_bf16(out, self.bias)


def ffn_forward(x_bits: np.ndarray, lin1: OracleFp8Linear, lin2: OracleFp8Linear, div=None,
                return_intermediate: bool = False, fp32_matmul: bool = False):
    """QuantLinear('fp8') -> GELU-tanh (bf16) -> QuantLinear('fp8'), as the reference runs it."""
    h = gelu_tanh_bf16(lin1.forward_bits(x_bits, div, fp32_matmul))
    y = lin2.forward_bits(f32_to_bf16_bits(h), div, fp32_matmul)
    if return_intermediate:
        return y, h
    return y
