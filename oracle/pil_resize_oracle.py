"""CPU oracle for the Pillow-exact bicubic resize (TEST INFRASTRUCTURE ONLY).

This module is a test oracle, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` may import it.

The reference resizes 426x240 RGB frames to 1704x960, crops 1664x896 and maps
the bytes to bf16 in [-1, 1] (pil_exact_gpu.py:30-150, used by
chunked_input.py:111-113), reproducing Pillow's ``Image.resize(...,
Image.BICUBIC)`` bit for bit.  That algorithm lives in Pillow (pinned by the
reference at pillow==11.2.1, requirements-runtime.txt:8; 12.2.0 is installed
here), ``libImaging/Resample.c``: ``precompute_coeffs`` (bicubic filter with
a = -0.5, support 2 for upscaling, per output position the taps
``filter(x + xmin - center + 0.5)`` normalised by their sum, all in double),
``normalize_coeffs_8bpc`` (weights to signed 22-bit fixed point, rounded half
away from zero), and the two 8-bit passes -- horizontal first, into a uint8
image, then vertical -- each accumulating ``2^21 + sum(pixel * weight)`` in
int32, shifting right by 22 and clipping to [0, 255].  The normalisation is
the reference's ``(p / 255.0 * 2.0 - 1.0).to(bf16)`` in fp32
(pil_exact_gpu.py:117-121).

Restricted to upscaling (output at least as large as the input in both
dimensions: support 2, at most 4 taps), which is what the reference uses.

Parity status: pinned against Pillow itself (``Image.resize`` on CPU) in the
tests, on seeded random frames of several sizes.
"""
from __future__ import annotations

import numpy as np

PRECISION_BITS = 22


def bicubic(x: float) -> float:
    """Pillow's bicubic_filter, a = -0.5, evaluated in the same order."""
    if x < 0.0:
        x = -x
    if x < 1.0:
        return ((1.5 * x - 2.5) * x * x + 1.0)
    if x < 2.0:
        return (((x - 5.0) * x + 8.0) * x - 4.0) * -0.5
    return 0.0


def coefficients(in_size: int, out_size: int):
    """(first tap index [out], fixed-point weights [out, 4]) for an upscale in_size -> out_size."""
    if out_size < in_size:
        raise ValueError("only upscaling is restated (support 2, at most 4 taps)")
    scale = in_size / out_size
    support = 2.0
    starts = np.zeros(out_size, dtype=np.int64)
    weights = np.zeros((out_size, 4), dtype=np.int64)
    for xx in range(out_size):
        center = (xx + 0.5) * scale
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), in_size) - xmin
        taps = [bicubic(x + xmin - center + 0.5) for x in range(xmax)]
        ww = 0.0
        for w in taps:
            ww += w
        starts[xx] = xmin
        for j, w in enumerate(taps):
            k = w / ww if ww != 0.0 else w
            v = k * (1 << PRECISION_BITS)
            weights[xx, j] = int(-0.5 + v) if k < 0 else int(0.5 + v)
    return starts, weights


def _pass(src: np.ndarray, starts: np.ndarray, weights: np.ndarray, axis: int) -> np.ndarray:
    """One 8-bit pass along `axis` of a uint8 array."""
    n_in = src.shape[axis]
    acc = np.full(np.delete(src.shape, axis).tolist()[:axis] + [len(starts)]
                  + np.delete(src.shape, axis).tolist()[axis:], 1 << (PRECISION_BITS - 1),
                  dtype=np.int64)
    for j in range(4):
        idx = np.minimum(starts + j, n_in - 1)
        taken = np.take(src.astype(np.int64), idx, axis=axis)
        shape = [1] * src.ndim
        shape[axis] = len(starts)
        acc += taken * weights[:, j].reshape(shape)
    return np.clip(acc >> PRECISION_BITS, 0, 255).astype(np.uint8)


def resize(frames: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """uint8 [T, H, W, 3] (or [H, W, 3]) -> uint8 [T, out_h, out_w, 3], Pillow BICUBIC."""
    squeeze = frames.ndim == 3
    f = frames[None] if squeeze else frames
    hs, hw = coefficients(f.shape[2], out_w)
    vs, vw = coefficients(f.shape[1], out_h)
    temp = _pass(f, hs, hw, axis=2)
    out = _pass(temp, vs, vw, axis=1)
    return out[0] if squeeze else out


def normalization_lut() -> np.ndarray:
    """bf16 bits of (p / 255.0 * 2.0 - 1.0) in fp32, p = 0..255."""
    p = np.arange(256, dtype=np.float32)
    v = ((p / np.float32(255.0)).astype(np.float32) * np.float32(2.0)).astype(np.float32)
    v = (v - np.float32(1.0)).astype(np.float32)
    u = v.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def resize_crop_normalize(frames: np.ndarray, out_h: int = 960, out_w: int = 1704,
                          crop=(32, 20, 896, 1664)):
    """(cropped uint8 [T, h, w, 3], bf16 bits [T, 3, h, w]) as the reference pipeline produces."""
    y, x, h, w = crop
    big = resize(frames, out_h, out_w)
    cropped = np.ascontiguousarray(big[:, y:y + h, x:x + w, :])
    planes = normalization_lut()[cropped].transpose(0, 3, 1, 2)
    return cropped, np.ascontiguousarray(planes)
