"""Drop-in for the reference's ``pil_exact_gpu.py``: Pillow-exact bicubic resize
of the input pipeline on the GPU (pil_exact_gpu.py:30-150; the caller is
chunked_input.py:111-113, ``normalize_exact_gpu(resize_exact_gpu(small))``).

* ``resize_exact_gpu(frames)``: uint8 [T, 240, 426, 3] (any device) -> uint8
  [T, 896, 1664, 3] on CUDA: Pillow's ``resize((1704, 960), BICUBIC)`` cropped
  to (20, 32, 1684, 928), bit for bit.  The reference returns a strided view of
  the uncropped image; this returns the same values contiguous.
* ``normalize_exact_gpu(cropped)``: uint8 [T, 896, 1664, 3] on CUDA (any
  strides with adjacent channels) -> bf16 [T, 3, 896, 1664] of
  ``p / 255 * 2 - 1`` evaluated in fp32.
* ``resize_normalize_exact_gpu(frames)``: both in one kernel pass, without the
  uint8 intermediate in HBM; equal to ``normalize_exact_gpu(resize_exact_gpu(frames))``.
* ``pil_bicubic_resize(frames, out_h, out_w, crop, u8, bf16)``: the general form
  (any upscale, any crop whose width is a multiple of 8).

Shape errors raise ``ValueError`` with the reference's messages; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["resize_exact_gpu", "normalize_exact_gpu", "resize_normalize_exact_gpu",
           "pil_bicubic_resize"]

IN_H, IN_W = 240, 426
OUT_H, OUT_W = 960, 1704
CROP = (32, 20, 896, 1664)          # y, x, h, w: out[:, 32:928, 20:1684]
_MAX_FRAMES = 65535                 # frames per launch


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def pil_bicubic_resize(frames: torch.Tensor, out_h: int, out_w: int,
                       crop: tuple[int, int, int, int] | None = None, u8: bool = True,
                       bf16: bool = False):
    """uint8 [T, H, W, 3] -> (uint8 [T, h, w, 3] or None, bf16 [T, 3, h, w] or None)."""
    if frames.dim() != 4 or frames.shape[-1] != 3 or frames.dtype != torch.uint8:
        raise ValueError("Expected [T,H,W,3] uint8 input")
    if not (u8 or bf16):
        raise ValueError("pil_bicubic_resize: request at least one output")
    if frames.device.type != "cuda":
        frames = frames.to("cuda")
    frames = frames.contiguous()
    t, in_h, in_w, _ = frames.shape
    cy, cx, ch, cw = crop if crop is not None else (0, 0, out_h, out_w)
    dev = frames.device
    out8 = torch.empty((t, ch, cw, 3), dtype=torch.uint8, device=dev) if u8 else None
    outb = torch.empty((t, 3, ch, cw), dtype=torch.bfloat16, device=dev) if bf16 else None
    for f0 in range(0, t, _MAX_FRAMES):
        n = min(_MAX_FRAMES, t - f0)
        _lib.call("fvq_pil_resize", frames[f0:f0 + n].data_ptr(), n, in_h, in_w, out_h, out_w,
                  cy, cx, ch, cw, None if out8 is None else out8[f0:f0 + n].data_ptr(),
                  None if outb is None else outb[f0:f0 + n].data_ptr(), _stream(frames))
    return out8, outb


def resize_exact_gpu(frames: torch.Tensor) -> torch.Tensor:
    """pil_exact_gpu.py:95-112: cropped RGB uint8 frames [T, 896, 1664, 3] on CUDA."""
    if frames.ndim != 4 or tuple(frames.shape[1:]) != (IN_H, IN_W, 3) or frames.dtype != torch.uint8:
        raise ValueError("Expected [T,240,426,3] uint8 input")
    out, _ = pil_bicubic_resize(frames, OUT_H, OUT_W, CROP, u8=True, bf16=False)
    return out


def normalize_exact_gpu(cropped: torch.Tensor) -> torch.Tensor:
    """pil_exact_gpu.py:137-150: [T, 3, 896, 1664] bf16 of p / 255 * 2 - 1."""
    if cropped.ndim != 4 or tuple(cropped.shape[1:]) != (CROP[2], CROP[3], 3) or \
            cropped.dtype != torch.uint8:
        raise ValueError("Expected [T,896,1664,3] uint8 input")
    if cropped.device.type != "cuda":
        raise ValueError("Input must be on CUDA")
    if cropped.stride(3) != 1:
        cropped = cropped.contiguous()
    t = cropped.shape[0]
    out = torch.empty((t, 3, CROP[2], CROP[3]), dtype=torch.bfloat16, device=cropped.device)
    if t:
        _lib.call("fvq_pil_normalize", cropped.data_ptr(), t, CROP[2], CROP[3], cropped.stride(0),
                  cropped.stride(1), cropped.stride(2), out.data_ptr(), _stream(cropped))
    return out


def resize_normalize_exact_gpu(frames: torch.Tensor) -> torch.Tensor:
    """normalize_exact_gpu(resize_exact_gpu(frames)) in one pass: bf16 [T, 3, 896, 1664]."""
    if frames.ndim != 4 or tuple(frames.shape[1:]) != (IN_H, IN_W, 3) or frames.dtype != torch.uint8:
        raise ValueError("Expected [T,240,426,3] uint8 input")
    _, out = pil_bicubic_resize(frames, OUT_H, OUT_W, CROP, u8=False, bf16=True)
    return out
