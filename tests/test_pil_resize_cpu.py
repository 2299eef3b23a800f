"""The Pillow-exact resize oracle on CPU, pinned against Pillow itself, and the
library's argument checks for the resize entry points (no GPU needed)."""
import ctypes

import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import _lib
from oracle import pil_resize_oracle as R

Image = pytest.importorskip("PIL.Image")


@pytest.mark.parametrize("h,w,oh,ow", [(240, 426, 960, 1704), (7, 5, 29, 13), (16, 16, 16, 16),
                                       (33, 50, 100, 208), (240, 426, 480, 852), (1, 1, 4, 4)])
def test_oracle_equals_pillow_bicubic(h, w, oh, ow):
    rng = np.random.default_rng(h * 1000 + w)
    frames = rng.integers(0, 256, (2, h, w, 3), dtype=np.uint8)
    want = np.stack([np.asarray(Image.fromarray(f).resize((ow, oh), Image.BICUBIC)) for f in frames])
    assert np.array_equal(R.resize(frames, oh, ow), want)


def test_oracle_normalization_table_equals_torch():
    lut = (torch.arange(256, dtype=torch.float32) / 255.0 * 2.0 - 1.0).to(torch.bfloat16)
    assert np.array_equal(lut.view(torch.int16).numpy().view(np.uint16), R.normalization_lut())


def test_oracle_coefficients_sum_to_one_in_fixed_point():
    starts, w = R.coefficients(426, 1704)
    assert starts.min() == 0 and starts.max() <= 425
    assert np.all(np.abs(w.sum(axis=1) - (1 << 22)) <= 2)


def test_resize_entry_points_check_arguments():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(1 << 16)
    b = (ctypes.addressof(buf) + 15) // 16 * 16
    rz = lambda *a: lib.fvq_pil_resize(*a)  # noqa: E731
    # downscale, crop outside, crop width not a multiple of 16, no output, unaligned output
    assert rz(b, 1, 240, 426, 120, 213, 0, 0, 120, 208, b, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 1, 240, 426, 960, 1704, 900, 0, 96, 1664, b, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 1, 240, 426, 960, 1704, 32, 20, 896, 1660, b, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 1, 240, 426, 960, 1704, 0, 0, 960, 1700, b, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 1, 240, 426, 960, 1704, 32, 20, 896, 1664, None, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 0, 240, 426, 960, 1704, 32, 20, 896, 1664, b, None, None) == _lib.FVQ_EINVAL
    assert rz(b, 1, 240, 426, 960, 1704, 32, 20, 896, 1664, b + 4, None, None) == _lib.FVQ_EALIGN
    nz = lambda *a: lib.fvq_pil_normalize(*a)  # noqa: E731
    assert nz(b, 1, 896, 1660, 896 * 1660 * 3, 1660 * 3, 3, b, None) == _lib.FVQ_EINVAL
    assert nz(b, 1, 896, 1664, 10, 1664 * 3, 3, b, None) == _lib.FVQ_EINVAL
    assert nz(b, 1, 896, 1664, 896 * 1664 * 3, 1664 * 3, 3, b + 2, None) == _lib.FVQ_EALIGN
