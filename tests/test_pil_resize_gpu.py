"""Pillow-exact resize on the GPU (reference pil_exact_gpu.py): bit-exact against
Pillow's Image.resize(..., BICUBIC) run on the host, and the bf16 normalisation
bit-exact against the reference's fp32 formula."""
import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import ops, pil_exact as P
from oracle import pil_resize_oracle as R

pytestmark = pytest.mark.gpu
Image = pytest.importorskip("PIL.Image")


def _pillow(frames: np.ndarray, oh: int, ow: int) -> np.ndarray:
    return np.stack([np.asarray(Image.fromarray(f).resize((ow, oh), Image.BICUBIC)) for f in frames])


def _frames(t, h, w, seed, smooth=False):
    rng = np.random.default_rng(seed)
    if not smooth:
        return rng.integers(0, 256, (t, h, w, 3), dtype=np.uint8)
    yy, xx = np.meshgrid(np.linspace(0, 1, h), np.linspace(0, 1, w), indexing="ij")
    base = np.stack([yy, xx, (yy + xx) / 2], axis=-1)[None] * 255
    noise = rng.normal(0, 12, (t, h, w, 3))
    return np.clip(base + noise, 0, 255).astype(np.uint8)


@pytest.mark.parametrize("smooth", [False, True])
def test_resize_exact_gpu_equals_pillow(smooth):
    frames = _frames(5, 240, 426, seed=1, smooth=smooth)
    got = P.resize_exact_gpu(torch.from_numpy(frames))
    want = _pillow(frames, 960, 1704)[:, 32:928, 20:1684]
    assert got.shape == (5, 896, 1664, 3) and got.is_cuda
    assert np.array_equal(got.cpu().numpy(), want)


def test_fused_normalisation_equals_reference_formula():
    frames = _frames(3, 240, 426, seed=2, smooth=True)
    cropped = P.resize_exact_gpu(torch.from_numpy(frames))
    fused = P.resize_normalize_exact_gpu(torch.from_numpy(frames))
    lut = (torch.arange(256, dtype=torch.float32) / 255.0 * 2.0 - 1.0).to(torch.bfloat16)
    want = lut[cropped.cpu().long()].permute(0, 3, 1, 2).contiguous()
    assert fused.dtype == torch.bfloat16 and fused.shape == (3, 3, 896, 1664)
    assert torch.equal(fused.cpu(), want)
    assert torch.equal(P.normalize_exact_gpu(cropped), fused)


def test_normalize_accepts_the_references_strided_view():
    frames = _frames(2, 240, 426, seed=3)
    full, _ = P.pil_bicubic_resize(torch.from_numpy(frames), 960, 1704)   # uncropped
    view = full[:, 32:928, 20:1684, :]                                    # as the reference returns
    assert not view.is_contiguous()
    assert torch.equal(P.normalize_exact_gpu(view), P.normalize_exact_gpu(view.contiguous()))
    assert torch.equal(view.contiguous(), P.resize_exact_gpu(torch.from_numpy(frames)))


@pytest.mark.parametrize("h,w,oh,ow,crop", [
    (7, 5, 29, 32, (0, 0, 29, 32)),
    (33, 50, 100, 208, (3, 8, 90, 192)),
    (16, 16, 16, 16, (0, 0, 16, 16)),
    (240, 426, 480, 852, (0, 2, 480, 848)),
    (135, 240, 540, 2048, (10, 0, 500, 2048)),
    (240, 426, 960, 1704, (0, 0, 960, 1704)),
    (20, 30, 41, 72, (1, 0, 40, 72)),
    (1, 1, 4, 16, (0, 0, 4, 16)),
])
def test_general_geometry_equals_pillow(h, w, oh, ow, crop):
    frames = _frames(3, h, w, seed=h + w)
    y, x, ch, cw = crop
    got, gotb = P.pil_bicubic_resize(torch.from_numpy(frames), oh, ow, crop, u8=True, bf16=True)
    want = _pillow(frames, oh, ow)[:, y:y + ch, x:x + cw]
    assert np.array_equal(got.cpu().numpy(), want)
    assert np.array_equal(gotb.cpu().view(torch.int16).numpy().view(np.uint16),
                          R.normalization_lut()[want].transpose(0, 3, 1, 2))


def test_unaligned_source_frames():
    """The input rows are staged with 16-byte loads; a source starting at an odd
    address exercises the unaligned head and tail."""
    frames = _frames(3, 240, 426, seed=4)
    flat = torch.empty(frames.size + 7, dtype=torch.uint8, device="cuda")
    src = flat[7:].view(3, 240, 426, 3)
    src.copy_(torch.from_numpy(frames))
    assert src.data_ptr() % 16 != 0
    got, _ = P.pil_bicubic_resize(src, 960, 1704, P.CROP)
    assert np.array_equal(got.cpu().numpy(), _pillow(frames, 960, 1704)[:, 32:928, 20:1684])
    assert ops.read_device_error() == 0


def test_shape_errors_match_the_reference():
    with pytest.raises(ValueError):
        P.resize_exact_gpu(torch.zeros(2, 240, 427, 3, dtype=torch.uint8))
    with pytest.raises(ValueError):
        P.resize_exact_gpu(torch.zeros(2, 240, 426, 3, dtype=torch.float32))
    with pytest.raises(ValueError):
        P.normalize_exact_gpu(torch.zeros(1, 896, 1664, 3, dtype=torch.uint8))  # CPU tensor
    assert P.resize_exact_gpu(torch.zeros(0, 240, 426, 3, dtype=torch.uint8)).shape == (0, 896, 1664, 3)
