"""CPU checks of the oracle's building blocks (no GPU)."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O
from flashvsr_optimizations_b200 import workloads as W


def test_e4m3_encode_matches_torch_with_saturation():
    rng = np.random.default_rng(0)
    x = np.abs(rng.standard_normal(100000).astype(np.float32)
               * np.float32(10.0) ** rng.integers(-5, 4, 100000).astype(np.float32))
    x = np.concatenate([x, np.array([0, 448, 449, 463.99, 464, 465, 1e30, 2.0 ** -9, 2.0 ** -10,
                                     1.5 * 2.0 ** -10, 2.0 ** -6], dtype=np.float32)])
    mine = O.f32_to_e4m3(x)
    ref = torch.from_numpy(np.minimum(x, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, ref)


def test_e4m3_decode_matches_torch():
    b = np.arange(256, dtype=np.uint8)
    mine = O.e4m3_to_f32(b)
    ref = torch.from_numpy(b).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(mine[ok], ref[ok])


def test_e2m1_round_to_nearest_even_and_saturation():
    v = np.array([0, 0.24, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.01, 6, 7, 1e9,
                  -0.1, -0.25, -5.0, np.inf, -np.inf], dtype=np.float32)
    want = [0, 0, 0, 1, 2, 2, 4, 4, 6, 6, 7, 7, 7, 7, 8, 8, 14, 7, 15]
    assert O.f32_to_e2m1(v).tolist() == want


def test_e2m1_values_round_trip():
    codes = np.arange(16, dtype=np.uint8)
    assert np.array_equal(O.f32_to_e2m1(O.E2M1_VALUES), codes)


def test_swizzle_offsets_are_a_permutation():
    rows, cols = 256, 96
    off = O.sf_swizzled_offsets(rows, cols)
    assert np.array_equal(np.sort(off.ravel()), np.arange(rows * cols))
    # the 512-byte atom: (row % 32) * 16 + (row % 128 // 32) * 4 + col % 4
    assert off[0, 0] == 0 and off[1, 0] == 16 and off[32, 0] == 4 and off[0, 1] == 1
    assert off[0, 4] == 512 and off[128, 0] == (cols // 4) * 512


def test_global_scale_is_reciprocal_times_2688():
    x = W.gaussian(64, 64, seed=0)
    amax = O.amax_f32(x)
    t = torch.tensor([amax], dtype=torch.float32)
    assert O.global_scale(x) == (2688. / t.clamp_min(1e-12)).item()
    assert O.global_scale_from_amax(0.0) == np.float32(np.float32(1.0) / np.float32(1e-12)) * np.float32(2688)


def test_quantize_dequantize_error_bound():
    """|x - deq/g| <= half an E2M1 step of the block scale (plus the scale's own rounding)."""
    xb = W.gaussian(128, 256, seed=1)
    g = O.global_scale(xb)
    q, s = O.nvfp4_quantize(xb, g)
    deq = O.dequantize(q, s, 128, 256) / g
    x = O.bf16_bits_to_f32(xb)
    blk = np.abs(x.reshape(128, 16, 16)).max(axis=2, keepdims=True)
    err = np.abs(x.reshape(128, 16, 16) - deq.reshape(128, 16, 16))
    assert np.all(err <= blk * (1.0 / 6.0) * 1.2 + 1e-12)


def test_padded_scale_rows_are_zero():
    xb = W.gaussian(130, 128, seed=2)
    _, s = O.nvfp4_quantize(xb, O.global_scale(xb))
    assert s.size == 256 * 8
    off = O.sf_swizzled_offsets(256, 8)
    assert not s[off[130:].ravel()].any()
    assert s[off[:130].ravel()].all()


def test_rcp_table_overrides():
    g = np.float32(3.0)
    key = int(np.array([g]).view(np.uint32)[0])
    fake = int(np.array([np.float32(0.25)]).view(np.uint32)[0])
    assert O.rcp_approx(g, {key: fake}) == np.float32(0.25)
    assert O.rcp_approx(np.float32(0.0)) == np.inf


@pytest.mark.parametrize("gen", [W.gaussian, W.student_t, W.with_outliers])
def test_generators_are_deterministic(gen):
    assert np.array_equal(gen(8, 64, seed=3), gen(8, 64, seed=3))
