"""Pin the CPU oracle against the reference's outputs (golden fixtures, no GPU).

The fixtures were produced by FlashInfer's quantizer and mm_fp4 -- the
kernels the reference calls -- on a B200 (tests/golden/make_golden.py), with
the GPU's rcp.approx results for every reciprocal argument each case needs.
With those, the oracle must reproduce codes, scale factors and global scales
bit for bit; GEMM/FFN outputs agree within fp32-accumulation rounding.
"""
import hashlib

import numpy as np
import pytest

from flashvsr_optimizations_b200 import workloads as W
from helpers import f32_from_bits, golden, golden_meta, table_from
from oracle import nvfp4_oracle as O

GEN = {"gaussian": W.gaussian, "with_outliers": W.with_outliers, "student_t": W.student_t,
       "edge_case_tensor": W.edge_case_tensor}


def _regen(c):
    return GEN[c["generator"]](**{k: c[k] for k in ("m", "k", "seed")})


@pytest.mark.parametrize("name", ["q_gauss_128x1536", "q_gauss_200x192", "q_outlier_16x8960",
                                  "q_studentt_64x1536", "q_edge_130x256",
                                  "q_edge_130x256_g1e6", "q_edge_130x256_g1e-3"])
def test_oracle_quantizer_bit_exact(name):
    c = golden_meta()["cases"][name]
    fix = golden(name)
    xb = _regen(c)
    g = np.float32(c["g"]) if "g" in c else O.global_scale(xb)
    assert np.array_equal(np.array([g], dtype=np.float32).view(np.uint32), fix["g_bits"])
    q, s = O.nvfp4_quantize(xb, g, rcp_table=table_from(fix["rcp_args"], fix["rcp_res"]))
    assert np.array_equal(q, fix["codes"]), f"{(q != fix['codes']).sum()} code bytes differ"
    assert np.array_equal(s, fix["sf"]), f"{(s != fix['sf']).sum()} scale bytes differ"


def test_oracle_without_gpu_reciprocals_is_nearly_exact():
    """IEEE 1/x instead of the measured rcp.approx changes at most a handful of codes."""
    name = "q_studentt_64x1536"
    c = golden_meta()["cases"][name]
    fix = golden(name)
    xb = _regen(c)
    q, s = O.nvfp4_quantize(xb, O.global_scale(xb))
    assert np.mean(q != fix["codes"]) < 1e-3
    assert np.mean(s != fix["sf"]) < 1e-3


@pytest.mark.parametrize("name", ["h_outlier_1024x1536", "h_outlier_1024x8960", "h_gauss_4096x1536"])
def test_oracle_quantizer_digests(name):
    c = golden_meta()["cases"][name]
    fix = golden(name)
    xb = _regen(c)
    g = O.global_scale(xb)
    assert np.array_equal(np.array([g], dtype=np.float32).view(np.uint32), fix["g_bits"])
    q, s = O.nvfp4_quantize(xb, g, rcp_table=table_from(fix["rcp_args"], fix["rcp_res"]))
    assert hashlib.sha256(q.tobytes()).hexdigest() == c["codes_sha256"]
    assert hashlib.sha256(s.reshape(-1, c["k"] // 16).tobytes()).hexdigest() == c["sf_sha256"]


def test_oracle_quant_linear_matches_reference():
    c = golden_meta()["cases"]["lin_200x1536x256"]
    fix = golden("lin_200x1536x256")
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    xb = W.gaussian(200, 1536, seed=31)
    lin = O.OracleQuantLinear(wb, bb)
    assert np.array([lin.global_sf], dtype=np.float32).view(np.uint32)[0] == fix["gw_bits"][0]
    assert hashlib.sha256(lin.qweight.tobytes()).hexdigest() == c["qweight_sha256"]
    y = lin.forward_bits(xb)
    ref = O.bf16_bits_to_f32(fix["y"])
    assert O.frobenius_rel(y, ref) <= 2e-3
    assert np.mean(O.f32_to_bf16_bits(y) == fix["y"]) >= 0.95


def test_oracle_ffn_matches_reference():
    """One FFN layer at 64 tokens: Frobenius-relative <= 5e-3 (the path's tolerance)."""
    c = golden_meta()["cases"]["ffn_64"]
    fix = golden("ffn_64")
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    l1, l2 = O.OracleQuantLinear(w1, b1), O.OracleQuantLinear(w2, b2)
    assert np.array([l1.global_sf], dtype=np.float32).view(np.uint32)[0] == c["global_sf1_bits"]
    assert np.array([l2.global_sf], dtype=np.float32).view(np.uint32)[0] == c["global_sf2_bits"]
    assert hashlib.sha256(l1.qweight.tobytes()).hexdigest() == c["qweight1_sha256"]
    assert hashlib.sha256(l2.scale.reshape(-1, W.D_FF // 16).tobytes()).hexdigest() == c["scale2_sha256"]
    xb = W.student_t(64, W.D_MODEL, seed=1)
    y, h = O.ffn_forward(xb, l1, l2, return_intermediate=True)
    assert O.global_scale(xb) == f32_from_bits(fix["g1_bits"])
    assert O.frobenius_rel(h, O.bf16_bits_to_f32(fix["h"])) <= 2e-3
    assert O.frobenius_rel(y, O.bf16_bits_to_f32(fix["y"])) <= 5e-3
