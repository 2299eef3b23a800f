"""The FP8 oracle on CPU: pinned against the reference's golden vectors (codes and
scales of its Triton quantizers and outputs of torch._scaled_mm run on a B200),
plus unit checks of its arithmetic that need no fixture."""
import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN
from flashvsr_optimizations_b200 import workloads as W
from helpers import golden
from oracle import fp8_oracle as F
from oracle import nvfp4_oracle as O

GEMM_TOL = 2e-3
FFN_TOL = 5e-3


def _meta() -> dict:
    p = GOLDEN / "golden_fp8_meta.json"
    if not p.exists():
        pytest.skip("FP8 golden fixtures not generated yet (tests/golden/make_golden_fp8.py on a B200)")
    return json.loads(p.read_text())["cases"]


def _table(fix) -> F.DivTable:
    return F.DivTable(fix["div_a"], fix["div_b"], fix["div_q"])


ROW_CASES = {
    "f8_row_gauss_128x1536": (W.gaussian, dict(m=128, k=1536, seed=10)),
    "f8_row_studentt_64x8960": (W.student_t, dict(m=64, k=8960, seed=12)),
    "f8_row_outlier_16x8960": (W.with_outliers, dict(m=16, k=8960, seed=2)),
    "f8_row_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
    "f8_row_weight_256x1536": (lambda m, k, seed: W.linear_params(m, k, seed=seed)[0],
                               dict(m=256, k=1536, seed=30)),
}


@pytest.mark.parametrize("name", sorted(ROW_CASES))
def test_row_quant_oracle_matches_reference(name):
    gen, kw = ROW_CASES[name]
    fix = golden(name)
    xb = gen(**kw)
    q, s = F.row_quant(xb, _table(fix))
    assert np.array_equal(s.view(np.uint32), fix["s_bits"])
    assert np.array_equal(q, fix["q"].reshape(q.shape))


@pytest.mark.parametrize("name,gen,kw", [
    ("f8_hrow_outlier_1024x8960", W.with_outliers, dict(m=1024, k=8960, seed=2)),
    ("f8_hrow_gauss_4096x1536", W.gaussian, dict(m=4096, k=1536, seed=13)),
])
def test_row_quant_oracle_digests(name, gen, kw):
    meta = _meta()[name]
    q, s = F.row_quant(gen(**kw), _table(golden(name)))
    assert hashlib.sha256(q.tobytes()).hexdigest() == meta["q_sha256"]
    assert hashlib.sha256(s.reshape(-1, 1).tobytes()).hexdigest() == meta["s_sha256"]


TENSOR_CASES = {
    "f8_tensor_gauss_2x64x24x40": (W.gaussian, dict(m=2 * 24 * 40, k=64, seed=40)),
    "f8_tensor_outlier_3x48x20x36": (W.with_outliers, dict(m=3 * 20 * 36, k=48, seed=41)),
    "f8_tensor_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
}


@pytest.mark.parametrize("name", sorted(TENSOR_CASES))
def test_tensor_quant_oracle_matches_reference(name):
    gen, kw = TENSOR_CASES[name]
    fix = golden(name)
    q, s = F.quantize_activation(gen(**kw), _table(fix))
    assert np.float32(s).view(np.uint32) == fix["scale_bits"][0]
    assert np.array_equal(q.reshape(-1), fix["q"].reshape(-1))


def test_linear_oracle_matches_reference_scaled_mm():
    fix = golden("f8_lin_200x1536x256")
    meta = _meta()["f8_lin_200x1536x256"]
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    lin = F.OracleFp8Linear(wb, bb, div=_table(fix))
    assert np.array_equal(lin.scale.view(np.uint32), fix["sw_bits"])
    assert hashlib.sha256(lin.qweight.tobytes()).hexdigest() == meta["qweight_sha256"]
    y = lin.forward_bits(W.gaussian(200, 1536, seed=31), div=_table(fix))
    want = O.bf16_bits_to_f32(fix["y"])
    assert O.frobenius_rel(y, want) <= GEMM_TOL
    assert float(np.mean(y == want)) >= 0.95


def test_ffn_oracle_matches_reference():
    fix = golden("f8_ffn_64")
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    div = _table(fix)
    l1, l2 = F.OracleFp8Linear(w1, b1, div), F.OracleFp8Linear(w2, b2, div)
    meta = _meta()["f8_ffn_64"]
    assert hashlib.sha256(l1.qweight.tobytes()).hexdigest() == meta["qweight1_sha256"]
    assert hashlib.sha256(l2.scale.reshape(-1, 1).tobytes()).hexdigest() == meta["scale2_sha256"]
    y, h = F.ffn_forward(W.student_t(64, W.D_MODEL, seed=1), l1, l2, div,
                         return_intermediate=True)
    assert O.frobenius_rel(h, O.bf16_bits_to_f32(fix["h"])) <= GEMM_TOL
    assert O.frobenius_rel(y, O.bf16_bits_to_f32(fix["y"])) <= FFN_TOL


# ---------------------------------------------------------------- no fixtures needed
def test_div_table_overrides_only_listed_pairs():
    a = np.array([1.0, 2.0, 3.0, 3.0], np.float32)
    b = np.array([3.0, 3.0, 7.0, 3.0], np.float32)
    want = (a / b).astype(np.float32)
    forced = np.array([want[2].view(np.uint32) + 1], np.uint32)
    t = F.DivTable(a[2:3].view(np.uint32), b[2:3].view(np.uint32), forced)
    got = F.div_f32(a, b, t)
    assert got[2].view(np.uint32) == forced[0]
    assert np.array_equal(np.delete(got, 2), np.delete(want, 2))
    merged = F.merge_tables(t, F.DivTable())
    assert len(merged) == 1 and np.array_equal(F.div_f32(a, b, merged), got)


def test_row_scales_floor_and_zero_rows():
    xb = W.edge_case_tensor(130, 256, seed=5)
    q, s = F.row_quant(xb)
    assert s[4] == np.float32(1e-12) and not q[4].any()       # the all-zero row
    assert np.all(s >= np.float32(1e-12))
    # each row's largest magnitude maps to the top of the E4M3 range (448)
    top = np.abs(O.e4m3_to_f32(q)).max(axis=1)[s > np.float32(1e-12)]
    assert np.all(top == 448)


def test_quantize_activation_clamps_to_448():
    xb = O.f32_to_bf16_bits(np.array([[1.0, -2.0, 3.0, 0.0, -0.0, 1e-30]], np.float32))
    q, s = F.quantize_activation(xb)
    # torch's tensor / 448. multiplies by the fp32 reciprocal (here 1 ulp above 3 / 448)
    assert s == np.float32(np.float32(3.0) * (np.float32(1.0) / np.float32(448.0)))
    vals = O.e4m3_to_f32(q)
    assert vals.max() == 448 and np.all(np.abs(vals) <= 448)
    assert q[0, 4] == 0x80 and q[0, 3] == 0x00       # signed zeros kept


def test_scaled_mm_is_exact_for_small_integers():
    qa = O.f32_to_e4m3(np.array([[1, 2, 3, 4]], np.float32))
    qw = O.f32_to_e4m3(np.array([[1, 1, 1, 1], [2, 0, 0, 0]], np.float32))
    y = F.scaled_mm(qa, np.array([0.5], np.float32), qw, np.array([2.0, 4.0], np.float32))
    assert np.array_equal(y, np.array([[10.0, 4.0]], np.float32))
