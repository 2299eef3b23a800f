"""FP8 (E4M3, W8A8) mode on the GPU: quantizers, scaled GEMM, QuantLinear('fp8') and the FFN.

Bars: the row and tensor quantizers are bit-exact against the reference's
Triton kernels (golden codes and scales from a B200) and against the CPU
oracle given the GPU's measured divisions; the GEMM and FFN outputs are
within Frobenius-relative 5e-3 of the reference (torch._scaled_mm) and of
the oracle, with per-element agreement reported.
"""
import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import FP8FFN, QuantLinear, install_ffn
from helpers import bits_to_dev, dev_to_bits, golden
from oracle import fp8_oracle as F
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

FFN_TOL = 5e-3
GEMM_TOL = 2e-3


def _meta() -> dict:
    p = GOLDEN / "golden_fp8_meta.json"
    if not p.exists():
        pytest.skip("FP8 golden fixtures not generated yet (tests/golden/make_golden_fp8.py on a B200)")
    return json.loads(p.read_text())["cases"]


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(_u8(t).tobytes()).hexdigest()


def _f32_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().cpu().numpy().view(np.uint32).reshape(-1)


def _probe_div(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """div.full.f32 on the GPU: the reference's division, as a divider for the oracle."""
    q = ops.div_full_probe(torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda(),
                           torch.from_numpy(np.ascontiguousarray(b, np.float32)).cuda())
    return q.cpu().numpy()


ROW_CASES = {
    "f8_row_gauss_128x1536": (W.gaussian, dict(m=128, k=1536, seed=10)),
    "f8_row_studentt_64x8960": (W.student_t, dict(m=64, k=8960, seed=12)),
    "f8_row_outlier_16x8960": (W.with_outliers, dict(m=16, k=8960, seed=2)),
    "f8_row_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5)),
    "f8_row_weight_256x1536": (lambda m, k, seed: W.linear_params(m, k, seed=seed)[0],
                               dict(m=256, k=1536, seed=30)),
}


@pytest.mark.parametrize("name", sorted(ROW_CASES))
def test_row_quant_bit_exact_vs_reference(name):
    gen, kw = ROW_CASES[name]
    fix = golden(name)
    q, s = ops.fp8_row_quant(bits_to_dev(gen(**kw)))
    assert np.array_equal(_f32_bits(s), fix["s_bits"]), "row scales differ"
    got = _u8(q)
    assert np.array_equal(got, fix["q"]), f"{int((got != fix['q']).sum())} codes differ"


@pytest.mark.parametrize("name,gen,kw", [
    ("f8_hrow_outlier_1024x8960", W.with_outliers, dict(m=1024, k=8960, seed=2)),
    ("f8_hrow_gauss_4096x1536", W.gaussian, dict(m=4096, k=1536, seed=13)),
])
def test_row_quant_digests_vs_reference(name, gen, kw):
    meta = _meta()[name]
    q, s = ops.fp8_row_quant(bits_to_dev(gen(**kw)))
    assert _sha(q) == meta["q_sha256"] and _sha(s) == meta["s_sha256"]


def test_reference_division_is_div_full():
    """The reference's Triton `/` produced exactly libfvq's div.full.f32 on every operand pair."""
    for name, case in _meta().items():
        if "quotients_differing_from_div_full" in case:
            assert case["quotients_differing_from_div_full"] == 0, name


TENSOR_CASES = {
    "f8_tensor_gauss_2x64x24x40": (W.gaussian, dict(m=2 * 24 * 40, k=64, seed=40), (2, 64, 24, 40)),
    "f8_tensor_outlier_3x48x20x36": (W.with_outliers, dict(m=3 * 20 * 36, k=48, seed=41),
                                     (3, 48, 20, 36)),
    "f8_tensor_edge_130x256": (W.edge_case_tensor, dict(m=130, k=256, seed=5), None),
}


@pytest.mark.parametrize("name", sorted(TENSOR_CASES))
def test_tensor_quant_bit_exact_vs_reference(name):
    gen, kw, nchw = TENSOR_CASES[name]
    fix = golden(name)
    xb = gen(**kw)
    x = bits_to_dev(xb)
    q, scale = ops.fp8_quantize_activation(x)
    assert _f32_bits(scale)[0] == fix["scale_bits"][0]
    assert np.array_equal(_u8(q).reshape(-1), fix["q"].reshape(-1))
    if nchw is not None:
        # the same memory as a channels_last NCHW activation: same codes, same layout
        n, c, h, w = nchw
        x4 = x.reshape(n, h, w, c).permute(0, 3, 1, 2)
        assert x4.is_contiguous(memory_format=torch.channels_last)
        q4, s4 = ops.fp8_quantize_activation(x4)
        assert q4.stride() == x4.stride() and torch.equal(s4, scale)
        assert np.array_equal(_u8(q4.permute(0, 2, 3, 1)).reshape(-1), fix["q"].reshape(-1))


@pytest.mark.parametrize("m,k", [(1, 8), (3, 64), (130, 256), (257, 1536), (9, 8960), (5, 16384),
                                 (40, 4104)])
def test_row_quant_vs_oracle_with_measured_division(m, k):
    xb = W.student_t(m, k, seed=m + k)
    q, s = ops.fp8_row_quant(bits_to_dev(xb))
    oq, os_ = F.row_quant(xb, _probe_div)
    assert np.array_equal(_f32_bits(s), os_.view(np.uint32))
    assert np.array_equal(_u8(q), oq)


def _e4m3_midpoints() -> np.ndarray:
    """Every value halfway between adjacent E4M3 magnitudes (the rounding ties)."""
    mags = np.unique(np.abs(O.e4m3_to_f32(np.arange(0, 0x7F, dtype=np.uint8))))
    return ((mags[1:] + mags[:-1]) / 2).astype(np.float32)


def test_row_quant_ties_and_near_midpoints():
    """Quotients on and next to E4M3 rounding midpoints: the one-multiply path must
    hand these to div.full, and ties must round to even as the reference's do."""
    mids = _e4m3_midpoints()
    rows = []
    # amax 448 -> scale exactly 1 and amax 7 -> scale 2^-6: every quotient is exact,
    # so bf16 midpoints are exact ties
    for amax, scale in ((448.0, 1.0), (7.0, 2.0 ** -6)):
        r = np.zeros(256, np.float32)
        r[0] = amax
        ties = (mids * np.float32(scale)).astype(np.float32)
        ties = ties[O.round_bf16(ties) == ties][:255]
        r[1:1 + ties.size] = ties
        r[1 + ties.size:] = -r[1:256 - ties.size]
        rows.append(r)
    # scales with long mantissas: quotients land within a few ulp of midpoints
    rng = np.random.default_rng(3)
    for amax in (3.0, 5.0, 11.0, 13.0, 0.1, 1e-3, 300.0, 97.0):
        r = rng.standard_normal(256).astype(np.float32) * np.float32(amax / 4)
        r[0] = amax
        rows.append(np.clip(r, -amax, amax))
    xb = O.f32_to_bf16_bits(np.stack(rows))
    q, s = ops.fp8_row_quant(bits_to_dev(xb))
    oq, os_ = F.row_quant(xb, _probe_div)
    assert np.array_equal(_f32_bits(s), os_.view(np.uint32))
    assert np.array_equal(_u8(q), oq)
    # a large random case hits ~3e-5 of its quotients inside the fallback window
    xb = W.student_t(512, 8960, seed=77)
    q, s = ops.fp8_row_quant(bits_to_dev(xb))
    oq, _ = F.row_quant(xb, _probe_div)
    assert np.array_equal(_u8(q), oq)


@pytest.mark.parametrize("numel", [1, 7, 8, 4099, 1 << 20])
def test_tensor_quant_vs_oracle_with_measured_division(numel):
    xb = W.with_outliers(1, numel, seed=numel)
    q, s = ops.fp8_quantize_activation(bits_to_dev(xb).reshape(-1))
    oq, os_ = F.quantize_activation(xb.reshape(-1), _probe_div)
    assert _f32_bits(s)[0] == np.float32(os_).view(np.uint32)
    assert np.array_equal(_u8(q), oq)


def _scaled_ref(qa, sa, qw, sw):
    """torch fp32 reference of the scaled GEMM: bf16((A W^T) * sa * sw)."""
    acc = qa.float() @ qw.float().t()
    return ((acc * sa.reshape(-1, 1)) * sw.reshape(1, -1)).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(1, 256, 128), (127, 256, 256), (300, 512, 1536),
                                   (256, 1536, 8960), (1000, 8960, 1536), (7680, 1536, 8960)])
def test_scaled_mm_vs_torch_fp32(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(torch.bfloat16)
    qa, sa = ops.fp8_row_quant(a)
    qw, sw = ops.fp8_row_quant(w)
    bias = (0.01 * torch.randn(n, device="cuda", generator=g)).to(torch.bfloat16)
    y = ops.fp8_scaled_mm(qa, sa, qw, sw, bias)
    ref = (_scaled_ref(qa, sa, qw, sw) + bias)
    rel = float((y.float() - ref.float()).norm() / ref.float().norm())
    assert rel <= GEMM_TOL, rel
    same = float((y == ref).float().mean())
    assert same >= 0.95, same


def test_scaled_mm_vs_reference_golden():
    """QuantLinear('fp8').forward against torch._scaled_mm + bias on the reference's steps."""
    meta = _meta()["f8_lin_200x1536x256"]
    fix = golden("f8_lin_200x1536x256")
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    lin = torch.nn.Linear(1536, 256, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    ql = QuantLinear(lin, "fp8")
    assert _sha(ql.qweight) == meta["qweight_sha256"] and _sha(ql.scale) == meta["scale_sha256"]
    assert ql.scale.shape == (256, 1) and ql.qweight.dtype == torch.float8_e4m3fn
    y = ql(bits_to_dev(W.gaussian(200, 1536, seed=31)))
    got = O.bf16_bits_to_f32(dev_to_bits(y))
    want = O.bf16_bits_to_f32(fix["y"])
    assert O.frobenius_rel(got, want) <= GEMM_TOL
    assert float(np.mean(got == want)) >= 0.95


def test_scaled_mm_vs_oracle():
    xb = W.gaussian(96, 1536, seed=5)
    wb, _ = W.linear_params(512, 1536, seed=6)
    qa, sa = ops.fp8_row_quant(bits_to_dev(xb))
    qw, sw = ops.fp8_row_quant(bits_to_dev(wb))
    y = ops.fp8_scaled_mm(qa, sa, qw, sw)
    want = F.scaled_mm(_u8(qa), sa.cpu().numpy(), _u8(qw), sw.cpu().numpy())
    got = O.bf16_bits_to_f32(dev_to_bits(y))
    assert O.frobenius_rel(got, want) <= GEMM_TOL
    assert float(np.mean(got == want)) >= 0.95


def _linear(out_f, in_f, wb, bb):
    lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    return lin


@pytest.fixture(scope="module")
def fp8_layer():
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    seq = torch.nn.Sequential(_linear(W.D_FF, W.D_MODEL, w1, b1), torch.nn.GELU(approximate="tanh"),
                              _linear(W.D_MODEL, W.D_FF, w2, b2))
    return FP8FFN(QuantLinear(seq[0], "fp8"), seq[1], QuantLinear(seq[2], "fp8")), (w1, b1, w2, b2)


def test_fp8_weights_match_reference(fp8_layer):
    ffn, _ = fp8_layer
    meta = _meta()["f8_ffn_64"]
    for i, lin in ((1, ffn[0]), (2, ffn[2])):
        assert _sha(lin.qweight) == meta[f"qweight{i}_sha256"]
        assert _sha(lin.scale) == meta[f"scale{i}_sha256"]


def test_fp8_ffn_fused_equals_unfused(fp8_layer):
    """The fused call computes exactly QuantLinear -> GELU -> QuantLinear."""
    ffn, _ = fp8_layer
    x = bits_to_dev(W.student_t(300, W.D_MODEL, seed=9))
    y_fused = ffn(x)
    y_seq = ffn[2](ffn[1](ffn[0](x)))
    assert torch.equal(y_fused, y_seq)


def test_fp8_ffn_vs_reference_golden(fp8_layer):
    ffn, _ = fp8_layer
    fix = golden("f8_ffn_64")
    x = bits_to_dev(W.student_t(64, W.D_MODEL, seed=1))
    h = ffn[1](ffn[0](x))
    rel_h = O.frobenius_rel(O.bf16_bits_to_f32(dev_to_bits(h)), O.bf16_bits_to_f32(fix["h"]))
    assert rel_h <= GEMM_TOL, rel_h
    y = ffn(x)
    got, want = O.bf16_bits_to_f32(dev_to_bits(y)), O.bf16_bits_to_f32(fix["y"])
    assert O.frobenius_rel(got, want) <= FFN_TOL
    fix = golden("f8_ffn_7680_rows")
    meta = _meta()["f8_ffn_7680_rows"]
    y = ffn(bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1)))
    got = O.bf16_bits_to_f32(dev_to_bits(y[torch.from_numpy(fix["rows"]).cuda()]))
    assert O.frobenius_rel(got, O.bf16_bits_to_f32(fix["y_rows"])) <= FFN_TOL
    assert abs(float(y.float().norm()) / meta["y_fro"] - 1) <= FFN_TOL


def test_fp8_ffn_vs_oracle(fp8_layer):
    ffn, (w1, b1, w2, b2) = fp8_layer
    xb = W.student_t(48, W.D_MODEL, seed=3)
    y = ffn(bits_to_dev(xb))
    l1 = F.OracleFp8Linear(w1, b1, _probe_div)
    l2 = F.OracleFp8Linear(w2, b2, _probe_div)
    assert np.array_equal(_u8(ffn[0].qweight), l1.qweight)
    assert np.array_equal(_f32_bits(ffn[2].scale), l2.scale.view(np.uint32))
    want = F.ffn_forward(xb, l1, l2, _probe_div)
    assert O.frobenius_rel(O.bf16_bits_to_f32(dev_to_bits(y)), want) <= FFN_TOL


def test_install_ffn_fp8_mode():
    class Block(torch.nn.Module):
        def __init__(self, seed):
            super().__init__()
            w1, b1 = W.linear_params(1024, 512, seed=seed, b_std=0.01)
            w2, b2 = W.linear_params(512, 1024, seed=seed + 1, b_std=0.01)
            self.ffn = torch.nn.Sequential(_linear(1024, 512, w1, b1),
                                           torch.nn.GELU(approximate="tanh"),
                                           _linear(512, 1024, w2, b2))

    class Pipe:
        def __init__(self):
            self.dit = torch.nn.Module()
            self.dit.blocks = torch.nn.ModuleList([Block(s) for s in (1, 3)])

    pipe = Pipe()
    x = bits_to_dev(W.gaussian(2 * 77, 512, seed=8)).reshape(2, 77, 512)
    meta = install_ffn(pipe, "fp8")
    assert meta["quantized_linears"] == 4 and meta["fused_ffn_blocks"] == 2
    assert meta["ffn_bytes_after"] < meta["ffn_bytes_before"]
    ffn = pipe.dit.blocks[0].ffn
    assert isinstance(ffn, FP8FFN) and ffn[0].mode == "fp8"
    y = ffn(x)
    assert y.shape == x.shape and torch.equal(y, ffn[2](ffn[1](ffn[0](x))))


@pytest.mark.parametrize("m", [1, 129, 300, 384, 1000, 7680])
def test_fp8_sm_pair_and_single_sm_gemms_give_the_same_bits(fp8_layer, m):
    """The SM-pair kernels (256 x 256 tiles, cta_group::2; the default) and the
    one-SM kernels agree bit for bit, including pair tiles over the end of A
    (m = 129: the odd CTA holds one row; m = 384: its rows are all past the end)."""
    from flashvsr_optimizations_b200 import _lib
    ffn, _ = fp8_layer
    lib = _lib.load()
    x = bits_to_dev(W.student_t(m, W.D_MODEL, seed=m))
    l1, l2 = ffn[0], ffn[2]
    outs = []
    try:
        for mode in (2, 1, 0):  # all GEMMs paired, the default split, none
            lib.fvq_set_fp8_gemm_pairing(mode)
            y = ops.fp8_ffn(x, l1.qweight, l1.scale, l1.bias, l2.qweight, l2.scale, l2.bias)
            h = ffn[1](ffn[0](x))
            outs.append((y, h))
    finally:
        lib.fvq_set_fp8_gemm_pairing(1)
    assert ops.read_device_error() == 0
    for y, h in outs[1:]:
        assert torch.equal(outs[0][1], h) and torch.equal(outs[0][0], y)
    assert lib.fvq_set_fp8_gemm_pairing(3) == _lib.FVQ_EINVAL
