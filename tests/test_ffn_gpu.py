"""Whole NVFP4 FFN (QuantLinear -> GELU-tanh -> QuantLinear) on the GPU.

Tolerance: Frobenius-relative error <= 5e-3 (the bar this path is held to) against the
reference's own NVFP4 FFN (golden outputs of FlashInfer's kernels on a B200)
and against the CPU oracle.
"""
import hashlib

import numpy as np
import pytest
import torch

import flashvsr_optimizations_b200 as fvq
from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, QuantLinear, install_ffn
from helpers import bits_to_dev, dev_to_bits, f32_from_bits, golden, golden_meta, gpu_rcp_table
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

FFN_TOL = 5e-3


def _linear(out_f, in_f, wb, bb):
    lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    return lin


@pytest.fixture(scope="module")
def ffn_layer():
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    seq = torch.nn.Sequential(_linear(W.D_FF, W.D_MODEL, w1, b1), torch.nn.GELU(approximate="tanh"),
                              _linear(W.D_MODEL, W.D_FF, w2, b2))
    q1 = QuantLinear(seq[0], "nvfp4")
    q2 = QuantLinear(seq[2], "nvfp4")
    return NVFP4FFN(q1, seq[1], q2), (w1, b1, w2, b2)


def test_weight_quantization_matches_reference(ffn_layer):
    ffn, _ = ffn_layer
    meta = golden_meta()["cases"]["ffn_64"]
    for i, lin in ((1, ffn[0]), (2, ffn[2])):
        assert hashlib.sha256(lin.qweight.cpu().numpy().tobytes()).hexdigest() == meta[f"qweight{i}_sha256"]
        assert hashlib.sha256(lin.scale.cpu().numpy().tobytes()).hexdigest() == meta[f"scale{i}_sha256"]
        assert int(lin.global_sf.cpu().numpy().view(np.uint32)[0]) == meta[f"global_sf{i}_bits"]


def test_ffn_small_matches_reference_golden(ffn_layer):
    ffn, _ = ffn_layer
    fix = golden("ffn_64")
    xb = W.student_t(64, W.D_MODEL, seed=1)
    y = ffn(bits_to_dev(xb))
    rel = O.frobenius_rel(O.bf16_bits_to_f32(dev_to_bits(y)), O.bf16_bits_to_f32(fix["y"]))
    assert rel <= FFN_TOL, rel


def test_ffn_bit_identical_to_reference(ffn_layer):
    """Same kernel order and roundings as FlashInfer's mm_fp4 + torch bias/GELU:
    the fused FFN reproduces the reference's bf16 output bit for bit."""
    ffn, _ = ffn_layer
    fix = golden("ffn_64")
    y = ffn(bits_to_dev(W.student_t(64, W.D_MODEL, seed=1)))
    got = dev_to_bits(y)
    assert np.array_equal(got, fix["y"]), f"{int((got != fix['y']).sum())} of {got.size} differ"
    fix = golden("ffn_7680_rows")
    y = ffn(bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1)))
    got = dev_to_bits(y[torch.from_numpy(fix["rows"]).cuda()])
    assert np.array_equal(got, fix["y_rows"]), f"{int((got != fix['y_rows']).sum())} differ"


def test_ffn_fused_equals_unfused_modules(ffn_layer):
    """The fused call computes exactly what QuantLinear -> GELU -> QuantLinear computes."""
    ffn, _ = ffn_layer
    x = bits_to_dev(W.student_t(300, W.D_MODEL, seed=9))
    y_fused = ffn(x)
    h = ffn[0](x)
    h = torch.nn.functional.gelu(h, approximate="tanh")
    y_mod = ffn[2](h)
    rel = O.frobenius_rel(y_fused.float().cpu().numpy(), y_mod.float().cpu().numpy())
    assert rel <= 1e-3, rel


def test_ffn_one_layer_7680_matches_reference_rows(ffn_layer):
    ffn, _ = ffn_layer
    fix = golden("ffn_7680_rows")
    meta = golden_meta()["cases"]["ffn_7680_rows"]
    xb = W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1)
    y = ffn(bits_to_dev(xb))
    rows = torch.from_numpy(fix["rows"]).cuda()
    got = O.bf16_bits_to_f32(dev_to_bits(y[rows]))
    rel = O.frobenius_rel(got, O.bf16_bits_to_f32(fix["y_rows"]))
    assert rel <= FFN_TOL, rel
    fro = float(y.float().norm().item())
    assert abs(fro - meta["y_fro"]) / meta["y_fro"] <= FFN_TOL


@pytest.mark.parametrize("m,seed", [(64, 1), (130, 5), (300, 9)])
def test_ffn_matches_oracle(ffn_layer, m, seed):
    """Oracle with this GPU's measured reciprocals: agreement to accumulation rounding."""
    ffn, (w1, b1, w2, b2) = ffn_layer
    l1 = O.OracleQuantLinear(w1, b1, gpu_rcp_table)
    l2 = O.OracleQuantLinear(w2, b2, gpu_rcp_table)
    xb = W.student_t(m, W.D_MODEL, seed=seed)
    y_ref = O.ffn_forward(xb, l1, l2, rcp_provider=gpu_rcp_table)
    y = ffn(bits_to_dev(xb))
    rel = O.frobenius_rel(O.bf16_bits_to_f32(dev_to_bits(y)), y_ref)
    assert rel <= FFN_TOL, (m, rel)


def test_ffn_3d_input_and_repeatability(ffn_layer):
    ffn, _ = ffn_layer
    x = bits_to_dev(W.gaussian(2 * 100, W.D_MODEL, seed=4)).reshape(2, 100, W.D_MODEL)
    y1 = ffn(x)
    y2 = ffn(x)
    assert y1.shape == (2, 100, W.D_MODEL)
    assert torch.equal(y1, y2)


class _Block(torch.nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.ffn = torch.nn.Sequential(torch.nn.Linear(d, f), torch.nn.GELU(approximate="tanh"),
                                       torch.nn.Linear(f, d))


class _Dit(torch.nn.Module):
    def __init__(self, n, d, f):
        super().__init__()
        self.blocks = torch.nn.ModuleList([_Block(d, f) for _ in range(n)])


class _Pipe:
    def __init__(self, n=30, d=256, f=512):
        self.dit = _Dit(n, d, f).cuda().to(torch.bfloat16)


def test_install_ffn_counts_and_matches_quantlinear():
    torch.manual_seed(0)
    pipe = _Pipe()
    ref_pipe = _Pipe()
    ref_pipe.dit.load_state_dict(pipe.dit.state_dict())
    with torch.no_grad():
        meta = install_ffn(pipe, "nvfp4")
        meta_unfused = install_ffn(ref_pipe, "nvfp4", fused=False)
    assert meta["quantized_linears"] == 60 and meta_unfused["quantized_linears"] == 60
    assert meta["fused_ffn_blocks"] == 30
    assert meta["ffn_bytes_after"] < meta["ffn_bytes_before"]
    assert isinstance(pipe.dit.blocks[0].ffn, NVFP4FFN)
    assert isinstance(pipe.dit.blocks[0].ffn[0], QuantLinear)
    x = torch.randn(4, 64, 256, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        for b_fused, b_ref in zip(pipe.dit.blocks, ref_pipe.dit.blocks):
            y_f = b_fused.ffn(x)
            y_r = b_ref.ffn(x)
            rel = O.frobenius_rel(y_f.float().cpu().numpy(), y_r.float().cpu().numpy())
            assert rel <= 1e-3
            x = y_f


def test_no_silent_fallback_on_cpu_tensors():
    with pytest.raises(RuntimeError):
        ops.global_scale(torch.zeros(16, 64, dtype=torch.bfloat16))


def test_shape_errors_raise():
    x = torch.zeros(16, 100, dtype=torch.bfloat16, device="cuda")
    g = torch.ones(1, device="cuda")
    with pytest.raises(fvq.FvqError) as e:
        ops.nvfp4_quantize(x, g)
    assert e.value.code == -1


def test_ffn_profile_entry_point_same_output_and_times(ffn_layer):
    """fvq_nvfp4_ffn_profile runs fvq_nvfp4_ffn's launches with events around them:
    the same output bits, and four positive device times."""
    import ctypes
    from flashvsr_optimizations_b200 import _lib
    ffn, _ = ffn_layer
    q1, q2 = ffn[0], ffn[2]
    x = bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=5))
    ref = ffn(x)
    lib = _lib.load()
    m, d, f = W.M_ONE_LAYER, W.D_MODEL, W.D_FF
    ws = torch.zeros(lib.fvq_nvfp4_ffn_workspace_bytes(m, d, f), dtype=torch.uint8, device="cuda")
    l1 = _lib.FvqLinear(q1.qweight.data_ptr(), q1.scale.data_ptr(), q1.global_sf.data_ptr(),
                        q1.bias.data_ptr(), d, f)
    l2 = _lib.FvqLinear(q2.qweight.data_ptr(), q2.scale.data_ptr(), q2.global_sf.data_ptr(),
                        q2.bias.data_ptr(), f, d)
    y = torch.empty_like(ref)
    ms = (ctypes.c_float * 4)()
    _lib.call("fvq_nvfp4_ffn_profile", x.data_ptr(), m, ctypes.byref(l1), ctypes.byref(l2),
              y.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream, ms)
    assert torch.equal(y, ref)
    assert all(t > 0 for t in ms), list(ms)


@pytest.mark.parametrize("mode,m", [(1, 7680), (2, 7680), (1, 300), (2, 300), (1, 1920), (1, 8100),
                                    (1, 3840), (2, 3840)])
def test_ffn_same_bits_with_and_without_sm_pairs(ffn_layer, mode, m):
    """With fvq_set_gemm_pairing(1 or 2), GEMM2 of the FFN runs on SM pairs (raw or
    replicated W scales), ragged row counts included (300, 1920 and 8100 rows leave the
    last 256-row pair tile partly or, for one CTA, wholly past m), and with the last
    partial round split into 256 x 128 halves (7680 and 3840 rows: 180 and 90 tiles on 74
    pairs; 300 rows: 12 tiles, all split); the output bits equal the one-SM kernel's."""
    from flashvsr_optimizations_b200 import _lib
    ffn, _ = ffn_layer
    x = bits_to_dev(W.student_t(m, W.D_MODEL, seed=9))
    try:
        _lib.call("fvq_set_gemm_pairing", 0)
        single = ffn(x)
        _lib.call("fvq_set_gemm_pairing", mode)
        paired = ffn(x)
    finally:
        _lib.call("fvq_set_gemm_pairing", 1)   # the library default
    torch.cuda.synchronize()
    assert torch.equal(paired, single)


def test_global_scale_shards_reproduce_the_single_gpu_layer(ffn_layer):
    """Sharding with global scales (sharding.nvfp4_ffn_global_scales): each shard quantizes
    with the amax of the whole tensor, so the gathered rows equal the unsharded FFN bit for
    bit.  The reductions are emulated in one process by a reducer that returns the
    whole-tensor maxima (what all_reduce(MAX) over the shards yields)."""
    from flashvsr_optimizations_b200.sharding import nvfp4_ffn_global_scales, row_range
    ffn, _ = ffn_layer
    x = bits_to_dev(W.student_t(1000, W.D_MODEL, seed=17))
    l1 = ffn[0]
    a_full = ops.amax(x)
    q, s, g = ops.nvfp4_quantize_from_amax(x, a_full)
    assert torch.equal(g, ops.global_scale(x))
    _, amax_h_full = ops.nvfp4_gemm(q, s, g, l1.qweight, l1.scale, l1.global_sf, l1.bias, gelu=True)
    want = ffn(x)
    parts = []
    for world in (2, 3):
        parts = []
        for rank in range(world):
            lo, hi = row_range(x.shape[0], world, rank)
            maxima = iter([a_full.clone(), amax_h_full.clone()])
            parts.append(nvfp4_ffn_global_scales(x[lo:hi], ffn, reduce_amax=lambda a, grp: next(maxima)))
        assert torch.equal(torch.cat(parts), want), world
    # a rank without rows still takes part in both reductions
    calls = []
    empty = nvfp4_ffn_global_scales(x[:0], ffn, reduce_amax=lambda a, grp: calls.append(1) or a)
    assert empty.shape == (0, W.D_MODEL) and len(calls) == 2
