"""Block-scaled NVFP4 GEMM (tcgen05) on the GPU.

The GEMM is checked against the oracle's dequantise-and-multiply on random
codes and scale bytes (this exercises the operand, scale-factor and TMEM
layouts independently of the quantizer), against the reference's own
QuantLinear output (golden, flashinfer.mm_fp4 on a B200), and the GELU/amax
epilogue against the oracle's GELU.
Tolerance: the GPU accumulates in fp32 in its own order while the oracle sums
in float64, so outputs agree to within one bf16 rounding: relative Frobenius
error <= 2e-3 and every element within 2 bf16 ulps (+ a tiny absolute slack).
"""
import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import QuantLinear
from helpers import bits_to_dev, dev_to_bits, f32_from_bits, golden, golden_meta
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 2e-3


def _random_operand(rows, k, rng, sf_lo=0x30, sf_hi=0x48):
    """Random E2M1 codes and E4M3 scale bytes in a moderate range (swizzled layout)."""
    codes = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
    sf_un = rng.integers(sf_lo, sf_hi, size=(rows, k // 16), dtype=np.uint8)
    sf = np.zeros(O.sf_swizzled_size(rows, k), dtype=np.uint8)
    sf[O.sf_swizzled_offsets(rows, k // 16)] = sf_un
    return codes, sf


def _close_bf16(got_bits, ref_f32, ulps=2):
    got = O.bf16_bits_to_f32(got_bits).astype(np.float64)
    ref = np.asarray(ref_f32, dtype=np.float64)
    rel = O.frobenius_rel(got, ref)
    ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -8
    worst = np.max(np.abs(got - ref) / (ulp + 1e-6 * np.abs(ref).max()))
    return rel, worst


# (2560, 2048, 512): 160 tiles on 148 SMs, so the 12 past the first round run as
# 24 N = 128 halves
@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (200, 512, 512), (300, 256, 1536),
                                   (1, 256, 256), (513, 768, 768), (2560, 2048, 512)])
def test_gemm_random_operands_vs_oracle(m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    a, a_sf = _random_operand(m, k, rng)
    w, w_sf = _random_operand(n, k, rng)
    g_a = torch.tensor([1.5], device="cuda")
    g_w = torch.tensor([0.75], device="cuda")
    out, _ = ops.nvfp4_gemm(torch.from_numpy(a).cuda(), torch.from_numpy(a_sf).cuda(), g_a,
                            torch.from_numpy(w).cuda(), torch.from_numpy(w_sf).cuda(), g_w)
    alpha = O.gemm_alpha(np.float32(1.5), np.float32(0.75))
    ref = alpha * (O.dequantize(a, a_sf, m, k).astype(np.float64)
                   @ O.dequantize(w, w_sf, n, k).astype(np.float64).T)
    rel, worst = _close_bf16(dev_to_bits(out), ref)
    assert rel <= REL_FRO_TOL, rel
    assert worst <= 2.0, worst


def test_gemm_scale_placement_one_hot():
    """Unit codes, all scales 1 except one block per operand: pins the scale layout."""
    m, n, k = 256, 256, 512
    one = 0x22  # two E2M1 codes of 1.0
    a = np.full((m, k // 2), one, dtype=np.uint8)
    w = np.full((n, k // 2), one, dtype=np.uint8)
    sf_one = 0x38  # E4M3 1.0
    a_un = np.full((m, k // 16), sf_one, dtype=np.uint8)
    w_un = np.full((n, k // 16), sf_one, dtype=np.uint8)
    a_un[77, 19] = 0x40  # 2.0
    w_un[201, 5] = 0x48  # 4.0
    a_sf = np.zeros(O.sf_swizzled_size(m, k), dtype=np.uint8)
    w_sf = np.zeros(O.sf_swizzled_size(n, k), dtype=np.uint8)
    a_sf[O.sf_swizzled_offsets(m, k // 16)] = a_un
    w_sf[O.sf_swizzled_offsets(n, k // 16)] = w_un
    g1 = torch.ones(1, device="cuda")
    out, _ = ops.nvfp4_gemm(torch.from_numpy(a).cuda(), torch.from_numpy(a_sf).cuda(), g1,
                            torch.from_numpy(w).cuda(), torch.from_numpy(w_sf).cuda(), g1)
    got = O.bf16_bits_to_f32(dev_to_bits(out))
    ref = O.dequantize(a, a_sf, m, k).astype(np.float64) @ O.dequantize(w, w_sf, n, k).astype(np.float64).T
    assert np.array_equal(got, O.round_bf16(ref.astype(np.float32)))


def test_gemm_bias_and_gelu_epilogue_vs_oracle():
    m, n, k = 200, 512, 768
    rng = np.random.default_rng(3)
    a, a_sf = _random_operand(m, k, rng, 0x28, 0x38)
    w, w_sf = _random_operand(n, k, rng, 0x28, 0x38)
    bias = W.f32_to_bf16_bits(rng.standard_normal(n).astype(np.float32) * np.float32(0.1))
    g = torch.tensor([2.0], device="cuda")
    args = (torch.from_numpy(a).cuda(), torch.from_numpy(a_sf).cuda(), g,
            torch.from_numpy(w).cuda(), torch.from_numpy(w_sf).cuda(), g, bits_to_dev(bias))
    y, _ = ops.nvfp4_gemm(*args, gelu=False)
    h, amax = ops.nvfp4_gemm(*args, gelu=True)
    alpha = O.gemm_alpha(np.float32(2.0), np.float32(2.0))
    acc = (O.dequantize(a, a_sf, m, k).astype(np.float64) @ O.dequantize(w, w_sf, n, k).astype(np.float64).T)
    y_ref = O.bias_add_bf16(O.round_bf16((alpha * acc).astype(np.float32)), bias)
    rel, worst = _close_bf16(dev_to_bits(y), y_ref)
    assert rel <= REL_FRO_TOL and worst <= 2.0
    # GELU applied to the GPU's own pre-activation: differences come only from tanh
    h_ref = O.gelu_tanh_bf16(O.bf16_bits_to_f32(dev_to_bits(y)))
    rel, worst = _close_bf16(dev_to_bits(h), h_ref)
    assert rel <= 1e-3 and worst <= 2.0
    h_bits = dev_to_bits(h)
    assert np.float32(amax.item()) == np.abs(O.bf16_bits_to_f32(h_bits)).max()


def test_quant_linear_matches_reference_golden():
    meta = golden_meta()["cases"]["lin_200x1536x256"]
    fix = golden("lin_200x1536x256")
    wb, bb = W.linear_params(256, 1536, seed=30, b_std=0.01)
    xb = W.gaussian(200, 1536, seed=31)
    lin = torch.nn.Linear(1536, 256, bias=True).cuda()
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb).float())
        lin.bias.copy_(bits_to_dev(bb).float())
    ql = QuantLinear(lin, "nvfp4")
    import hashlib
    assert hashlib.sha256(ql.qweight.cpu().numpy().tobytes()).hexdigest() == meta["qweight_sha256"]
    assert hashlib.sha256(ql.scale.cpu().numpy().tobytes()).hexdigest() == meta["scale_sha256"]
    assert np.uint32(ql.global_sf.cpu().numpy().view(np.uint32)[0]) == fix["gw_bits"][0]
    y = ql(bits_to_dev(xb))
    got = dev_to_bits(y)
    ref = O.bf16_bits_to_f32(fix["y"])
    rel, worst = _close_bf16(got, ref)
    assert rel <= REL_FRO_TOL and worst <= 2.0
    # report how often the two fp32 accumulation orders round to the same bf16
    same = np.mean(got == fix["y"])
    assert same >= 0.95, same


def test_mm_fp4_device_alpha_equals_gscales():
    rng = np.random.default_rng(11)
    m, n, k = 130, 256, 512
    a, a_sf = _random_operand(m, k, rng)
    w, w_sf = _random_operand(n, k, rng)
    ga = torch.tensor([3.0], device="cuda")
    gw = torch.tensor([0.3], device="cuda")
    ta, tas, tw, tws = (torch.from_numpy(v).cuda() for v in (a, a_sf, w, w_sf))
    y1, _ = ops.nvfp4_gemm(ta, tas, ga, tw, tws, gw)
    y2 = ops.mm_fp4(ta, tas, tw, tws, 1. / (ga * gw))
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("order", ["sorted", "shuffled", "shuffled_odd"])
def test_epilogue_gelu_matches_torch_on_every_bf16_input(order):
    """The GELU epilogue (shared-memory table plus exact formula) equals torch's
    GELU(approximate='tanh') on all 65536 bf16 inputs, NaNs compared as NaN.
    The probe pairs values 2i, 2i+1 into one bf16x2 word as the epilogue does;
    the shuffled orders pair table-range values with out-of-range ones."""
    from flashvsr_optimizations_b200 import _lib
    bits = torch.arange(0, 1 << 16, dtype=torch.int32)
    if order != "sorted":
        bits = bits[torch.randperm(bits.numel(), generator=torch.Generator().manual_seed(7))]
    if order == "shuffled_odd":
        bits = bits[:-1]
    bits = bits.to(torch.int16).cuda()
    x = bits.view(torch.bfloat16)
    out = torch.empty_like(bits)
    _lib.call("fvq_gelu_bf16_probe", bits.data_ptr(), out.data_ptr(), bits.numel(),
              torch.cuda.current_stream().cuda_stream)
    ref = torch.nn.functional.gelu(x, approximate="tanh")
    got = out.view(torch.bfloat16)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(got), nan)
    mismatch = (got.view(torch.int16) != ref.view(torch.int16)) & ~nan
    assert int(mismatch.sum()) == 0, bits[mismatch][:10].tolist()


def _replicate_ref(sf, n, k):
    """The replicated W-scale layout, restated with numpy: atom (2*nb + h, j) of
    the 128x4 layout at ((((nb * k64 + j) * 2 + h) * 4 + r) * 512) for r = 0..3."""
    k64 = k // 64
    atoms = sf.reshape(n // 256, 2, k64, 512).transpose(0, 2, 1, 3)        # [nb, j, h, 512]
    return np.ascontiguousarray(np.broadcast_to(atoms[:, :, :, None, :],
                                                (n // 256, k64, 2, 4, 512))).reshape(-1)


@pytest.mark.parametrize("n,k", [(256, 256), (512, 768), (1536, 8960)])
def test_replicated_w_scales_layout(n, k):
    from flashvsr_optimizations_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(n + k)
    sf = rng.integers(0, 256, size=n * k // 16, dtype=np.uint8)
    assert lib.fvq_w_scales_replicated_bytes(n, k) == 4 * sf.size
    dsf = torch.from_numpy(sf).cuda()
    rep = torch.empty(4 * sf.size, dtype=torch.uint8, device="cuda")
    _lib.call("fvq_replicate_w_scales", dsf.data_ptr(), n, k, rep.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    assert np.array_equal(rep.cpu().numpy(), _replicate_ref(sf, n, k))


# m % 256 == 0 runs on SM pairs (clusters of two CTAs, tcgen05.mma.cta_group::2);
# (2560, 2048, 512) has 80 pair tiles for 74 pairs, so some pairs take two tiles
@pytest.mark.parametrize("m,n,k", [(1, 256, 256), (200, 512, 512), (300, 256, 1536),
                                   (513, 768, 768), (256, 256, 256), (512, 768, 512),
                                   (768, 256, 1536), (2560, 2048, 512), (7680, 1536, 8960)])
@pytest.mark.parametrize("pairing", [0, 1, 2])
def test_gemm_with_replicated_w_scales_is_bit_identical(m, n, k, pairing):
    """fvq_nvfp4_gemm_wrep (four 128x256b W-scale copies per K tile; on SM pairs
    when pairing is on and m % 256 == 0) and, with pairing on, fvq_nvfp4_gemm on
    SM pairs with the W scales in the library layout, give the same bits as
    fvq_nvfp4_gemm on one SM per tile (eight 32x128b.warpx4 copies), bias included."""
    from flashvsr_optimizations_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(m + 3 * n + k)
    a, a_sf = _random_operand(m, k, rng)
    w, w_sf = _random_operand(n, k, rng)
    ta, tas, tw, tws = (torch.from_numpy(v).cuda() for v in (a, a_sf, w, w_sf))
    ga = torch.tensor([1.25], device="cuda")
    gw = torch.tensor([0.5], device="cuda")
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(k)) * 0.05).to(torch.bfloat16).cuda()
    st = torch.cuda.current_stream().cuda_stream
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    rep = torch.empty(lib.fvq_w_scales_replicated_bytes(n, k), dtype=torch.uint8, device="cuda")
    raw = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    try:
        _lib.call("fvq_set_gemm_pairing", 0)
        _lib.call("fvq_nvfp4_gemm", ta.data_ptr(), tas.data_ptr(), ga.data_ptr(), tw.data_ptr(),
                  tws.data_ptr(), gw.data_ptr(), bias.data_ptr(), ref.data_ptr(), m, n, k,
                  _lib.EPI_BF16, None, st)
        _lib.call("fvq_replicate_w_scales", tws.data_ptr(), n, k, rep.data_ptr(), st)
        _lib.call("fvq_set_gemm_pairing", pairing)
        _lib.call("fvq_nvfp4_gemm_wrep", ta.data_ptr(), tas.data_ptr(), ga.data_ptr(), tw.data_ptr(),
                  rep.data_ptr(), gw.data_ptr(), bias.data_ptr(), got.data_ptr(), m, n, k, st)
        _lib.call("fvq_nvfp4_gemm", ta.data_ptr(), tas.data_ptr(), ga.data_ptr(), tw.data_ptr(),
                  tws.data_ptr(), gw.data_ptr(), bias.data_ptr(), raw.data_ptr(), m, n, k,
                  _lib.EPI_BF16, None, st)
    finally:
        _lib.call("fvq_set_gemm_pairing", 1)   # the library default
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(raw.view(torch.int16), ref.view(torch.int16))
