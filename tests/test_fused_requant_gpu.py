"""The FFN with the intermediate quantized inside GEMM1's epilogue (fvq_nvfp4_ffn_fused).

The reference scales the GELU output h by 2688 / amax(h) of the whole tensor
(ffn_quantization.py:63-64), which is known only after GEMM1 has finished, so the exact
path keeps h in bf16 for one round trip through HBM.  The fused path quantizes h in
GEMM1's epilogue with a provisional scale from an estimate of max |h| instead.

What is checked here:
* the epilogue's quantizer is the activation quantizer's recipe: given the true amax(h)
  as the estimate, the fused FFN equals the exact FFN (and the reference's golden
  output) bit for bit; with one bit of headroom (half the encode scale, a power of two)
  it is bit-identical too;
* with a provisional scale that is not the exact one (delayed scaling from another
  batch, a static estimate) the output is a different but equally accurate quantization:
  its distance to the unquantized FFN (bf16 weights, fp32 math) is within 2% of the
  reference's own distance, and its distance to the reference's NVFP4 output stays
  below FUSED_VS_REF (stated bound: a different E4M3 scale grid moves single E2M1
  codes; measured on the 7680-token layer: 0.083 with delayed scaling);
* saturation (an estimate far below max |h|) sets flag bit 0 and the module can rerun
  the exact path; scale underflow sets bit 1.
"""
import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, QuantLinear
from helpers import bits_to_dev, dev_to_bits, golden, golden_meta
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

FUSED_VS_REF = 0.12       # Frobenius-relative distance to the reference NVFP4 output
ACCURACY_SLACK = 1.02     # fused distance to the unquantized FFN <= 1.02 x the reference's


def _linear(wb, bb):
    out_f, in_f = wb.shape
    lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    return lin


@pytest.fixture(scope="module")
def layer():
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    l1, l2 = _linear(w1, b1), _linear(w2, b2)
    ffn = NVFP4FFN(QuantLinear(l1, "nvfp4"), torch.nn.GELU(approximate="tanh"), QuantLinear(l2, "nvfp4"))
    return ffn, (l1, l2)


def _fused(ffn, x, hint, headroom=0):
    l1, l2 = ffn[0], ffn[2]
    seen = torch.zeros(1, dtype=torch.float32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.nvfp4_ffn_fused(x, l1.qweight, l1.scale, l1.global_sf, l1.bias, l2.qweight, l2.scale,
                            l2.global_sf, l2.bias, hint, headroom, seen, flags)
    return y, seen, flags


def _amax_h(ffn, x):
    l1 = ffn[0]
    g = ops.global_scale(x)
    q, s = ops.nvfp4_quantize(x, g)
    _, amax_h = ops.nvfp4_gemm(q, s, g, l1.qweight, l1.scale, l1.global_sf, l1.bias, gelu=True)
    return amax_h


def _unquantized(lins, x):
    l1, l2 = lins
    with torch.no_grad():
        h = torch.nn.functional.gelu(x.float() @ l1.weight.float().t() + l1.bias.float(),
                                     approximate="tanh")
        return h @ l2.weight.float().t() + l2.bias.float()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


@pytest.mark.parametrize("m", [64, 300, 7680])
def test_true_amax_hint_gives_the_exact_ffn(layer, m):
    ffn, _ = layer
    x = bits_to_dev(W.student_t(m, W.D_MODEL, seed=1))
    exact = ffn(x)
    amax_h = _amax_h(ffn, x)
    y, seen, flags = _fused(ffn, x, amax_h)
    torch.cuda.synchronize()
    assert float(seen.item()) == float(amax_h.item())
    assert int(flags.item()) & 1 == 0
    assert torch.equal(y, exact), f"{int((y != exact).sum())} values differ"
    # one bit of headroom, or twice the estimate: half the encode scale, an exact power of
    # two, which moves every block scale by one binade and leaves the codes and the output
    for hint, headroom in ((amax_h, 1), (amax_h * 2.0, 0)):
        y2, _, flags2 = _fused(ffn, x, hint, headroom=headroom)
        assert torch.equal(y2, exact)
        assert int(flags2.item()) & 1 == 0


def test_true_amax_hint_matches_the_reference_golden(layer):
    ffn, _ = layer
    fix = golden("ffn_7680_rows")
    x = bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1))
    y, _, _ = _fused(ffn, x, _amax_h(ffn, x))
    got = dev_to_bits(y[torch.from_numpy(fix["rows"]).cuda()])
    assert np.array_equal(got, fix["y_rows"])


@pytest.mark.parametrize("mode", ["delayed", "static"])
def test_provisional_scale_is_as_accurate_as_the_reference(layer, mode):
    """7680-token layer (two latent frames): delayed scaling seeded by another batch of the
    same stream, or a static estimate 1.5x the true maximum; compared with the reference's
    golden rows and with the unquantized FFN."""
    ffn, lins = layer
    fix = golden("ffn_7680_rows")
    meta = golden_meta()["cases"]["ffn_7680_rows"]
    x = bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=1))
    exact = ffn(x)
    m = NVFP4FFN(ffn[0], ffn[1], ffn[2])
    if mode == "delayed":
        m.set_h_scaling("delayed")
        m(bits_to_dev(W.student_t(W.M_ONE_LAYER, W.D_MODEL, seed=2)))   # seeds the estimate
    else:
        m.set_h_scaling("static", amax=1.5 * float(_amax_h(ffn, x).item()))
    y = m(x)
    torch.cuda.synchronize()
    assert m.h_flags() & 1 == 0
    rows = torch.from_numpy(fix["rows"]).cuda()
    vs_ref = O.frobenius_rel(O.bf16_bits_to_f32(dev_to_bits(y[rows])), O.bf16_bits_to_f32(fix["y_rows"]))
    assert vs_ref <= FUSED_VS_REF, vs_ref
    assert abs(float(y.float().norm()) - meta["y_fro"]) / meta["y_fro"] <= FUSED_VS_REF
    truth = _unquantized(lins, x)
    err_fused, err_ref = _rel(y, truth), _rel(exact, truth)
    assert err_fused <= ACCURACY_SLACK * err_ref, (err_fused, err_ref)


def test_saturation_is_flagged_and_rerun_gives_the_exact_path(layer):
    ffn, _ = layer
    x = bits_to_dev(W.student_t(1024, W.D_MODEL, seed=3))
    exact = ffn(x)
    amax_h = _amax_h(ffn, x)
    _, _, flags = _fused(ffn, x, amax_h * 0.25)
    torch.cuda.synchronize()
    assert int(flags.item()) & 1
    m = NVFP4FFN(ffn[0], ffn[1], ffn[2])
    m.set_h_scaling("static", amax=0.25 * float(amax_h.item()), rerun_on_saturation=True)
    y = m(x)
    assert torch.equal(y, exact)
    # an estimate far above max |h| pushes small blocks' scales below E4M3's range
    _, _, flags = _fused(ffn, x, amax_h * float(2 ** 20))
    torch.cuda.synchronize()
    assert int(flags.item()) & 2


def test_delayed_module_updates_its_estimate_without_host_sync(layer):
    """Consecutive calls alternate the estimate and the observed maximum on the device;
    the second call's estimate is the first call's max |h|."""
    ffn, _ = layer
    m = NVFP4FFN(ffn[0], ffn[1], ffn[2]).set_h_scaling("delayed", headroom_log2=0)
    xs = [bits_to_dev(W.student_t(512, W.D_MODEL, seed=s)) for s in (7, 8, 9)]
    m(xs[0])                                         # exact, seeds the estimate
    seen0 = float(_amax_h(ffn, xs[0]).item())
    m(xs[1])
    torch.cuda.synchronize()
    assert float(m._h_state[0].item()) == seen0          # the estimate of the second call
    assert float(m._h_state[1].item()) == float(_amax_h(ffn, xs[1]).item())
    y3 = m(xs[2])
    assert y3.shape == (512, W.D_MODEL)


def test_rejects_aliased_hint_and_bad_headroom(layer):
    ffn, _ = layer
    import flashvsr_optimizations_b200 as fvq
    x = bits_to_dev(W.student_t(128, W.D_MODEL, seed=4))
    l1, l2 = ffn[0], ffn[2]
    a = torch.ones(1, dtype=torch.float32, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(fvq.FvqError):
        ops.nvfp4_ffn_fused(x, l1.qweight, l1.scale, l1.global_sf, l1.bias, l2.qweight, l2.scale,
                            l2.global_sf, l2.bias, a, 0, a, flags)
    with pytest.raises(fvq.FvqError):
        ops.nvfp4_ffn_fused(x, l1.qweight, l1.scale, l1.global_sf, l1.bias, l2.qweight, l2.scale,
                            l2.global_sf, l2.bias, a, 31, torch.zeros_like(a), flags)
