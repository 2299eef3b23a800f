"""The DiT block's FFN step on the GPU: x + gate * FFN(LN(x) * (1 + scale) + shift).

The block is upstream code around the reference's FFN (the caller of
``block.ffn`` that ffn_quantization.py:77-80 patches), so its parity is checked
against torch's composition of the same steps on bf16 tensors:

* ``ln_modulate`` against ``F.layer_norm(x) * (1 + scale) + shift``: torch
  reduces mean and variance in another order (Welford), so a bf16 rounding can
  land one ulp apart; at least 99% of the values are equal and none is off by
  more than one ulp of the larger of its terms.
* the gated residual, given the same u, bit for bit: ``x + gate * FFN(u)``
  with the fused FFN's own result.
* the whole step against torch's LN/modulation feeding the same FFN:
  Frobenius-relative error of the FFN branch <= 5e-3 (the FFN bar).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from flashvsr_optimizations_b200 import ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, QuantLinear
from helpers import bits_to_dev
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

EPS = 1e-6
FFN_TOL = 5e-3


def _linear(out_f, in_f, wb, bb):
    lin = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(bits_to_dev(wb))
        lin.bias.copy_(bits_to_dev(bb))
    return lin


@pytest.fixture(scope="module")
def ffn():
    w1, b1 = W.linear_params(W.D_FF, W.D_MODEL, seed=20, b_std=0.01)
    w2, b2 = W.linear_params(W.D_MODEL, W.D_FF, seed=21, b_std=0.01)
    seq = torch.nn.Sequential(_linear(W.D_FF, W.D_MODEL, w1, b1), torch.nn.GELU(approximate="tanh"),
                              _linear(W.D_MODEL, W.D_FF, w2, b2))
    return NVFP4FFN(QuantLinear(seq[0], "nvfp4"), seq[1], QuantLinear(seq[2], "nvfp4"))


def _modulation(d, seed):
    g = torch.Generator().manual_seed(seed)
    shift = (torch.randn(d, generator=g) * 0.2).to(torch.bfloat16).cuda()
    scale = (torch.randn(d, generator=g) * 0.2).to(torch.bfloat16).cuda()
    gate = (torch.randn(d, generator=g) * 0.5).to(torch.bfloat16).cuda()
    return shift, scale, gate


def _x(m, d, seed):
    return bits_to_dev(W.student_t(m, d, seed=seed))


def _torch_u(x, shift, scale):
    return F.layer_norm(x, (x.shape[-1],), eps=EPS) * (1 + scale) + shift


def _ulp_bf16(v):
    """One bf16 ulp at |v| (fp32 tensor)."""
    e = torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -126)))
    return torch.pow(2.0, e - 7)


@pytest.mark.parametrize("m,d", [(1, 1536), (300, 1536), (4096, 1536), (77, 8), (64, 2048),
                                 (33, 264), (128, 1032)])
def test_ln_modulate_matches_torch(m, d):
    x = _x(m, d, seed=m + d)
    shift, scale, _ = _modulation(d, seed=d)
    u = ops.ln_modulate(x, shift, scale, EPS)
    ref = _torch_u(x, shift, scale)
    eq = (u == ref).float().mean().item()
    assert eq >= 0.99, eq
    # LN(x) one ulp apart, carried through the product, then each of the two
    # roundings (product, sum) half an ulp either side: |du| <= ulp(n)|1 + s| +
    # ulp(n (1 + s)) + ulp(u), ulps taken at the larger binade of the two values
    n = F.layer_norm(x.float(), (d,), eps=EPS)
    one_s = (1 + scale.float()).abs()
    bound = (_ulp_bf16(n * 1.01) * one_s + _ulp_bf16(n * one_s * 1.01)
             + _ulp_bf16(torch.maximum(u.float().abs(), ref.float().abs())))
    diff = (u.float() - ref.float()).abs()
    bad = diff > bound
    assert not bool(bad.any()), (int(bad.sum()), float((diff / bound).max()))


def test_ln_modulate_constant_rows_give_shift():
    d = 1536
    x = torch.full((16, d), 0.75, dtype=torch.bfloat16, device="cuda")
    x[3] = -2.0
    shift, scale, _ = _modulation(d, seed=5)
    u = ops.ln_modulate(x, shift, scale, EPS)
    assert torch.equal(u, shift.expand(16, d))
    assert torch.equal(u, _torch_u(x, shift, scale))


def test_gated_residual_bit_exact_given_u(ffn):
    """out = bf16(x + bf16(gate * FFN(u))) with FFN(u) the fused FFN's own output."""
    for m, seed in ((64, 1), (300, 2), (W.M_ONE_LAYER, 3)):
        x = _x(m, W.D_MODEL, seed=seed)
        shift, scale, gate = _modulation(W.D_MODEL, seed=seed)
        out = ffn.modulated(x, shift, scale, gate, EPS)
        u = ops.ln_modulate(x, shift, scale, EPS)
        ref = x + gate * ffn(u)
        assert torch.equal(out, ref), f"m={m}: {int((out != ref).sum())} of {out.numel()} differ"


def test_block_matches_torch_composition(ffn):
    m = W.M_ONE_LAYER
    x = _x(m, W.D_MODEL, seed=11)
    shift, scale, gate = _modulation(W.D_MODEL, seed=11)
    out = ffn.modulated(x, shift, scale, gate, EPS)
    ref = x + gate * ffn(_torch_u(x, shift, scale))
    branch = (out.float() - x.float()).cpu().numpy()
    branch_ref = (ref.float() - x.float()).cpu().numpy()
    rel = O.frobenius_rel(branch, branch_ref)
    assert rel <= FFN_TOL, rel
    assert O.frobenius_rel(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= FFN_TOL


def test_block_3d_input_ragged_rows_and_repeat(ffn):
    shift, scale, gate = _modulation(W.D_MODEL, seed=4)
    x = _x(2 * 129, W.D_MODEL, seed=4)
    flat = ffn.modulated(x, shift, scale, gate, EPS)
    x3 = x.view(2, 129, W.D_MODEL)
    out3 = ffn.modulated(x3, shift, scale, gate, EPS)
    assert out3.shape == x3.shape
    assert torch.equal(out3.reshape(-1, W.D_MODEL), flat)
    assert torch.equal(ffn.modulated(x3, shift, scale, gate, EPS), out3)
    one = ffn.modulated(x[:1], shift, scale, gate, EPS)
    assert torch.equal(one, x[:1] + gate * ffn(ops.ln_modulate(x[:1], shift, scale, EPS)))


def test_block_rejects_bad_modulation_vectors(ffn):
    x = _x(8, W.D_MODEL, seed=1)
    shift, scale, gate = _modulation(W.D_MODEL, seed=1)
    with pytest.raises(ValueError):
        ffn.modulated(x, shift[:-8], scale, gate, EPS)
    with pytest.raises(ValueError):
        ffn.modulated(x, shift, scale.float(), gate, EPS)
    with pytest.raises(ValueError):
        ops.ln_modulate(x, shift, scale[:100], EPS)


@pytest.mark.parametrize("m", [7680, 512, 300])
def test_block_same_bits_on_one_sm_and_on_sm_pairs(ffn, m):
    """The gated-residual GEMM runs on SM pairs by default when m % 256 == 0 and on one SM per
    tile with pairing off (or for other row counts); both give the same bits."""
    from flashvsr_optimizations_b200 import _lib
    x = _x(m, W.D_MODEL, seed=m)
    shift, scale, gate = _modulation(W.D_MODEL, seed=m)
    try:
        _lib.call("fvq_set_gemm_pairing", 0)
        single = ffn.modulated(x, shift, scale, gate, EPS)
        _lib.call("fvq_set_gemm_pairing", 1)
        paired = ffn.modulated(x, shift, scale, gate, EPS)
    finally:
        _lib.call("fvq_set_gemm_pairing", 1)   # the library default
    torch.cuda.synchronize()
    assert torch.equal(paired, single)


@pytest.mark.parametrize("d,f,m", [(256, 512, 300), (512, 768, 512), (1024, 512, 129), (2048, 512, 384)])
def test_block_other_widths_bit_exact_given_u(d, f, m):
    """The block's first launch normalises and modulates x inside the quantizer (one
    instantiation per row width); at every width its result equals running the stand-alone
    LayerNorm + modulation kernel first: out = x + gate * FFN(ln_modulate(x)), bit for bit."""
    g = torch.Generator().manual_seed(d + f)
    seq = torch.nn.Sequential(torch.nn.Linear(d, f), torch.nn.GELU(approximate="tanh"), torch.nn.Linear(f, d))
    with torch.no_grad():
        for lin in (seq[0], seq[2]):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
            lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.01)
    seq = seq.to(device="cuda", dtype=torch.bfloat16)
    blk = NVFP4FFN(QuantLinear(seq[0], "nvfp4"), seq[1], QuantLinear(seq[2], "nvfp4"))
    x = (torch.randn(m, d, generator=g) * 0.7).to(torch.bfloat16).cuda()
    shift, scale, gate = _modulation(d, seed=d)
    out = blk.modulated(x, shift, scale, gate, EPS)
    ref = x + gate * blk(ops.ln_modulate(x, shift, scale, EPS))
    torch.cuda.synchronize()
    assert torch.equal(out, ref), f"{int((out != ref).sum())} of {out.numel()} differ"
