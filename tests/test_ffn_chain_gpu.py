"""FFNs that feed each other directly: fvq_nvfp4_ffn_chain / NVFP4FFNStack.

Each call's second GEMM produces max |y| in its epilogue and the next call quantizes its
input with it instead of running its own amax pass (the 30-layer FFN-stack workloads; the
reference's DiT blocks put attention between FFNs, so it has no such call).  Checked: the
outputs equal the unchained FFN bit for bit, the handed-on maximum equals the library's
amax of the output (which the reference's global_scale would take, ffn_quantization.py:29-32),
at ragged and SM-pair row counts and with every GEMM pairing mode, and aliasing the two
maxima is rejected.
"""
import ctypes

import pytest
import torch

from flashvsr_optimizations_b200 import _lib, ops, workloads as W
from flashvsr_optimizations_b200.ffn_quantization import NVFP4FFN, NVFP4FFNStack, QuantLinear
from helpers import bits_to_dev

pytestmark = pytest.mark.gpu


def _ffn(layer):
    w1, b1, w2, b2 = W.stack_layer_params(layer)

    def lin(wb, bb):
        out_f, in_f = wb.shape
        m = torch.nn.Linear(in_f, out_f, bias=True, device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            m.weight.copy_(bits_to_dev(wb))
            m.bias.copy_(bits_to_dev(bb))
        return QuantLinear(m, "nvfp4")
    return NVFP4FFN(lin(w1, b1), torch.nn.GELU(approximate="tanh"), lin(w2, b2))


@pytest.fixture(scope="module")
def ffns():
    return [_ffn(layer) for layer in range(3)]


def _args(ffn):
    l1, l2 = ffn[0], ffn[2]
    return (l1.qweight, l1.scale, l1.global_sf, l1.bias, l2.qweight, l2.scale, l2.global_sf, l2.bias)


@pytest.mark.parametrize("m", [64, 300, 1920, 7680])
def test_stack_equals_layer_by_layer(ffns, m):
    x = bits_to_dev(W.gaussian(m, W.D_MODEL, seed=3))
    want = x
    for f in ffns:
        want = f(want)
    got = NVFP4FFNStack(ffns)(x)
    assert torch.equal(got, want)


@pytest.mark.parametrize("pairing", [0, 1, 2])
@pytest.mark.parametrize("m", [300, 2048])
def test_chain_output_and_amax(ffns, m, pairing):
    """y equals nvfp4_ffn's; y_amax equals the amax kernel's max |y|; given x_amax (the
    amax kernel's max |x|) the call computes the same y as without it."""
    ffn = ffns[0]
    x = bits_to_dev(W.student_t(m, W.D_MODEL, seed=11))
    try:
        _lib.call("fvq_set_gemm_pairing", pairing)
        want = ops.nvfp4_ffn(x, *_args(ffn))
        y0, a0 = ops.nvfp4_ffn_chain(x, *_args(ffn))
        y1, a1 = ops.nvfp4_ffn_chain(x, *_args(ffn), ops.amax(x))
    finally:
        _lib.call("fvq_set_gemm_pairing", 1)   # the library default
    assert torch.equal(y0, want) and torch.equal(y1, want)
    ref = ops.amax(want)
    assert torch.equal(a0, ref.reshape(1)) and torch.equal(a1, ref.reshape(1))


def test_chain_rejects_aliased_maxima(ffns):
    ffn = ffns[0]
    lib = _lib.load()
    m, d, f = 128, W.D_MODEL, W.D_FF
    x = bits_to_dev(W.gaussian(m, d, seed=2))
    y = torch.empty_like(x)
    amax = torch.zeros(1, dtype=torch.float32, device="cuda")
    nbytes = lib.fvq_nvfp4_ffn_workspace_bytes(m, d, f)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    l1, l2 = ffn[0], ffn[2]
    s1 = _lib.FvqLinear(l1.qweight.data_ptr(), l1.scale.data_ptr(), l1.global_sf.data_ptr(),
                        l1.bias.data_ptr(), d, f)
    s2 = _lib.FvqLinear(l2.qweight.data_ptr(), l2.scale.data_ptr(), l2.global_sf.data_ptr(),
                        l2.bias.data_ptr(), f, d)
    rc = lib.fvq_nvfp4_ffn_chain(x.data_ptr(), m, ctypes.byref(s1), ctypes.byref(s2), y.data_ptr(),
                                 amax.data_ptr(), amax.data_ptr(), ws.data_ptr(), nbytes,
                                 torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FVQ_EINVAL
    assert b"alias" in lib.fvq_last_error()


@pytest.mark.parametrize("m", [300, 1920])
def test_graphed_stack_equals_eager(ffns, m):
    """GraphedFFNStack: the stack's launches captured into one CUDA graph over a fixed input
    buffer; each replay recomputes from the buffer's current contents, bit-identical to the
    eager stack."""
    stack = NVFP4FFNStack(ffns)
    x = bits_to_dev(W.gaussian(m, W.D_MODEL, seed=7))
    buf = x.clone()
    g = stack.graphed(buf)
    assert torch.equal(g(), stack(x))
    x2 = bits_to_dev(W.student_t(m, W.D_MODEL, seed=8))
    buf.copy_(x2)
    got = g()
    assert torch.equal(got, stack(x2))
    assert g() is got                     # the same output tensor, overwritten per replay
    assert ops.read_device_error() == 0
