"""The reference-facing Python API on CPU: installer semantics and error
behaviour (ffn_quantization.py:35-86), and that nothing falls back to a CPU path."""
import pytest
import torch

import flashvsr_optimizations_b200 as fvq
from flashvsr_optimizations_b200 import ops
from flashvsr_optimizations_b200.ffn_quantization import QuantLinear, install_ffn


class _Block(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.ffn = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(approximate="tanh"),
                                       torch.nn.Linear(512, 256))


class _Pipe:
    def __init__(self, n=3):
        self.dit = torch.nn.Module()
        self.dit.blocks = torch.nn.ModuleList([_Block() for _ in range(n)])


def test_install_bf16_is_a_no_op_with_reference_metadata():
    pipe = _Pipe()
    meta = install_ffn(pipe, "bf16")
    assert meta["mode"] == "bf16" and meta["quantized_linears"] == 0
    assert meta["ffn_bytes_before"] == meta["ffn_bytes_after"] == 3 * (256 * 512 * 2 + 512 + 256) * 4
    for key in ("mode", "quantized_linears", "ffn_bytes_before", "ffn_bytes_after", "fp8", "nvfp4", "scope"):
        assert key in meta
    assert isinstance(pipe.dit.blocks[0].ffn[0], torch.nn.Linear)


def test_unknown_mode_raises_value_error():
    with pytest.raises(ValueError):
        QuantLinear(torch.nn.Linear(256, 256), "int3")


def test_fp8_on_cpu_weights_raises_instead_of_falling_back():
    with pytest.raises(RuntimeError):
        QuantLinear(torch.nn.Linear(256, 256), "fp8")
    with pytest.raises(RuntimeError):
        install_ffn(_Pipe(), "fp8")


def test_nvfp4_on_cpu_weights_raises_instead_of_falling_back():
    with pytest.raises(RuntimeError):
        install_ffn(_Pipe(), "nvfp4")


def test_ops_reject_cpu_tensors():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.global_scale(x)
    with pytest.raises(RuntimeError):
        ops.nvfp4_quantize(x, torch.ones(1))
    with pytest.raises(RuntimeError):
        ops.fp8_row_quant(x)
    with pytest.raises(RuntimeError):
        ops.fp8_quantize_activation(x)


def test_custom_ops_registered_with_fake_kernels():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(300, 1536, dtype=torch.bfloat16, device="cuda" if False else "cpu")
        q, s = torch.ops.fvq.nvfp4_quantize(x, torch.empty(1))
        assert q.shape == (300, 768) and s.shape == (384, 96)
        y = torch.ops.fvq.nvfp4_ffn(x, torch.empty(8960, 768, dtype=torch.uint8),
                                    torch.empty(8960, 96, dtype=torch.uint8), torch.empty(1), None,
                                    torch.empty(1536, 4480, dtype=torch.uint8),
                                    torch.empty(1536, 560, dtype=torch.uint8), torch.empty(1), None)
        assert y.shape == (300, 1536) and y.dtype == torch.bfloat16


def test_fp8_custom_ops_have_fake_kernels():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(300, 1536, dtype=torch.bfloat16)
        q, s = torch.ops.fvq.fp8_row_quant(x)
        assert q.shape == (300, 1536) and q.dtype == torch.float8_e4m3fn and s.shape == (300, 1)
        y = torch.ops.fvq.fp8_ffn(x, torch.empty(8960, 1536, dtype=torch.float8_e4m3fn),
                                  torch.empty(8960, 1), None,
                                  torch.empty(1536, 8960, dtype=torch.float8_e4m3fn),
                                  torch.empty(1536, 1), None)
        assert y.shape == (300, 1536) and y.dtype == torch.bfloat16
        z = torch.empty(2, 16, 8, 8, dtype=torch.bfloat16).to(memory_format=torch.channels_last)
        qz, sz = torch.ops.fvq.fp8_quantize_activation(z)
        assert qz.shape == z.shape and qz.stride() == z.stride() and sz.shape == (1,)


def test_graphed_stack_rejects_host_and_non_bf16_buffers():
    """GraphedFFNStack captures over a CUDA bf16 buffer only; there is no host path."""
    stack = fvq.NVFP4FFNStack([])
    with pytest.raises(ValueError):
        fvq.GraphedFFNStack(stack, torch.zeros(4, 8, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        stack.graphed(torch.zeros(4, 8))
