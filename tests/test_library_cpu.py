"""The C-ABI library on a machine without a GPU: it loads, exports every entry
point include/fvq.h declares, and its host-side checks reject bad arguments
with the documented status codes before any device work."""
import ctypes
import re

import pytest

from conftest import ROOT
from flashvsr_optimizations_b200 import _lib


def _declared():
    text = (ROOT / "include" / "fvq.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(fvq_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with include/fvq.h"


def test_version_and_workspace_sizes():
    lib = _lib.load()
    assert lib.fvq_version() == 100
    assert lib.fvq_amax_workspace_bytes() >= 64 + 4 * 148 * 8
    ws = lib.fvq_nvfp4_ffn_workspace_bytes(7680, 1536, 8960)
    # codes + scales of x, bf16 intermediate, codes + scales of the intermediate,
    # W2 scales replicated four times
    need = (7680 * 768 + 7680 * 96 + 7680 * 8960 * 2 + 7680 * 4480 + 7680 * 560
            + 4 * 1536 * 8960 // 16)
    assert need <= ws <= need + 64 * 1024
    assert lib.fvq_nvfp4_ffn_workspace_bytes(0, 1536, 8960) == 0
    assert lib.fvq_w_scales_replicated_bytes(1536, 8960) == 4 * 1536 * 8960 // 16
    assert lib.fvq_w_scales_replicated_bytes(0, 8960) == 0


def _rc(name, *args):
    return getattr(_lib.load(), name)(*args)


def test_quantize_rejects_bad_shapes_and_alignment():
    buf = ctypes.create_string_buffer(4096 + 16)
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    assert _rc("fvq_nvfp4_quantize", base, 4, 100, base, base, base, None) == _lib.FVQ_EINVAL
    assert b"multiple of 64" in _lib.load().fvq_last_error()
    assert _rc("fvq_nvfp4_quantize", base, 0, 64, base, base, base, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_nvfp4_quantize", None, 4, 64, base, base, base, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_nvfp4_quantize", base + 2, 4, 64, base, base, base, None) == _lib.FVQ_EALIGN
    assert _rc("fvq_nvfp4_quantize", base + 16 if base % 32 == 0 else base, 4, 64, base, base, base, None) == _lib.FVQ_EALIGN


def test_gemm_rejects_bad_shapes_and_epilogue():
    buf = ctypes.create_string_buffer(4096 + 16)
    b = (ctypes.addressof(buf) + 15) // 16 * 16
    gemm = lambda m, n, k, epi=0, amax=None: _rc(  # noqa: E731
        "fvq_nvfp4_gemm", b, b, b, b, b, b, None, b, m, n, k, epi, amax, None)
    assert gemm(128, 200, 256) == _lib.FVQ_EINVAL
    assert gemm(128, 256, 100) == _lib.FVQ_EINVAL
    assert gemm(0, 256, 256) == _lib.FVQ_EINVAL
    assert gemm(128, 256, 256, epi=7) == _lib.FVQ_EINVAL
    assert gemm(128, 256, 256, epi=1, amax=None) == _lib.FVQ_EINVAL
    wrep = lambda m, n, k, ptr=b: _rc(  # noqa: E731
        "fvq_nvfp4_gemm_wrep", b, b, b, b, ptr, b, None, b, m, n, k, None)
    assert wrep(128, 200, 256) == _lib.FVQ_EINVAL
    assert wrep(128, 256, 100) == _lib.FVQ_EINVAL
    assert wrep(128, 256, 256, ptr=None) == _lib.FVQ_EINVAL
    assert wrep(128, 256, 256, ptr=b + 8) == _lib.FVQ_EALIGN
    assert _rc("fvq_replicate_w_scales", b, 300, 256, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_replicate_w_scales", b, 256, 320, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_replicate_w_scales", b, 256, 256, b + 4, None) == _lib.FVQ_EALIGN


def test_linear_and_ffn_check_descriptors():
    lin_bad = _lib.FvqLinear(None, None, None, None, 1536, 8960)
    assert _rc("fvq_nvfp4_linear", 16, 4, ctypes.byref(lin_bad), 16, 16, 1 << 20, None) == _lib.FVQ_EINVAL
    buf = ctypes.create_string_buffer(64)
    b = (ctypes.addressof(buf) + 15) // 16 * 16
    l1 = _lib.FvqLinear(b, b, b, None, 1536, 8960)
    l2 = _lib.FvqLinear(b, b, b, None, 8960, 1024)   # does not chain back to 1536
    assert _rc("fvq_nvfp4_ffn", b, 4, ctypes.byref(l1), ctypes.byref(l2), b, b, 1 << 30,
               None) == _lib.FVQ_EINVAL
    l2 = _lib.FvqLinear(b, b, b, None, 8960, 1536)
    assert _rc("fvq_nvfp4_ffn", b, 4, ctypes.byref(l1), ctypes.byref(l2), b, b, 16,
               None) == _lib.FVQ_EWORKSPACE


def test_block_entry_points_check_arguments():
    buf = ctypes.create_string_buffer(256)
    b = (ctypes.addressof(buf) + 31) // 32 * 32
    eps = ctypes.c_float(1e-6)
    assert _rc("fvq_ln_modulate", b, 4, 1532, b, b, eps, b, None) == _lib.FVQ_EINVAL   # d % 8
    assert _rc("fvq_ln_modulate", b, 4, 2056, b, b, eps, b, None) == _lib.FVQ_EINVAL   # d > 2048
    assert _rc("fvq_ln_modulate", b, 0, 1536, b, b, eps, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_ln_modulate", b, 4, 1536, b, b, ctypes.c_float(-1.0), b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_ln_modulate", b, 4, 1536, None, b, eps, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_ln_modulate", b + 8, 4, 1536, b, b, eps, b, None) == _lib.FVQ_EALIGN
    lib = _lib.load()
    need = lib.fvq_nvfp4_ffn_block_workspace_bytes(4, 1536, 8960)
    assert need >= lib.fvq_nvfp4_ffn_workspace_bytes(4, 1536, 8960) + 4 * 2 * 4   # + row statistics
    assert lib.fvq_nvfp4_ffn_block_workspace_bytes(0, 1536, 8960) == 0
    l1 = _lib.FvqLinear(b, b, b, None, 1536, 8960)
    l2 = _lib.FvqLinear(b, b, b, None, 8960, 1536)
    blk = lambda x=b, rows=4, l2=l2, ws=b, wsb=need, e=eps: _rc(  # noqa: E731
        "fvq_nvfp4_ffn_block", x, rows, b, b, b, e, ctypes.byref(l1), ctypes.byref(l2), b, ws, wsb,
        None)
    assert blk(l2=_lib.FvqLinear(b, b, b, None, 8960, 1024)) == _lib.FVQ_EINVAL
    assert blk(rows=0) == _lib.FVQ_EINVAL
    assert blk(x=None) == _lib.FVQ_EINVAL
    assert blk(e=ctypes.c_float(float("nan"))) == _lib.FVQ_EINVAL
    assert blk(wsb=need - 1) == _lib.FVQ_EWORKSPACE
    assert blk(x=b + 8) == _lib.FVQ_EALIGN
    assert blk(ws=b + 16) == _lib.FVQ_EALIGN


def test_pairing_modes_checked():
    assert _rc("fvq_set_gemm_pairing", 3) == _lib.FVQ_EINVAL
    assert _rc("fvq_set_gemm_pairing", -1) == _lib.FVQ_EINVAL
    assert _rc("fvq_set_gemm_pairing", 0) == _lib.FVQ_OK
    assert _rc("fvq_set_gemm_pairing", 1) == _lib.FVQ_OK   # back to the default


def test_valid_call_without_gpu_fails_loudly():
    """A well-formed call on a machine without a usable GPU returns an error, never computes on CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    buf = ctypes.create_string_buffer(4096 + 32)
    b = (ctypes.addressof(buf) + 31) // 32 * 32
    rc = _rc("fvq_nvfp4_quantize", b, 4, 64, b, b, b, None)
    assert rc in (_lib.FVQ_ECUDA, _lib.FVQ_EDEVICE)


def test_fp8_entry_points_check_arguments():
    lib = _lib.load()
    buf = ctypes.create_string_buffer(4096 + 32)
    b = (ctypes.addressof(buf) + 31) // 32 * 32
    # row quantizer: k a multiple of 8 up to 16384, 16-byte x and q
    assert _rc("fvq_fp8_row_quantize", b, 4, 100, b, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_fp8_row_quantize", b, 4, 16392, b, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_fp8_row_quantize", b, 0, 64, b, b, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_fp8_row_quantize", b + 8, 4, 64, b, b, None) == _lib.FVQ_EALIGN
    assert _rc("fvq_fp8_row_quantize", b, 4, 64, b, b + 2, None) == _lib.FVQ_EALIGN
    # tensor quantizer: workspace size, alignment
    wsb = lib.fvq_fp8_tensor_quantize_workspace_bytes()
    assert wsb >= lib.fvq_amax_workspace_bytes() + 4
    assert _rc("fvq_fp8_tensor_quantize", b, 100, b, b, b, wsb - 1, None) == _lib.FVQ_EWORKSPACE
    assert _rc("fvq_fp8_tensor_quantize", b, 0, b, b, b, wsb, None) == _lib.FVQ_EINVAL
    assert _rc("fvq_fp8_tensor_quantize", b, 100, b + 4, b, b, wsb, None) == _lib.FVQ_EALIGN
    # scaled_mm: n % 256, k % 128, 16-byte W scales
    mm = lambda m, n, k, sw=b: _rc("fvq_fp8_scaled_mm", b, b, b, sw, None, b, m, n, k, None)  # noqa: E731
    assert mm(128, 200, 256) == _lib.FVQ_EINVAL
    assert mm(128, 256, 192) == _lib.FVQ_EINVAL
    assert mm(0, 256, 256) == _lib.FVQ_EINVAL
    assert mm(128, 256, 256, sw=b + 4) == _lib.FVQ_EALIGN
    # linear / ffn descriptors and workspace sizes
    assert lib.fvq_fp8_linear_workspace_bytes(7680, 1536) >= 7680 * 1536 + 7680 * 4
    need = 7680 * 4 * 3 + 7680 * 1536 + 7680 * 8960 * 3
    assert need <= lib.fvq_fp8_ffn_workspace_bytes(7680, 1536, 8960) <= need + 4096
    bad = _lib.FvqLinearFp8(None, None, None, 1536, 8960)
    assert _rc("fvq_fp8_linear", b, 4, ctypes.byref(bad), b, b, 1 << 20, None) == _lib.FVQ_EINVAL
    l1 = _lib.FvqLinearFp8(b, b, None, 1536, 8960)
    l2 = _lib.FvqLinearFp8(b, b, None, 8960, 1024)
    assert _rc("fvq_fp8_ffn", b, 4, ctypes.byref(l1), ctypes.byref(l2), b, b, 1 << 30,
               None) == _lib.FVQ_EINVAL
    l2 = _lib.FvqLinearFp8(b, b, None, 8960, 1536)
    assert _rc("fvq_fp8_ffn", b, 4, ctypes.byref(l1), ctypes.byref(l2), b, b, 16,
               None) == _lib.FVQ_EWORKSPACE
