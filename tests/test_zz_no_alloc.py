"""fvq_nvfp4_linear_noalloc: QuantLinear.forward without a caller workspace.

Some callers cannot allocate device memory where they run the layer (code
inside another runtime's memory arena, plugins given only input and output
buffers).  This entry point takes its scratch from a fixed array built into
the library.  Checked here through the C ABI against the regular entry point
(fvq_nvfp4_linear, caller workspace) on two calls in a row, with the GEMM
tests' tolerance (Frobenius-relative <= 2e-3; the arithmetic is the same, so
the results are expected to be identical), plus the size limit.
"""
import ctypes

import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import _lib, ops, workloads as W

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _bits_to_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def layer():
    wb, bb = W.linear_params(8960, 1536, seed=50, b_std=0.01)
    w = _bits_to_dev(wb)
    g = ops.global_scale(w)
    q, s = ops.nvfp4_quantize(w, g)
    b = _bits_to_dev(bb)
    lin = _lib.FvqLinear(q.data_ptr(), s.data_ptr(), g.data_ptr(), b.data_ptr(), 1536, 8960)
    return lin, (q, s, g, b)  # keep the buffers alive


def _regular(lib, x, lin):
    rows = x.shape[0]
    y = torch.empty(rows, 8960, dtype=torch.bfloat16, device="cuda")
    nbytes = lib.fvq_nvfp4_linear_workspace_bytes(rows, 1536)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    _lib.check("fvq_nvfp4_linear", lib.fvq_nvfp4_linear(
        x.data_ptr(), rows, ctypes.byref(lin), y.data_ptr(), ws.data_ptr(), nbytes,
        torch.cuda.current_stream().cuda_stream))
    return y


def _noalloc(lib, x, lin):
    rows = x.shape[0]
    y = torch.empty(rows, 8960, dtype=torch.bfloat16, device="cuda")
    _lib.check("fvq_nvfp4_linear_noalloc", lib.fvq_nvfp4_linear_noalloc(
        x.data_ptr(), rows, ctypes.byref(lin), y.data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    return y


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


def test_noalloc_matches_workspace_entry_point_twice(layer):
    lib = _lib.load()
    lin, _ = layer
    x1 = _bits_to_dev(W.student_t(2048, 1536, seed=51))
    x2 = _bits_to_dev(W.gaussian(777, 1536, seed=52))
    y1 = _noalloc(lib, x1, lin)
    y2 = _noalloc(lib, x2, lin)          # second call in a row reuses the same scratch
    r1 = _regular(lib, x1, lin)
    r2 = _regular(lib, x2, lin)
    torch.cuda.synchronize()
    assert _rel(y1, r1) <= TOL and _rel(y2, r2) <= TOL
    assert torch.equal(y1, r1) and torch.equal(y2, r2)


def test_noalloc_rejects_rows_beyond_its_scratch(layer):
    lib = _lib.load()
    lin, _ = layer
    cap = lib.fvq_noalloc_scratch_bytes()
    rows = 1
    while lib.fvq_nvfp4_linear_workspace_bytes(rows, 1536) <= cap:
        rows *= 2
    # no launch happens: the size check runs before any device work
    rc = lib.fvq_nvfp4_linear_noalloc(16, rows, ctypes.byref(lin), 16,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FVQ_EWORKSPACE
    assert b"fvq_nvfp4_linear_noalloc" in lib.fvq_last_error()


def test_noalloc_recovers_after_a_timed_out_call(layer):
    """The shared scratch array cannot be zeroed again by the caller, so a call
    whose bounded waits gave up (1 ns wait limit: the fused quantizer's grid
    barrier and the GEMM's pipeline waits) must still leave the array's amax
    counters re-armed: the error word reports the timeout and the next call,
    with the default limit, equals fvq_nvfp4_linear bit for bit."""
    lib = _lib.load()
    lin, _ = layer
    x = _bits_to_dev(W.gaussian(7680, 1536, seed=53))
    assert ops.read_device_error() == 0
    try:
        ops.set_wait_limit(1)
        _noalloc(lib, x, lin)
        flags = ops.read_device_error()            # synchronises, returns and clears
    finally:
        ops.set_wait_limit(0)
    assert flags != 0
    y = _noalloc(lib, x, lin)
    r = _regular(lib, x, lin)
    torch.cuda.synchronize()
    assert ops.read_device_error() == 0
    assert torch.equal(y, r)
