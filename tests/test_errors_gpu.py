"""Failure detection without faulting the GPU: every pipeline wait inside the
GEMM is bounded in wall time.  A wait limit of 1 ns makes the waits give up;
the kernel then drains its own copies and MMAs, frees TMEM, sets the device
error word and returns.  The host reads the word, and the context stays
usable for the next, normal launch."""
import numpy as np
import pytest
import torch

from flashvsr_optimizations_b200 import ops
from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu


def _operands(m, n, k, seed):
    rng = np.random.default_rng(seed)
    def op(rows):
        codes = rng.integers(0, 256, size=(rows, k // 2), dtype=np.uint8)
        sf = np.zeros(O.sf_swizzled_size(rows, k), dtype=np.uint8)
        sf[O.sf_swizzled_offsets(rows, k // 16)] = rng.integers(0x30, 0x40, size=(rows, k // 16),
                                                                 dtype=np.uint8)
        return torch.from_numpy(codes).cuda(), torch.from_numpy(sf).cuda()
    return op(m), op(n)


@pytest.mark.parametrize("gelu", [False, True])
def test_wait_timeout_sets_error_word_and_context_survives(gelu):
    (a, asf), (w, wsf) = _operands(512, 1024, 1536, seed=3)
    g = torch.ones(1, device="cuda")
    assert ops.read_device_error() == 0
    ref, _ = ops.nvfp4_gemm(a, asf, g, w, wsf, g, gelu=gelu)
    try:
        ops.set_wait_limit(1)                      # 1 ns: waits give up at once
        ops.nvfp4_gemm(a, asf, g, w, wsf, g, gelu=gelu)
        flags = ops.read_device_error()            # synchronises, returns and clears
    finally:
        ops.set_wait_limit(0)
    assert flags != 0
    assert ops.read_device_error() == 0
    again, _ = ops.nvfp4_gemm(a, asf, g, w, wsf, g, gelu=gelu)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)
    assert ops.read_device_error() == 0


def test_fused_quantizer_grid_wait_timeout_sets_error_word():
    """The fused amax+quantize kernel's grid barrier is bounded as well: with a
    1 ns limit the CTAs that wait give up (kErrWaitGrid, bit 5), the barrier is
    still re-armed by the last CTA to arrive, and the next call is exact."""
    from flashvsr_optimizations_b200 import _lib, workloads as W
    xb = W.gaussian(7680, 1536, seed=21)
    x = torch.from_numpy(xb.astype(np.int16)).view(torch.bfloat16).cuda()
    g_ref = ops.global_scale(x)
    q_ref, s_ref = ops.nvfp4_quantize(x, g_ref)
    lib = _lib.load()
    ws = torch.zeros(lib.fvq_amax_workspace_bytes(), dtype=torch.uint8, device="cuda")
    q, s = torch.empty_like(q_ref), torch.empty_like(s_ref)
    g = torch.empty(1, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    call = lambda: _lib.call("fvq_nvfp4_quantize_dynamic", x.data_ptr(), 7680, 1536, None,  # noqa: E731
                             g.data_ptr(), q.data_ptr(), s.data_ptr(), ws.data_ptr(), ws.numel(), st)
    assert ops.read_device_error() == 0
    try:
        ops.set_wait_limit(1)
        call()
        flags = ops.read_device_error()
    finally:
        ops.set_wait_limit(0)
    assert flags & (1 << 5), flags
    assert not ws[:4].any(), "the arrival counter is re-armed even after timeouts"
    call()
    torch.cuda.synchronize()
    assert ops.read_device_error() == 0
    assert g.item() == g_ref.item() and torch.equal(q, q_ref) and torch.equal(s, s_ref)
