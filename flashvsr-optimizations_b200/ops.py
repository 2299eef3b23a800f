"""torch-facing NVFP4 and FP8 operators over the C ABI (libfvq.so).

Each function mirrors one call of the reference path and is registered as a
``torch.library`` custom op (namespace ``fvq``) with a fake implementation, so
it can sit inside traced / compiled graphs.  All work runs on the current
CUDA stream of the input's device; no host synchronisation happens.  There is
no CPU fallback: a non-CUDA tensor raises.

Layouts are the reference's (flashinfer's): codes uint8 [rows, k/2]; scale
factors uint8 [pad128(rows), k/16] in the 128x4 swizzled order; global scales
fp32 [1] on the device.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

__all__ = [
    "amax", "global_scale", "nvfp4_quantize", "nvfp4_quantize_from_amax", "mm_fp4", "nvfp4_gemm",
    "nvfp4_linear", "nvfp4_ffn", "rcp_approx_probe", "sf_rows", "read_device_error",
    "fp8_row_quant", "fp8_quantize_activation", "fp8_scaled_mm", "fp8_linear", "fp8_ffn",
    "div_full_probe", "ln_modulate", "nvfp4_ffn_block",
]


def sf_rows(rows: int) -> int:
    return (rows + 127) // 128 * 128


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(name: str, *ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name}: expected CUDA tensors (there is no CPU path)")


def _check_bf16(name: str, x: torch.Tensor) -> None:
    if x.dtype != torch.bfloat16:
        raise TypeError(f"{name}: expected bfloat16 input, got {x.dtype}")


def _aligned32(x: torch.Tensor) -> torch.Tensor:
    """The quantizer reads its bf16 input in 32-byte vectors: re-home a
    contiguous tensor whose storage offset breaks that alignment."""
    x = x.contiguous()
    return x if x.data_ptr() % 32 == 0 else x.clone()


# ---------------------------------------------------------------- workspaces
class _Workspaces:
    """Zero-initialised scratch buffers, one per (device, stream), grown on demand.

    The amax counter region of a workspace must start at zero and every call
    leaves it zero again, so a buffer is zeroed only when it is created.
    """

    def __init__(self):
        self._lock = threading.Lock()
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(),
               torch.cuda.current_stream(device).cuda_stream)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


_WS = _Workspaces()
# Scratch with no zero-state protocol (the FP8 linear and FFN carve their
# intermediates from it); kept apart from _WS, whose leading amax counters the
# NVFP4 calls rely on staying zero.
_SCRATCH = _Workspaces()


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    return _WS.get(device, nbytes)


def scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    return _SCRATCH.get(device, nbytes)


# ---------------------------------------------------------------- custom ops
@torch.library.custom_op("fvq::amax", mutates_args=())
def amax(x: torch.Tensor) -> torch.Tensor:
    """max |x| (fp32 [1]) of a bf16 tensor."""
    _check_cuda("amax", x)
    _check_bf16("amax", x)
    x = x.contiguous()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_amax_workspace_bytes())
    _lib.call("fvq_amax", _ptr(x), x.numel(), _ptr(out), None, _ptr(ws), ws.numel(), _stream(x))
    return out


@amax.register_fake
def _(x):
    return x.new_empty(1, dtype=torch.float32)


@torch.library.custom_op("fvq::global_scale", mutates_args=())
def global_scale(x: torch.Tensor) -> torch.Tensor:
    """``2688 / max(amax(x), 1e-12)`` as fp32 [1] -- ffn_quantization.py:29-32."""
    _check_cuda("global_scale", x)
    _check_bf16("global_scale", x)
    if x.numel() == 0:
        raise RuntimeError("global_scale: empty tensor (the reference's amax of no partials fails)")
    x = x.contiguous()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_amax_workspace_bytes())
    _lib.call("fvq_amax", _ptr(x), x.numel(), None, _ptr(out), _ptr(ws), ws.numel(), _stream(x))
    return out


@global_scale.register_fake
def _(x):
    return x.new_empty(1, dtype=torch.float32)


@torch.library.custom_op("fvq::nvfp4_quantize", mutates_args=())
def nvfp4_quantize(x: torch.Tensor, g: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(codes uint8 [M, K/2], scales uint8 [pad128(M), K/16]) -- flashinfer.nvfp4_quantize(x, g)."""
    _check_cuda("nvfp4_quantize", x, g)
    _check_bf16("nvfp4_quantize", x)
    if x.dim() != 2:
        raise ValueError("nvfp4_quantize: expected a 2-D [M, K] tensor")
    m, k = x.shape
    x = _aligned32(x)
    g = g.to(torch.float32).contiguous()
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
    sf = torch.empty((sf_rows(m), k // 16), dtype=torch.uint8, device=x.device)
    _lib.call("fvq_nvfp4_quantize", _ptr(x), m, k, _ptr(g), _ptr(codes), _ptr(sf), _stream(x))
    return codes, sf


@nvfp4_quantize.register_fake
def _(x, g):
    m, k = x.shape
    return (x.new_empty((m, k // 2), dtype=torch.uint8),
            x.new_empty((sf_rows(m), k // 16), dtype=torch.uint8))


@torch.library.custom_op("fvq::nvfp4_quantize_from_amax", mutates_args=())
def nvfp4_quantize_from_amax(x: torch.Tensor, amax: torch.Tensor
                             ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(codes, scales, g) with g = 2688 / max(amax, 1e-12) from a given max |x| (e.g. one
    all-reduced over ranks): ``nvfp4_quantize(x, global_scale(...))`` with the amax supplied."""
    _check_cuda("nvfp4_quantize_from_amax", x, amax)
    _check_bf16("nvfp4_quantize_from_amax", x)
    if x.dim() != 2:
        raise ValueError("nvfp4_quantize_from_amax: expected a 2-D [M, K] tensor")
    m, k = x.shape
    x = _aligned32(x)
    a = amax.to(torch.float32).reshape(1).contiguous()
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
    sf = torch.empty((sf_rows(m), k // 16), dtype=torch.uint8, device=x.device)
    g = torch.empty(1, dtype=torch.float32, device=x.device)
    _lib.call("fvq_nvfp4_quantize_dynamic", _ptr(x), m, k, _ptr(a), _ptr(g), _ptr(codes), _ptr(sf),
              None, 0, _stream(x))
    return codes, sf, g


@nvfp4_quantize_from_amax.register_fake
def _(x, amax):
    m, k = x.shape
    return (x.new_empty((m, k // 2), dtype=torch.uint8),
            x.new_empty((sf_rows(m), k // 16), dtype=torch.uint8),
            x.new_empty(1, dtype=torch.float32))


@torch.library.custom_op("fvq::mm_fp4", mutates_args=())
def mm_fp4(a: torch.Tensor, a_sf: torch.Tensor, w: torch.Tensor, w_sf: torch.Tensor,
           alpha: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(alpha * A @ W^T) [+ bias], operands in NVFP4.

    The reference passes ``qweight.t()`` / ``scale.t()`` to flashinfer.mm_fp4
    (ffn_quantization.py:65-67); here W is given in its stored [N, K/2] layout.
    """
    _check_cuda("mm_fp4", a, a_sf, w, w_sf, alpha, bias)
    m, kh = a.shape
    n = w.shape[0]
    if w.shape[1] != kh:
        raise ValueError(f"mm_fp4: K mismatch ({2 * kh} vs {2 * w.shape[1]})")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    _lib.call("fvq_nvfp4_mm", _ptr(a.contiguous()), _ptr(a_sf.contiguous()), _ptr(w.contiguous()),
              _ptr(w_sf.contiguous()), _ptr(alpha.to(torch.float32).contiguous()),
              _ptr(None if bias is None else bias.contiguous()), _ptr(out), m, n, 2 * kh,
              _stream(a))
    return out


@mm_fp4.register_fake
def _(a, a_sf, w, w_sf, alpha, bias=None):
    return a.new_empty((a.shape[0], w.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("fvq::nvfp4_gemm", mutates_args=())
def nvfp4_gemm(a: torch.Tensor, a_sf: torch.Tensor, g_a: torch.Tensor, w: torch.Tensor,
               w_sf: torch.Tensor, g_w: torch.Tensor, bias: torch.Tensor | None = None,
               gelu: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """GEMM with alpha = 1/(g_a*g_w); with gelu=True also GELU-tanh and amax of the result."""
    _check_cuda("nvfp4_gemm", a, a_sf, g_a, w, w_sf, g_w, bias)
    m, kh = a.shape
    n = w.shape[0]
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    amax_out = torch.zeros(1, dtype=torch.float32, device=a.device)
    _lib.call("fvq_nvfp4_gemm", _ptr(a.contiguous()), _ptr(a_sf.contiguous()), _ptr(g_a),
              _ptr(w.contiguous()), _ptr(w_sf.contiguous()), _ptr(g_w),
              _ptr(None if bias is None else bias.contiguous()), _ptr(out), m, n, 2 * kh,
              _lib.EPI_GELU_AMAX if gelu else _lib.EPI_BF16, _ptr(amax_out) if gelu else None,
              _stream(a))
    return out, amax_out


@nvfp4_gemm.register_fake
def _(a, a_sf, g_a, w, w_sf, g_w, bias=None, gelu=False):
    return (a.new_empty((a.shape[0], w.shape[0]), dtype=torch.bfloat16),
            a.new_empty(1, dtype=torch.float32))


def _linear_struct(qweight, scale, global_sf, bias, in_f, out_f) -> _lib.FvqLinear:
    return _lib.FvqLinear(_ptr(qweight), _ptr(scale), _ptr(global_sf), _ptr(bias), in_f, out_f)


@torch.library.custom_op("fvq::nvfp4_linear", mutates_args=())
def nvfp4_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor,
                 global_sf: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """QuantLinear.forward (ffn_quantization.py:54-70) on a 2-D bf16 input."""
    _check_cuda("nvfp4_linear", x, qweight, scale, global_sf, bias)
    _check_bf16("nvfp4_linear", x)
    m, k = x.shape
    n = qweight.shape[0]
    if m == 0:
        raise RuntimeError("nvfp4_linear: empty input (the reference's global_scale fails on it)")
    x = _aligned32(x)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_nvfp4_linear_workspace_bytes(m, k))
    lin = _linear_struct(qweight, scale, global_sf, bias, k, n)
    _lib.call("fvq_nvfp4_linear", _ptr(x), m, ctypes.byref(lin), _ptr(y), _ptr(ws), ws.numel(),
              _stream(x))
    return y


@nvfp4_linear.register_fake
def _(x, qweight, scale, global_sf, bias=None):
    return x.new_empty((x.shape[0], qweight.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("fvq::nvfp4_ffn", mutates_args=())
def nvfp4_ffn(x: torch.Tensor, q1: torch.Tensor, s1: torch.Tensor, g1: torch.Tensor,
              b1: torch.Tensor | None, q2: torch.Tensor, s2: torch.Tensor, g2: torch.Tensor,
              b2: torch.Tensor | None) -> torch.Tensor:
    """QuantLinear -> GELU-tanh -> QuantLinear on a 2-D bf16 input, as the reference computes it."""
    _check_cuda("nvfp4_ffn", x, q1, s1, g1, b1, q2, s2, g2, b2)
    _check_bf16("nvfp4_ffn", x)
    m, d = x.shape
    f = q1.shape[0]
    if m == 0:
        raise RuntimeError("nvfp4_ffn: empty input (the reference's global_scale fails on it)")
    x = _aligned32(x)
    y = torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_nvfp4_ffn_workspace_bytes(m, d, f))
    l1 = _linear_struct(q1, s1, g1, b1, d, f)
    l2 = _linear_struct(q2, s2, g2, b2, f, d)
    _lib.call("fvq_nvfp4_ffn", _ptr(x), m, ctypes.byref(l1), ctypes.byref(l2), _ptr(y), _ptr(ws),
              ws.numel(), _stream(x))
    return y


@nvfp4_ffn.register_fake
def _(x, q1, s1, g1, b1, q2, s2, g2, b2):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


@torch.library.custom_op("fvq::nvfp4_ffn_chain", mutates_args=())
def nvfp4_ffn_chain(x: torch.Tensor, q1: torch.Tensor, s1: torch.Tensor, g1: torch.Tensor,
                    b1: torch.Tensor | None, q2: torch.Tensor, s2: torch.Tensor, g2: torch.Tensor,
                    b2: torch.Tensor | None, x_amax: torch.Tensor | None = None
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """nvfp4_ffn for FFNs that feed each other directly (fvq_nvfp4_ffn_chain): returns
    (y, max |y|), and takes max |x| from the previous call when given, so that x is
    quantized without its own amax pass.  y equals nvfp4_ffn(x, ...) bit for bit."""
    _check_cuda("nvfp4_ffn_chain", x, q1, s1, g1, b1, q2, s2, g2, b2, x_amax)
    _check_bf16("nvfp4_ffn_chain", x)
    m, d = x.shape
    f = q1.shape[0]
    if m == 0:
        raise RuntimeError("nvfp4_ffn_chain: empty input (the reference's global_scale fails on it)")
    x = _aligned32(x)
    y = torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
    y_amax = torch.empty(1, dtype=torch.float32, device=x.device)
    if x_amax is not None:
        x_amax = x_amax.to(torch.float32).reshape(1).contiguous()
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_nvfp4_ffn_workspace_bytes(m, d, f))
    l1 = _linear_struct(q1, s1, g1, b1, d, f)
    l2 = _linear_struct(q2, s2, g2, b2, f, d)
    _lib.call("fvq_nvfp4_ffn_chain", _ptr(x), m, ctypes.byref(l1), ctypes.byref(l2), _ptr(y),
              _ptr(x_amax), _ptr(y_amax), _ptr(ws), ws.numel(), _stream(x))
    return y, y_amax


@nvfp4_ffn_chain.register_fake
def _(x, q1, s1, g1, b1, q2, s2, g2, b2, x_amax=None):
    return x.new_empty(x.shape, dtype=torch.bfloat16), x.new_empty(1, dtype=torch.float32)


@torch.library.custom_op("fvq::nvfp4_ffn_fused", mutates_args=("amax_seen", "flags"))
def nvfp4_ffn_fused(x: torch.Tensor, q1: torch.Tensor, s1: torch.Tensor, g1: torch.Tensor,
                    b1: torch.Tensor | None, q2: torch.Tensor, s2: torch.Tensor, g2: torch.Tensor,
                    b2: torch.Tensor | None, amax_hint: torch.Tensor, headroom_log2: int,
                    amax_seen: torch.Tensor, flags: torch.Tensor) -> torch.Tensor:
    """The FFN with the intermediate quantized inside GEMM1's epilogue (fvq_nvfp4_ffn_fused):
    h never reaches HBM in bf16; its encode scale is 2^-headroom_log2 * 2688 / amax_hint
    instead of 2688 / amax(h).  amax_seen (fp32 [1]) receives max |h|; flags (int32 [1]) is
    OR-ed with 1 when a block's scale saturated and 2 when a nonzero block's scale
    underflowed to zero."""
    _check_cuda("nvfp4_ffn_fused", x, q1, s1, g1, b1, q2, s2, g2, b2, amax_hint, amax_seen, flags)
    _check_bf16("nvfp4_ffn_fused", x)
    m, d = x.shape
    f = q1.shape[0]
    if m == 0:
        raise RuntimeError("nvfp4_ffn_fused: empty input")
    if amax_hint.dtype != torch.float32 or amax_seen.dtype != torch.float32 or \
            flags.dtype != torch.int32:
        raise ValueError("nvfp4_ffn_fused: amax_hint / amax_seen fp32, flags int32")
    x = _aligned32(x)
    y = torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_nvfp4_ffn_fused_workspace_bytes(m, d, f))
    l1 = _linear_struct(q1, s1, g1, b1, d, f)
    l2 = _linear_struct(q2, s2, g2, b2, f, d)
    _lib.call("fvq_nvfp4_ffn_fused", _ptr(x), m, ctypes.byref(l1), ctypes.byref(l2), _ptr(y),
              _ptr(amax_hint), int(headroom_log2), _ptr(amax_seen), _ptr(flags), _ptr(ws),
              ws.numel(), _stream(x))
    return y


@nvfp4_ffn_fused.register_fake
def _(x, q1, s1, g1, b1, q2, s2, g2, b2, amax_hint, headroom_log2, amax_seen, flags):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


# ---------------------------------------------------------------- the DiT block around the FFN
def _vec(name: str, v: torch.Tensor, d: int) -> torch.Tensor:
    v = v.reshape(-1)
    if v.numel() != d or v.dtype != torch.bfloat16:
        raise ValueError(f"{name}: expected a bf16 vector of {d} values")
    return _aligned16(v)


@torch.library.custom_op("fvq::ln_modulate", mutates_args=())
def ln_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                eps: float = 1e-6) -> torch.Tensor:
    """bf16(bf16(LN(x) * bf16(1 + scale)) + shift): the adaLN-modulated FFN input (LN without affine)."""
    _check_cuda("ln_modulate", x, shift, scale)
    _check_bf16("ln_modulate", x)
    m, d = x.shape
    x = _aligned16(x)
    u = torch.empty_like(x)
    if m:
        _lib.call("fvq_ln_modulate", _ptr(x), m, d, _ptr(_vec("shift", shift, d)),
                  _ptr(_vec("scale", scale, d)), float(eps), _ptr(u), _stream(x))
    return u


@ln_modulate.register_fake
def _(x, shift, scale, eps=1e-6):
    return torch.empty_like(x)


@torch.library.custom_op("fvq::nvfp4_ffn_block", mutates_args=())
def nvfp4_ffn_block(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, gate: torch.Tensor,
                    eps: float, q1: torch.Tensor, s1: torch.Tensor, g1: torch.Tensor,
                    b1: torch.Tensor | None, q2: torch.Tensor, s2: torch.Tensor, g2: torch.Tensor,
                    b2: torch.Tensor | None) -> torch.Tensor:
    """x + gate * FFN(LN(x) * (1 + scale) + shift), bf16 steps, the gated residual fused
    into the second GEMM (fvq_nvfp4_ffn_block)."""
    _check_cuda("nvfp4_ffn_block", x, shift, scale, gate, q1, s1, g1, b1, q2, s2, g2, b2)
    _check_bf16("nvfp4_ffn_block", x)
    m, d = x.shape
    f = q1.shape[0]
    if m == 0:
        return x.new_empty((0, d))
    x = _aligned16(x)
    out = torch.empty_like(x)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_nvfp4_ffn_block_workspace_bytes(m, d, f))
    l1 = _linear_struct(q1, s1, g1, b1, d, f)
    l2 = _linear_struct(q2, s2, g2, b2, f, d)
    _lib.call("fvq_nvfp4_ffn_block", _ptr(x), m, _ptr(_vec("shift", shift, d)),
              _ptr(_vec("scale", scale, d)), _ptr(_vec("gate", gate, d)), float(eps),
              ctypes.byref(l1), ctypes.byref(l2), _ptr(out), _ptr(ws), ws.numel(), _stream(x))
    return out


@nvfp4_ffn_block.register_fake
def _(x, shift, scale, gate, eps, q1, s1, g1, b1, q2, s2, g2, b2):
    return torch.empty_like(x)


# ---------------------------------------------------------------- FP8 (W8A8) mode
def _check_fp8(name: str, *ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.float8_e4m3fn:
            raise TypeError(f"{name}: expected float8_e4m3fn codes, got {t.dtype}")


def _dense(x: torch.Tensor) -> bool:
    """True when x's elements fill its storage span without gaps or overlaps
    (any permutation of a contiguous layout, channels_last included), so
    empty_like(x) has the same strides and both can be walked in memory order."""
    if x.is_contiguous():
        return True
    dims = sorted((st, sz) for st, sz in zip(x.stride(), x.shape) if sz != 1)
    expect = 1
    for st, sz in dims:
        if st != expect:
            return False
        expect *= sz
    return True


def _aligned16(x: torch.Tensor) -> torch.Tensor:
    x = x.contiguous()
    return x if x.data_ptr() % 16 == 0 else x.clone()


@torch.library.custom_op("fvq::fp8_row_quant", mutates_args=())
def fp8_row_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q float8_e4m3fn [M, K], scale fp32 [M, 1]) -- the reference's row_quant
    (ffn_quantization.py:22-26): scale = max(max|x_row| / 448, 1e-12), q = x / scale."""
    _check_cuda("fp8_row_quant", x)
    _check_bf16("fp8_row_quant", x)
    if x.dim() != 2:
        raise ValueError("fp8_row_quant: expected a 2-D [M, K] tensor")
    m, k = x.shape
    x = _aligned16(x)
    q = torch.empty((m, k), dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if m > 0:
        _lib.call("fvq_fp8_row_quantize", _ptr(x), m, k, _ptr(q), _ptr(scale), _stream(x))
    return q, scale


@fp8_row_quant.register_fake
def _(x):
    m, k = x.shape
    return (x.new_empty((m, k), dtype=torch.float8_e4m3fn),
            x.new_empty((m, 1), dtype=torch.float32))


@torch.library.custom_op("fvq::fp8_quantize_activation", mutates_args=())
def fp8_quantize_activation(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q float8_e4m3fn like x, scale fp32 [1]) with one scale for the whole tensor --
    decoder_fp8.py:17-24 (and lq_fp8.py:24-31): scale = max(amax / 448, 1e-12),
    q = clamp(x / scale, -448, 448).  x may be in any dense memory format
    (channels_last included); q keeps it."""
    _check_cuda("fp8_quantize_activation", x)
    _check_bf16("fp8_quantize_activation", x)
    if x.numel() == 0:
        raise RuntimeError("fp8_quantize_activation: empty tensor (the reference's amax of no "
                           "partials fails)")
    if not _dense(x):
        x = x.contiguous()
    q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    if x.data_ptr() % 16 != 0 or q.data_ptr() % 8 != 0:
        x = x.clone()
        q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws = workspace(x.device, lib.fvq_fp8_tensor_quantize_workspace_bytes())
    _lib.call("fvq_fp8_tensor_quantize", _ptr(x), x.numel(), _ptr(q), _ptr(scale), _ptr(ws),
              ws.numel(), _stream(x))
    return q, scale


@fp8_quantize_activation.register_fake
def _(x):
    return torch.empty_like(x, dtype=torch.float8_e4m3fn), x.new_empty(1, dtype=torch.float32)


@torch.library.custom_op("fvq::fp8_scaled_mm", mutates_args=())
def fp8_scaled_mm(a: torch.Tensor, scale_a: torch.Tensor, w: torch.Tensor, scale_w: torch.Tensor,
                  bias: torch.Tensor | None = None) -> torch.Tensor:
    """bf16((A @ W^T) * scale_a * scale_w) [+ bias] with E4M3 operands.

    The reference calls ``torch._scaled_mm(q, qweight.t(), scale_a=s,
    scale_b=scale.t(), out_dtype=bf16, use_fast_accum=False)``
    (ffn_quantization.py:58-60); here W is given in its stored [N, K] layout and
    the scales as [M, 1] / [N, 1] (or flat)."""
    _check_cuda("fp8_scaled_mm", a, scale_a, w, scale_w, bias)
    _check_fp8("fp8_scaled_mm", a, w)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"fp8_scaled_mm: K mismatch ({k} vs {w.shape[1]})")
    sa = scale_a.to(torch.float32).reshape(-1).contiguous()
    sw = _aligned16(scale_w.to(torch.float32).reshape(-1))
    if sa.numel() != m or sw.numel() != n:
        raise ValueError("fp8_scaled_mm: expected one scale per row of A and per row of W")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    _lib.call("fvq_fp8_scaled_mm", _ptr(_aligned16(a)), _ptr(sa), _ptr(_aligned16(w)), _ptr(sw),
              _ptr(None if bias is None else _aligned16(bias)), _ptr(out), m, n, k, _stream(a))
    return out


@fp8_scaled_mm.register_fake
def _(a, scale_a, w, scale_w, bias=None):
    return a.new_empty((a.shape[0], w.shape[0]), dtype=torch.bfloat16)


def _fp8_linear_struct(qweight, scale, bias, in_f, out_f) -> _lib.FvqLinearFp8:
    return _lib.FvqLinearFp8(_ptr(qweight), _ptr(scale), _ptr(bias), in_f, out_f)


def _fp8_weight_args(name, qweight, scale, bias):
    _check_fp8(name, qweight)
    return (_aligned16(qweight), _aligned16(scale.to(torch.float32).reshape(-1)),
            None if bias is None else _aligned16(bias))


@torch.library.custom_op("fvq::fp8_linear", mutates_args=())
def fp8_linear(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor,
               bias: torch.Tensor | None = None) -> torch.Tensor:
    """QuantLinear.forward in mode 'fp8' (ffn_quantization.py:54-60, :68-70) on a 2-D bf16 input."""
    _check_cuda("fp8_linear", x, qweight, scale, bias)
    _check_bf16("fp8_linear", x)
    m, k = x.shape
    n = qweight.shape[0]
    if m == 0:
        return x.new_empty((0, n))
    x = _aligned16(x)
    qweight, scale, bias = _fp8_weight_args("fp8_linear", qweight, scale, bias)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = scratch(x.device, lib.fvq_fp8_linear_workspace_bytes(m, k))
    lin = _fp8_linear_struct(qweight, scale, bias, k, n)
    _lib.call("fvq_fp8_linear", _ptr(x), m, ctypes.byref(lin), _ptr(y), _ptr(ws), ws.numel(),
              _stream(x))
    return y


@fp8_linear.register_fake
def _(x, qweight, scale, bias=None):
    return x.new_empty((x.shape[0], qweight.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("fvq::fp8_ffn", mutates_args=())
def fp8_ffn(x: torch.Tensor, q1: torch.Tensor, s1: torch.Tensor, b1: torch.Tensor | None,
            q2: torch.Tensor, s2: torch.Tensor, b2: torch.Tensor | None) -> torch.Tensor:
    """Linear -> GELU-tanh -> Linear in mode 'fp8', as the reference's QuantLinear modules compute it."""
    _check_cuda("fp8_ffn", x, q1, s1, b1, q2, s2, b2)
    _check_bf16("fp8_ffn", x)
    m, d = x.shape
    f = q1.shape[0]
    if m == 0:
        return x.new_empty((0, d))
    x = _aligned16(x)
    q1, s1, b1 = _fp8_weight_args("fp8_ffn", q1, s1, b1)
    q2, s2, b2 = _fp8_weight_args("fp8_ffn", q2, s2, b2)
    y = torch.empty((m, d), dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    ws = scratch(x.device, lib.fvq_fp8_ffn_workspace_bytes(m, d, f))
    l1 = _fp8_linear_struct(q1, s1, b1, d, f)
    l2 = _fp8_linear_struct(q2, s2, b2, f, d)
    _lib.call("fvq_fp8_ffn", _ptr(x), m, ctypes.byref(l1), ctypes.byref(l2), _ptr(y), _ptr(ws),
              ws.numel(), _stream(x))
    return y


@fp8_ffn.register_fake
def _(x, q1, s1, b1, q2, s2, b2):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


def div_full_probe(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """div.full.f32(a, b) elementwise on the GPU, the FP8 quantizers' division (test support)."""
    _check_cuda("div_full_probe", a, b)
    a = a.to(torch.float32).contiguous()
    b = b.to(torch.float32).expand_as(a).contiguous()
    out = torch.empty_like(a)
    _lib.call("fvq_div_full_probe", _ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(a))
    return out


# ---------------------------------------------------------------- support
def rcp_approx_probe(values: torch.Tensor) -> torch.Tensor:
    """rcp.approx.ftz.f32 of each fp32 value, computed on the GPU (test support)."""
    _check_cuda("rcp_approx_probe", values)
    v = values.to(torch.float32).contiguous()
    out = torch.empty_like(v)
    _lib.call("fvq_rcp_approx_probe", _ptr(v), _ptr(out), v.numel(), _stream(v))
    return out


def read_device_error(device: torch.device | None = None) -> int:
    """Synchronise and return (and clear) the library's device error word."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    flags = ctypes.c_uint32(0)
    _lib.call("fvq_read_device_error", torch.cuda.current_stream(dev).cuda_stream,
              ctypes.byref(flags))
    return int(flags.value)


def set_wait_limit(nanoseconds: int) -> None:
    """Bound (wall time per wait) on the GEMM's pipeline waits; 0 restores the 2 s default."""
    _lib.call("fvq_set_wait_limit", nanoseconds)
