"""ctypes binding of libfvq.so (the C ABI declared in include/fvq.h).

The library is loaded lazily on first use.  There is no fallback: if the
library is missing or the device is not an sm_100 GPU, every entry point
raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libfvq.so"

FVQ_OK = 0
FVQ_EINVAL = -1
FVQ_EALIGN = -2
FVQ_ECUDA = -3
FVQ_EDEVICE = -4
FVQ_EWORKSPACE = -5
FVQ_ETIMEOUT = -6

EPI_BF16 = 0
EPI_GELU_AMAX = 1

_c = ctypes
_vp = _c.c_void_p
_i64 = _c.c_int64
_sz = _c.c_size_t


class FvqLinear(_c.Structure):
    """Mirror of ``struct fvq_linear``."""

    _fields_ = [
        ("qweight", _vp),
        ("scale", _vp),
        ("global_sf", _vp),
        ("bias", _vp),
        ("in_features", _i64),
        ("out_features", _i64),
    ]


class FvqLinearFp8(_c.Structure):
    """Mirror of ``struct fvq_linear_fp8``."""

    _fields_ = [
        ("qweight", _vp),
        ("scale", _vp),
        ("bias", _vp),
        ("in_features", _i64),
        ("out_features", _i64),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "fvq_version": (_c.c_int, []),
    "fvq_last_error": (_c.c_char_p, []),
    "fvq_amax_workspace_bytes": (_sz, []),
    "fvq_amax": (_c.c_int, [_vp, _i64, _vp, _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_quantize": (_c.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "fvq_nvfp4_quantize_dynamic": (_c.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_gemm": (_c.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                  _c.c_int, _vp, _vp]),
    "fvq_nvfp4_mm": (_c.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "fvq_w_scales_replicated_bytes": (_sz, [_i64, _i64]),
    "fvq_set_gemm_pairing": (_c.c_int, [_c.c_int]),
    "fvq_set_fp8_gemm_pairing": (_c.c_int, [_c.c_int]),
    "fvq_replicate_w_scales": (_c.c_int, [_vp, _i64, _i64, _vp, _vp]),
    "fvq_nvfp4_gemm_wrep": (_c.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                       _vp]),
    "fvq_nvfp4_linear_workspace_bytes": (_sz, [_i64, _i64]),
    "fvq_nvfp4_linear": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear), _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_linear_noalloc": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear), _vp, _vp]),
    "fvq_noalloc_scratch_bytes": (_sz, []),
    "fvq_nvfp4_ffn_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "fvq_nvfp4_ffn": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear), _c.POINTER(FvqLinear), _vp,
                                 _vp, _sz, _vp]),
    "fvq_nvfp4_ffn_chain": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear), _c.POINTER(FvqLinear),
                                       _vp, _vp, _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_ffn_block_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "fvq_ln_modulate": (_c.c_int, [_vp, _i64, _i64, _vp, _vp, _c.c_float, _vp, _vp]),
    "fvq_nvfp4_ffn_block": (_c.c_int, [_vp, _i64, _vp, _vp, _vp, _c.c_float, _c.POINTER(FvqLinear),
                                       _c.POINTER(FvqLinear), _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_ffn_profile": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear),
                                         _c.POINTER(FvqLinear), _vp, _vp, _sz, _vp,
                                         _c.POINTER(_c.c_float)]),
    "fvq_nvfp4_ffn_chain_profile": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear),
                                               _c.POINTER(FvqLinear), _vp, _vp, _vp, _vp, _sz, _vp,
                                               _c.POINTER(_c.c_float)]),
    "fvq_nvfp4_ffn_fused_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "fvq_nvfp4_ffn_fused": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear), _c.POINTER(FvqLinear),
                                       _vp, _vp, _c.c_int, _vp, _vp, _vp, _sz, _vp]),
    "fvq_nvfp4_ffn_fused_profile": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinear),
                                               _c.POINTER(FvqLinear), _vp, _vp, _c.c_int, _vp,
                                               _vp, _vp, _sz, _vp, _c.POINTER(_c.c_float)]),
    "fvq_fp8_row_quantize": (_c.c_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "fvq_fp8_tensor_quantize_workspace_bytes": (_sz, []),
    "fvq_fp8_tensor_quantize": (_c.c_int, [_vp, _i64, _vp, _vp, _vp, _sz, _vp]),
    "fvq_fp8_scaled_mm": (_c.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "fvq_fp8_linear_workspace_bytes": (_sz, [_i64, _i64]),
    "fvq_fp8_linear": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinearFp8), _vp, _vp, _sz, _vp]),
    "fvq_fp8_ffn_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "fvq_fp8_ffn": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinearFp8), _c.POINTER(FvqLinearFp8),
                               _vp, _vp, _sz, _vp]),
    "fvq_fp8_ffn_profile": (_c.c_int, [_vp, _i64, _c.POINTER(FvqLinearFp8),
                                       _c.POINTER(FvqLinearFp8), _vp, _vp, _sz, _vp,
                                       _c.POINTER(_c.c_float)]),
    "fvq_div_full_probe": (_c.c_int, [_vp, _vp, _vp, _i64, _vp]),
    "fvq_pil_resize": (_c.c_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                  _vp, _vp, _vp]),
    "fvq_pil_normalize": (_c.c_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "fvq_rcp_approx_probe": (_c.c_int, [_vp, _vp, _i64, _vp]),
    "fvq_gelu_bf16_probe": (_c.c_int, [_vp, _vp, _i64, _vp]),
    "fvq_set_wait_limit": (_c.c_int, [_c.c_uint64]),
    "fvq_read_device_error": (_c.c_int, [_vp, _c.POINTER(_c.c_uint32)]),
}


class FvqError(RuntimeError):
    """A non-zero status from libfvq."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load libfvq.so and attach the signatures (raises if it is missing)."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise FileNotFoundError(
                f"{p} is missing: build it with `python flashvsr-optimizations_b200/build.py` "
                "(there is no fallback path)")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(fn_name: str, rc: int) -> None:
    if rc != FVQ_OK:
        msg = load().fvq_last_error()
        raise FvqError(fn_name, rc, msg.decode() if msg else "")


def call(fn_name: str, *args) -> None:
    lib = load()
    check(fn_name, getattr(lib, fn_name)(*args))
