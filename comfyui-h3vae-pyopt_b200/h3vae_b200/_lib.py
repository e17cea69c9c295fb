"""ctypes binding of libh3vae_b200.so (the C ABI declared in include/h3vae_b200.h).

The shared library is the only compute path.  There is deliberately no CPU or
PyTorch fallback: if the library is missing or a call fails, an exception is
raised (ValueError for contract violations, RuntimeError for CUDA/device
errors), mirroring the reference's fail-fast policy.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p, c_char_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libh3vae_b200.so"

H3B_OK = 0
H3B_EINVAL = -1
H3B_EUNSUPPORTED = -2
H3B_ECUDA = -3
H3B_EDEVICE = -4

_i64p = POINTER(c_int64)

# name -> (restype, argtypes)
_SIGNATURES = {
    "h3b_last_error": (c_char_p, []),
    "h3b_abi_version": (c_int, []),
    "h3b_device_error": (c_int, [POINTER(c_uint), c_int]),
    "h3b_probe_wait_timeout": (c_int, [c_uint, c_void_p]),
    "h3b_conv3d_i8": (c_int, [c_void_p, _i64p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_int,
                              c_void_p, c_void_p, c_void_p, c_void_p, _i64p, c_void_p, c_void_p, c_int, c_void_p]),
    "h3b_conv3d_f16": (c_int, [c_void_p, _i64p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_void_p, c_void_p, _i64p, c_void_p, c_int, c_void_p]),
    "h3b_conv3d_rgb_f16": (c_int, [c_void_p, _i64p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "h3b_conv3d_i8_token": (c_int, [c_void_p, _i64p, c_void_p, c_int64, c_int, c_int, c_int, c_int, c_int, c_int,
                                    c_void_p, c_void_p, c_void_p, c_void_p, _i64p, c_void_p, c_int, c_void_p]),
    "h3b_norm_pad_quant_token": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                         c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "h3b_conv_in_workspace_size": (c_size_t, [c_int64] * 4),
    "h3b_conv_in_f16": (c_int, [c_void_p, _i64p, _i64p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                c_void_p, c_size_t, c_void_p]),
    "h3b_im2col_causal_f16": (c_int, [c_void_p, _i64p, _i64p, c_void_p, c_void_p]),
    "h3b_quantize_tensor_workspace_size": (c_size_t, []),
    "h3b_quantize_tensor_i8": (c_int, [c_void_p, _i64p, _i64p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "h3b_norm_workspace_size": (c_size_t, [c_int64] * 5),
    "h3b_norm_pad_quant": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                   c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "h3b_norm_pad_quant_noalloc": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                           c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p]),
    "h3b_norm_pad_f16": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                 c_void_p, c_float, c_void_p, c_void_p, c_size_t, c_void_p]),
    "h3b_upsample_norm_pad_f16": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                          c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_size_t,
                                          c_void_p]),
    "h3b_residual_pack": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                                  c_void_p, c_void_p]),
    "h3b_gemm_i8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                            c_void_p, c_int64, c_void_p, c_void_p]),
    "h3b_gemm_i8_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                   c_void_p, c_void_p]),
    "h3b_gemm_i8_residual_parts": (c_int64, [c_int64]),
    "h3b_gemm_i8_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                     c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "h3b_rms_quant_parts": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p,
                                    c_void_p, c_void_p, c_void_p]),
    "h3b_gemm_f16": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "h3b_gemm_f16_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "h3b_gemm_i8_qkv_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                     c_int64, c_void_p, c_void_p, c_int64, c_float, c_void_p, c_void_p, c_void_p,
                                     c_void_p]),
    "h3b_row_quant": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "h3b_swiglu_quant": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "h3b_residual_rms_quant": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_int,
                                       c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "h3b_rms_norm_f16": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p]),
    "h3b_rms_quant": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p, c_void_p]),
    "h3b_final_residual_layernorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                             c_float, c_void_p, c_void_p]),
    "h3b_qk_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_float, c_void_p,
                            c_void_p, c_void_p]),
    "h3b_attention_f16": (c_int, [c_void_p, _i64p, c_void_p, _i64p, c_void_p, _i64p, c_void_p, _i64p, c_int64,
                                  c_int64, c_int64, c_int64, c_float, c_void_p]),
    "h3b_finalize_pixels": (c_int, [c_void_p, c_int, _i64p, _i64p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "h3b_blend_accumulate": (c_int, [c_void_p, c_int, _i64p, _i64p, c_void_p, c_void_p, _i64p, c_void_p]),
}

EXPORTED_SYMBOLS = tuple(name for name in _SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class H3BError(RuntimeError):
    """A CUDA or device-side failure reported by the library."""


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"h3vae_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (no CPU fallback exists)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def last_error() -> str:
    msg = load().h3b_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def check(rc: int) -> None:
    """Map a C status to the reference's exception conventions."""
    if rc == H3B_OK:
        return
    msg = last_error()
    if rc in (H3B_EINVAL, H3B_EUNSUPPORTED):
        raise ValueError(msg)
    raise H3BError(f"h3vae_b200 failure ({rc}): {msg}")


def i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (c_int64 * len(vals))(*vals)


def device_error(clear: bool = True) -> int:
    """Synchronize and return (optionally clearing) the device error word."""
    bits = c_uint(0)
    check(load().h3b_device_error(ctypes.byref(bits), 1 if clear else 0))
    return int(bits.value)
