"""ctypes binding of libadamw4bit_b200.so (the C ABI in include/adamw4bit_b200.h).

The shared library is the only compute path of this package.  Loading fails
loudly when it is missing or when no CUDA device is present at call time;
there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libadamw4bit_b200.so")

AW4_OK, AW4_ERR_INVALID, AW4_ERR_CUDA, AW4_ERR_UNSUPPORTED = 0, 1, 2, 3
F32, BF16, F16 = 0, 1, 2
RTN, SR_VALUE, SR_UPDATE, FP32_MOMENT = 0, 1, 2, 3
BLOCK = 128
LUT_BINS = 1024
ABI_VERSION = 5

DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


class Scheme(ctypes.Structure):
    _fields_ = [
        ("codebook", ctypes.c_float * 16),
        ("round_mode", ctypes.c_int32),
        ("zero_floor", ctypes.c_int32),
        ("lut_bins", ctypes.c_int32),
        ("lut", ctypes.c_uint8 * LUT_BINS),
        ("thr", ctypes.c_float * 18),
        ("zero_scale", ctypes.c_float),
        ("zero_scale_eden", ctypes.c_float),
        ("zero_code", ctypes.c_uint8),
        ("pad", ctypes.c_uint8 * 3),
    ]


class Hyper(ctypes.Structure):
    _fields_ = [
        ("w1", ctypes.c_float), ("w2", ctypes.c_float), ("decay", ctypes.c_float),
        ("neg_step", ctypes.c_float), ("sqrt_bc2", ctypes.c_float), ("eps", ctypes.c_float),
        ("sr_bias", ctypes.c_float), ("step", ctypes.c_uint32),
        ("m1_key", ctypes.c_uint64), ("m2_key", ctypes.c_uint64),
        ("grad_scale", ctypes.c_float), ("pad", ctypes.c_int32),
    ]


class QTensor(ctypes.Structure):
    _fields_ = [
        ("param", ctypes.c_void_p), ("grad", ctypes.c_void_p),
        ("m1_codes", ctypes.c_void_p), ("m1_scales", ctypes.c_void_p),
        ("m2_codes", ctypes.c_void_p), ("m2_scales", ctypes.c_void_p),
        ("m1_draws", ctypes.c_void_p), ("m2_draws", ctypes.c_void_p),
        ("numel", ctypes.c_int64), ("elem_offset", ctypes.c_int64),
        ("ordinal", ctypes.c_uint32), ("hyper", ctypes.c_int32),
        ("param_copy", ctypes.c_void_p),
        ("copy_multicast", ctypes.c_int32), ("grad_multicast", ctypes.c_int32),
    ]


class FTensor(ctypes.Structure):
    _fields_ = [
        ("param", ctypes.c_void_p), ("grad", ctypes.c_void_p),
        ("m1", ctypes.c_void_p), ("m2", ctypes.c_void_p),
        ("numel", ctypes.c_int64), ("hyper", ctypes.c_int32), ("pad", ctypes.c_int32),
    ]


class NativeError(RuntimeError):
    """An error status returned by the CUDA library."""


_lib = None
_lock = threading.Lock()

# Exported symbols and their ctypes signatures (kept in the order of the header).
_VP, _I32, _I64, _U32, _U64, _F = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                   ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float)
SIGNATURES = {
    "aw4_abi_version": ([], _I32),
    "aw4_last_error": ([], ctypes.c_char_p),
    "aw4_launch_count": ([], _U64),
    "aw4_scheme_prepare": ([_VP, _I32, _I32, ctypes.POINTER(Scheme)], _I32),
    "aw4_step_quantized": ([ctypes.POINTER(Scheme), ctypes.POINTER(Scheme), _I32, _I32, _I32,
                            ctypes.POINTER(QTensor), _I32, ctypes.POINTER(Hyper), _I32, _I32, _I32,
                            _VP], _I32),
    "aw4_step_fp32_state": ([_I32, _I32, ctypes.POINTER(FTensor), _I32, ctypes.POINTER(Hyper),
                             _I32, _I32, _VP], _I32),
    "aw4_init_zero_state": ([ctypes.POINTER(Scheme), _I32, _VP, _VP, _I64, _I32, _VP], _I32),
    "aw4_quantize_blocks": ([ctypes.POINTER(Scheme), _I32, _VP, _I64, _VP, _VP, _VP, _U64, _U32,
                             _U32, _F, _F, _I32, _VP], _I32),
    "aw4_dequantize_blocks": ([ctypes.POINTER(Scheme), _VP, _VP, _I64, _VP, _I32, _VP], _I32),
    "aw4_pack_codes": ([_VP, _I64, _VP, _I32, _VP], _I32),
    "aw4_unpack_codes": ([_VP, _I64, _VP, _I32, _VP], _I32),
    "aw4_reduce_multicast": ([_VP, _I32, _I64, _F, _VP, _I32, _VP], _I32),
    "aw4_selfcheck_math": ([_VP, _I32, _VP], _I32),
}


def lib() -> ctypes.CDLL:
    """Load the CUDA library (built by ``python -m adamw4bit_b200.build``)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m adamw4bit_b200.build` "
                    "(adamw4bit_b200 has no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = res
            if L.aw4_abi_version() != ABI_VERSION:
                raise ImportError(f"{LIB_PATH}: ABI version {L.aw4_abi_version()} != {ABI_VERSION}")
            _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != AW4_OK:
        msg = lib().aw4_last_error().decode(errors="replace")
        kind = {AW4_ERR_INVALID: "invalid argument", AW4_ERR_CUDA: "CUDA error",
                AW4_ERR_UNSUPPORTED: "unsupported"}.get(rc, f"status {rc}")
        raise NativeError(f"{what}: {kind}: {msg}")


def launch_count() -> int:
    return int(lib().aw4_launch_count())


def prepare_scheme(codebook, round_mode: int, zero_floor: bool) -> Scheme:
    cb = (ctypes.c_float * 16)(*[float(v) for v in codebook])
    s = Scheme()
    check(lib().aw4_scheme_prepare(ctypes.cast(cb, ctypes.c_void_p), round_mode, int(zero_floor),
                                   ctypes.byref(s)), "aw4_scheme_prepare")
    return s


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: adamw4bit_b200 runs on CUDA devices only (got {t.device})")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
