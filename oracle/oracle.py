"""ctypes binding of the CPU oracle (``oracle/aw4_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by ``__graft_entry__.smoke()``
as the checker and by ``bench.py``'s CPU-baseline legs.  The product package
``adamw4bit_b200`` never imports this module.

The oracle restates nubank/adamw4bit's CPU algorithm (see the C file header for
the per-function citations).  Codebooks are the reference's float32 tables,
written out bit-exactly; ``tests/test_oracle_golden.py`` pins them against
the values the reference itself produced (``tests/golden/codebooks.json``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libaw4_oracle.so")

RTN, SR_VALUE, SR_UPDATE = 0, 1, 2
F32, BF16, F16 = 0, 1, 2
BLOCK = 128

# Reference per-moment RNG seed offsets (adamw.py:122-125).
M1_OFFSET = 0x1A2B3C4D
M2_OFFSET = 0x5E6F7789


def _bits(words: list[int]) -> np.ndarray:
    return np.array(words, dtype=np.uint32).view(np.float32)


# quantization.py:401-422 (NF4 table, float32 rounding of the decimal literals)
NF4 = np.array(
    [-1.0, -0.6961928, -0.5250731, -0.3949175, -0.2844414, -0.1847734, -0.0910500, 0.0,
     0.0795803, 0.1609302, 0.2461123, 0.3379152, 0.4407098, 0.5626170, 0.7229568, 1.0],
    dtype=np.float32,
)
# quantization.py:201-237 _create_dynamic_map(signed=True, 3, 4)
SDYN4 = _bits([0xBF633333, 0xBF29999A, 0xBEE00000, 0xBE599999, 0xBD9EB852, 0xBD051EB9,
               0xBBB43958, 0x00000000, 0x3BB43958, 0x3D051EB9, 0x3D9EB852, 0x3E599999,
               0x3EE00000, 0x3F29999A, 0x3F633333, 0x3F800000])
# quantization.py:201-237 _create_dynamic_map(signed=False, 3, 4)
DYN4 = _bits([0x00000000, 0x3B54FDF4, 0x3BFDF3B5, 0x3CAE147B, 0x3D333333, 0x3D87AE15,
              0x3DB5C28F, 0x3E200000, 0x3E89999A, 0x3EC33333, 0x3EFCCCCD, 0x3F1B3334,
              0x3F380000, 0x3F54CCCC, 0x3F71999A, 0x3F800000])
# quantization.py:460-461 torch.linspace(0, 1, 16, dtype=float32)
LIN4 = _bits([0x00000000, 0x3D888889, 0x3E088889, 0x3E4CCCCE, 0x3E888889, 0x3EAAAAAB,
              0x3ECCCCCE, 0x3EEEEEF0, 0x3F088888, 0x3F199999, 0x3F2AAAAA, 0x3F3BBBBC,
              0x3F4CCCCD, 0x3F5DDDDE, 0x3F6EEEEF, 0x3F800000])
# quantization.py:469-470 torch.linspace(0, 1, 17)[1:]
LIN4_NZ = (np.arange(1, 17, dtype=np.float32) / np.float32(16)).astype(np.float32)

# scheme -> (codebook, rounding mode, zero floor)   (quantization.py:561-586)
SCHEMES = {
    "nf4": (NF4, RTN, 0),
    "nf4_sr": (NF4, SR_VALUE, 0),
    "sdyn4": (SDYN4, RTN, 0),
    "sdyn4_sr": (SDYN4, SR_VALUE, 0),
    "dyn4": (DYN4, RTN, 0),
    "dyn4_nz": (DYN4, RTN, 1),
    "dyn4_sr": (DYN4, SR_VALUE, 0),
    "dyn4_upd_sr_fp32read": (DYN4, SR_UPDATE, 0),
    "dyn4_lookahead_sr": (DYN4, SR_UPDATE, 0),
    "dyn4_upd_sr_fp32read_nextbc": (DYN4, SR_UPDATE, 0),
    "lin4": (LIN4, RTN, 0),
    "lin4_nz": (LIN4_NZ, RTN, 0),
    "lin4_sr": (LIN4, SR_VALUE, 0),
    "lin4_upd_sr_fp32read": (LIN4, SR_UPDATE, 0),
}
NEXT_BIAS = {"dyn4_lookahead_sr", "dyn4_upd_sr_fp32read_nextbc"}


class StepCfg(ctypes.Structure):
    _fields_ = [
        ("param_dtype", ctypes.c_int), ("grad_dtype", ctypes.c_int),
        ("m1_mode", ctypes.c_int), ("m2_mode", ctypes.c_int),
        ("m2_zero_floor", ctypes.c_int), ("eden", ctypes.c_int),
        ("m2_next_bias", ctypes.c_int),
        ("cb1", ctypes.c_void_p), ("cb2", ctypes.c_void_p),
        ("lr", ctypes.c_double), ("beta1", ctypes.c_double), ("beta2", ctypes.c_double),
        ("eps", ctypes.c_double), ("weight_decay", ctypes.c_double),
        ("step", ctypes.c_int64),
        ("m1_key", ctypes.c_uint64), ("m2_key", ctypes.c_uint64),
        ("ordinal", ctypes.c_uint32),
        ("elem_offset", ctypes.c_int64),
    ]


_lib = None


def build() -> str:
    """Compile the oracle shared library with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, i32, f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double
        L.aw4o_step.argtypes = [ctypes.POINTER(StepCfg), vp, vp, i64, vp, vp, vp, vp, vp, vp]
        L.aw4o_step_fp32_state.argtypes = [ctypes.POINTER(StepCfg), vp, vp, i64, vp, vp]
        L.aw4o_step_fp32_m1.argtypes = [ctypes.POINTER(StepCfg), vp, vp, i64, vp, vp, vp, vp]
        L.aw4o_quantize.argtypes = [vp, i64, vp, i32, i32, i32, vp, f64, f64, vp, vp]
        L.aw4o_dequantize.argtypes = [vp, vp, i64, vp, vp]
        L.aw4o_dequantize.restype = None
        L.aw4o_pack.argtypes = [vp, i64, vp]
        L.aw4o_pack.restype = None
        L.aw4o_unpack.argtypes = [vp, i64, vp]
        L.aw4o_unpack.restype = None
        L.aw4o_init_zero.argtypes = [vp, i32, i32, i32, i64, vp, vp]
        L.aw4o_philox_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint64]
        L.aw4o_philox_uniform.restype = ctypes.c_float
        L.aw4o_max_threads.restype = ctypes.c_int
        L.aw4o_set_threads.argtypes = [ctypes.c_int]
        L.aw4o_set_threads.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().aw4o_set_threads(int(n))


def max_threads() -> int:
    return int(lib().aw4o_max_threads())


def quantize(x: np.ndarray, scheme: str, *, eden: bool = False, draws: np.ndarray | None = None,
             bias_correction: float | None = None, eps: float | None = None):
    """quantize() for one 4-bit scheme, block 128; returns (codes uint8 unpacked, scales f32)."""
    cb, mode, floor = SCHEMES[scheme]
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    n = x.size
    codes = np.empty(n, np.uint8)
    scales = np.empty(n // BLOCK, np.float32)
    if mode != RTN:
        assert draws is not None and draws.size == n
        draws = np.ascontiguousarray(draws, dtype=np.float32).reshape(-1)
    bias = 1.0 if bias_correction is None else float(bias_correction)
    e = 1e-8 if eps is None else float(eps)
    rc = lib().aw4o_quantize(_ptr(x), n, _ptr(cb), mode, floor, int(eden), _ptr(draws),
                             bias, e, _ptr(codes), _ptr(scales))
    assert rc == 0
    return codes, scales


def dequantize(codes: np.ndarray, scales: np.ndarray, scheme: str) -> np.ndarray:
    cb = SCHEMES[scheme][0]
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1)
    out = np.empty(codes.size, np.float32)
    lib().aw4o_dequantize(_ptr(codes), _ptr(np.ascontiguousarray(scales, np.float32)),
                          codes.size, _ptr(cb), _ptr(out))
    return out


def pack(codes: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1)
    out = np.empty((codes.size + 1) // 2, np.uint8)
    lib().aw4o_pack(_ptr(codes), codes.size, _ptr(out))
    return out


def unpack(packed: np.ndarray, n: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint8).reshape(-1)
    out = np.empty(n, np.uint8)
    lib().aw4o_unpack(_ptr(packed), n, _ptr(out))
    return out


def philox_uniform(key: int, step: int, ordinal: int, elem: int) -> float:
    return float(lib().aw4o_philox_uniform(key, step, ordinal, elem))


def stream_key(seed: int, offset: int) -> int:
    """64-bit Philox key of one moment stream: (seed + offset) mod (2**63 - 1),
    the same seed derivation as the reference generators (adamw.py:297-305)."""
    return (seed + offset) % ((1 << 63) - 1)


def make_cfg(*, m1_scheme: str, m2_scheme: str, eden: bool, lr: float, betas, eps: float,
             weight_decay: float, step: int, param_dtype: int = F32, grad_dtype: int = F32,
             m1_key: int = 0, m2_key: int = 0, ordinal: int = 0, elem_offset: int = 0):
    cb2, mode2, floor2 = SCHEMES[m2_scheme]
    # an FP32 first moment (step_fp32_m1) has no codebook: m1 fields unused
    cb1, mode1, _ = (cb2, RTN, 0) if m1_scheme == "fp32" else SCHEMES[m1_scheme]
    cfg = StepCfg(param_dtype, grad_dtype, mode1, mode2, floor2, int(eden),
                  int(m2_scheme in NEXT_BIAS), cb1.ctypes.data, cb2.ctypes.data,
                  lr, betas[0], betas[1], eps, weight_decay, step, m1_key, m2_key, ordinal,
                  elem_offset)
    cfg._keep = (cb1, cb2)  # keep the codebook arrays alive
    return cfg


def step(cfg: StepCfg, param: np.ndarray, grad: np.ndarray, m1_codes: np.ndarray,
         m1_scales: np.ndarray, m2_codes: np.ndarray, m2_scales: np.ndarray,
         m1_draws: np.ndarray | None = None, m2_draws: np.ndarray | None = None) -> None:
    """In-place quantized step of one tensor (param f32 or uint16 bf16/f16 bits)."""
    n = param.size
    for a in (param, grad, m1_codes, m1_scales, m2_codes, m2_scales):
        assert a.flags["C_CONTIGUOUS"]
    rc = lib().aw4o_step(ctypes.byref(cfg), _ptr(param), _ptr(grad), n, _ptr(m1_codes),
                         _ptr(m1_scales), _ptr(m2_codes), _ptr(m2_scales), _ptr(m1_draws),
                         _ptr(m2_draws))
    assert rc == 0


def step_fp32_m1(cfg: StepCfg, param: np.ndarray, grad: np.ndarray, m1: np.ndarray,
                 m2_codes: np.ndarray, m2_scales: np.ndarray,
                 m2_draws: np.ndarray | None = None) -> None:
    """In-place step of one tensor with an FP32 m1 (float32[n]) next to a
    packed 4-bit m2 (cfg made with m1_scheme="fp32")."""
    for a in (param, grad, m1, m2_codes, m2_scales):
        assert a.flags["C_CONTIGUOUS"]
    rc = lib().aw4o_step_fp32_m1(ctypes.byref(cfg), _ptr(param), _ptr(grad), param.size,
                                 _ptr(m1), _ptr(m2_codes), _ptr(m2_scales), _ptr(m2_draws))
    assert rc == 0


def step_fp32_state(cfg: StepCfg, param: np.ndarray, grad: np.ndarray, m1: np.ndarray,
                    m2: np.ndarray) -> None:
    rc = lib().aw4o_step_fp32_state(ctypes.byref(cfg), _ptr(param), _ptr(grad), param.size,
                                    _ptr(m1), _ptr(m2))
    assert rc == 0


def init_zero(scheme: str, n: int, *, eden: bool = False):
    """Packed codes and scales of a zero moment (adamw.py:524-545)."""
    cb, mode, floor = SCHEMES[scheme]
    packed = np.empty(n // 2, np.uint8)
    scales = np.empty(n // BLOCK, np.float32)
    rc = lib().aw4o_init_zero(_ptr(cb), mode, floor, int(eden), n, _ptr(packed), _ptr(scales))
    assert rc == 0
    return packed, scales
