"""4-bit block codec: codebooks, QuantState, packing and GPU quantize/dequantize.

Mirrors the reference module ``adamw4bit.quantization`` (nubank/adamw4bit,
src/adamw4bit/quantization.py) for the 4-bit schemes the fused step supports.
Every numerical routine here runs on the CUDA library (``_native``); the
reference's 8-bit schemes, the lookahead oracle codec and the bitsandbytes
branch are outside this package's scope and raise ``NotImplementedError``.
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N

__all__ = [
    "QuantState", "SchemeInfo", "SCHEMES", "codebook", "default_block_size",
    "default_min_scale", "is_4bit_scheme", "pack_4bit_codes", "unpack_4bit_codes",
    "pack_codes_for_storage", "codes_for_dequantization", "quantize",
    "quantize_with_dequantized", "dequantize", "apply_eden_correction_to_quant_state",
]


class QuantState:
    """Per-tensor quantization metadata (quantization.py:15-30): block scales
    (``absmax``), logical shape, dtype of the quantized values, block size and
    whether codes are nibble-packed."""

    def __init__(self, absmax, shape=None, dtype=None, blocksize=None, packed: bool = False):
        self.absmax = absmax
        self.shape = shape
        self.dtype = dtype
        self.blocksize = blocksize
        self.packed = packed

    def __repr__(self) -> str:
        return (f"QuantState(absmax={tuple(self.absmax.shape)}, shape={tuple(self.shape)}, "
                f"dtype={self.dtype}, blocksize={self.blocksize}, packed={self.packed})")


def _bits(words) -> np.ndarray:
    return np.array(words, dtype=np.uint32).view(np.float32)


# Float32 tables equal, bit for bit, to the reference's codebooks:
#   NF4 (quantization.py:401-422), signed/unsigned dynamic maps from
#   _create_dynamic_map(signed, max_exponent_bits=3, total_bits=4)
#   (quantization.py:201-237), torch.linspace(0, 1, 16) and
#   torch.linspace(0, 1, 17)[1:] (quantization.py:457-470).
NF4 = _bits([0xBF800000, 0xBF3239B1, 0xBF066B31, 0xBECA32A0, 0xBE91A24E, 0xBE3D353D,
             0xBDBA786C, 0x00000000, 0x3DA2FAFF, 0x3E24CAE3, 0x3E7C04DD, 0x3EAD0339,
             0x3EE1A4B7, 0x3F1007AB, 0x3F3913B2, 0x3F800000])
SDYN4 = _bits([0xBF633333, 0xBF29999A, 0xBEE00000, 0xBE599999, 0xBD9EB852, 0xBD051EB9,
               0xBBB43958, 0x00000000, 0x3BB43958, 0x3D051EB9, 0x3D9EB852, 0x3E599999,
               0x3EE00000, 0x3F29999A, 0x3F633333, 0x3F800000])
DYN4 = _bits([0x00000000, 0x3B54FDF4, 0x3BFDF3B5, 0x3CAE147B, 0x3D333333, 0x3D87AE15,
              0x3DB5C28F, 0x3E200000, 0x3E89999A, 0x3EC33333, 0x3EFCCCCD, 0x3F1B3334,
              0x3F380000, 0x3F54CCCC, 0x3F71999A, 0x3F800000])
LIN4 = _bits([0x00000000, 0x3D888889, 0x3E088889, 0x3E4CCCCE, 0x3E888889, 0x3EAAAAAB,
              0x3ECCCCCE, 0x3EEEEEF0, 0x3F088888, 0x3F199999, 0x3F2AAAAA, 0x3F3BBBBC,
              0x3F4CCCCD, 0x3F5DDDDE, 0x3F6EEEEF, 0x3F800000])
LIN4_NZ = _bits([0x3D800000, 0x3E000000, 0x3E400000, 0x3E800000, 0x3EA00000, 0x3EC00000,
                 0x3EE00000, 0x3F000000, 0x3F100000, 0x3F200000, 0x3F300000, 0x3F400000,
                 0x3F500000, 0x3F600000, 0x3F700000, 0x3F800000])


@dataclass(frozen=True)
class SchemeInfo:
    """A 4-bit scheme: codebook, rounding mode, dyn4_nz zero floor, and for
    update-SR storage whether the bias correction targets step t+1."""
    name: str
    codebook: np.ndarray
    round_mode: int
    zero_floor: bool = False
    next_bias: bool = False
    signed: bool = False


# quantization.py:561-586, restricted to the schemes the fused kernel implements
# (the set the reference's own optimized backend accepts, _optimized.py:36-42).
SCHEMES: dict[str, SchemeInfo] = {
    "nf4": SchemeInfo("nf4", NF4, N.RTN, signed=True),
    "nf4_sr": SchemeInfo("nf4_sr", NF4, N.SR_VALUE, signed=True),
    "sdyn4": SchemeInfo("sdyn4", SDYN4, N.RTN, signed=True),
    "sdyn4_sr": SchemeInfo("sdyn4_sr", SDYN4, N.SR_VALUE, signed=True),
    "dyn4": SchemeInfo("dyn4", DYN4, N.RTN),
    "dyn4_nz": SchemeInfo("dyn4_nz", DYN4, N.RTN, zero_floor=True),
    "dyn4_sr": SchemeInfo("dyn4_sr", DYN4, N.SR_VALUE),
    "dyn4_upd_sr_fp32read": SchemeInfo("dyn4_upd_sr_fp32read", DYN4, N.SR_UPDATE),
    "dyn4_lookahead_sr": SchemeInfo("dyn4_lookahead_sr", DYN4, N.SR_UPDATE, next_bias=True),
    "dyn4_upd_sr_fp32read_nextbc": SchemeInfo("dyn4_upd_sr_fp32read_nextbc", DYN4, N.SR_UPDATE,
                                              next_bias=True),
    "lin4": SchemeInfo("lin4", LIN4, N.RTN),
    "lin4_nz": SchemeInfo("lin4_nz", LIN4_NZ, N.RTN),
    "lin4_sr": SchemeInfo("lin4_sr", LIN4, N.SR_VALUE),
    "lin4_upd_sr_fp32read": SchemeInfo("lin4_upd_sr_fp32read", LIN4, N.SR_UPDATE),
}

# Every 4-bit scheme the reference knows (quantization.py:604-610); the ones
# missing from SCHEMES are research ablations this package does not implement.
_REFERENCE_4BIT = {
    "sdyn4", "sdyn4_sr", "nf4", "nf4_sr", "lin4", "lin4_sr", "lin4_upd_sr",
    "lin4_upd_sr_store_eden", "lin4_upd_sr_fp32read", "lin4_nz", "dyn4", "dyn4_sr",
    "dyn4_upd_sr", "dyn4_upd_sr_store_eden", "dyn4_upd_sr_fp32read", "dyn4_lookahead_sr",
    "dyn4_upd_sr_fp32read_nextbc", "dyn4_la_upd_sr", "dyn4_proxy_la_upd_sr",
    "dyn4_vproxy_la_upd_sr", "dyn4_nz",
}
_REFERENCE_8BIT = {"linear", "dynamic"}


def is_4bit_scheme(mode: str) -> bool:
    """quantization.py:613-615 (16-entry codebook schemes)."""
    return mode in _REFERENCE_4BIT


def default_block_size(mode: str) -> int:
    """quantization.py:694-703: 4-bit schemes use 128-value blocks, others 256."""
    return 128 if mode in _REFERENCE_4BIT else 256


def default_min_scale(mode: str) -> float:
    """quantization.py:706-712: 1e-12 floor for 4-bit schemes, 1e-8 otherwise."""
    return 1e-12 if mode in _REFERENCE_4BIT else 1e-8


def scheme_info(mode: str) -> SchemeInfo:
    if mode not in SCHEMES:
        if mode in _REFERENCE_4BIT or mode in _REFERENCE_8BIT:
            raise NotImplementedError(
                f"scheme {mode!r} is not implemented by the fused B200 kernels "
                f"(supported: {sorted(SCHEMES)})")
        raise ValueError(f"Unsupported quantization mode: {mode}")
    return SCHEMES[mode]


def codebook(mode: str, device: torch.device | str = "cpu") -> torch.Tensor:
    return torch.from_numpy(scheme_info(mode).codebook.copy()).to(device)


@functools.lru_cache(maxsize=None)
def prepared(mode: str) -> N.Scheme:
    """Native rounding tables of a scheme (built once per process)."""
    info = scheme_info(mode)
    return N.prepare_scheme(info.codebook, info.round_mode, info.zero_floor)


# ---------------------------------------------------------------------------
# nibble packing (quantization.py:627-691)
# ---------------------------------------------------------------------------

def pack_4bit_codes(codes: torch.Tensor) -> torch.Tensor:
    """Two codes per byte, even element in the low nibble (quantization.py:627-638)."""
    if codes.dtype != torch.uint8:
        raise TypeError(f"4-bit codes must use torch.uint8, found {codes.dtype}")
    N.require_cuda(codes, "pack_4bit_codes")
    flat = codes.reshape(-1).contiguous()
    out = torch.empty((flat.numel() + 1) // 2, dtype=torch.uint8, device=codes.device)
    N.check(N.lib().aw4_pack_codes(N.ptr(flat), flat.numel(), N.ptr(out), codes.device.index,
                                   N.stream_handle(codes.device)), "aw4_pack_codes")
    return out


def unpack_4bit_codes(codes: torch.Tensor, *, numel: int) -> torch.Tensor:
    """quantization.py:641-654."""
    if codes.dtype != torch.uint8:
        raise TypeError(f"Packed 4-bit codes must use torch.uint8, found {codes.dtype}")
    expected = (numel + 1) // 2
    if codes.numel() != expected:
        raise ValueError(f"Packed code length mismatch: expected {expected}, found {codes.numel()}")
    N.require_cuda(codes, "unpack_4bit_codes")
    flat = codes.reshape(-1).contiguous()
    out = torch.empty(numel, dtype=torch.uint8, device=codes.device)
    N.check(N.lib().aw4_unpack_codes(N.ptr(flat), numel, N.ptr(out), codes.device.index,
                                     N.stream_handle(codes.device)), "aw4_unpack_codes")
    return out


def pack_codes_for_storage(codes: torch.Tensor, quant_state: QuantState, *, mode: str):
    """quantization.py:657-668."""
    if not is_4bit_scheme(mode):
        quant_state.packed = False
        return codes, quant_state
    quant_state.packed = True
    return pack_4bit_codes(codes), quant_state


def _numel(shape) -> int:
    if shape is None:
        raise ValueError("Quantized state is missing its logical shape")
    return int(math.prod(int(d) for d in shape))


def codes_for_dequantization(codes: torch.Tensor, quant_state: QuantState, *, mode: str):
    """Logical-shape codes from packed or legacy unpacked state (quantization.py:671-691)."""
    if not is_4bit_scheme(mode):
        return codes
    n = _numel(quant_state.shape)
    is_packed = bool(getattr(quant_state, "packed", False))
    if not is_packed and codes.numel() == n:
        return codes.reshape(quant_state.shape)
    if not is_packed and codes.numel() != (n + 1) // 2:
        raise ValueError("4-bit code storage does not match either the logical or packed shape")
    return unpack_4bit_codes(codes, numel=n).reshape(quant_state.shape)


def packed_codes(codes: torch.Tensor, quant_state: QuantState) -> torch.Tensor:
    """Packed storage of a moment whose codes may be legacy one-per-byte."""
    n = _numel(quant_state.shape)
    if getattr(quant_state, "packed", False) or codes.numel() != n or n == 1:
        return codes.reshape(-1)
    return pack_4bit_codes(codes)


# ---------------------------------------------------------------------------
# quantize / dequantize (quantization.py:715-1004), 128-value blocks
# ---------------------------------------------------------------------------

def _draws_for(x: torch.Tensor, generator, draws):
    if draws is not None:
        return draws.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    return torch.rand((x.numel() // 128, 128), device=x.device, dtype=torch.float32,
                      generator=generator).reshape(-1)


def _quantize_impl(x, block_size, mode, use_bitsandbytes, min_scale, eden_correction,
                   generator, bias_correction, eps, draws, return_dequantized):
    if use_bitsandbytes:
        raise NotImplementedError("bitsandbytes quantization is outside adamw4bit_b200")
    info = scheme_info(mode)
    if block_size != 128:
        raise NotImplementedError("the B200 codec uses 128-value blocks")
    if min_scale is not None and min_scale != default_min_scale(mode):
        raise NotImplementedError("custom min_scale is not supported")
    N.require_cuda(x, "quantize")
    n = x.numel()
    if n % 128:
        raise NotImplementedError("numel must be a multiple of the 128-value block")
    flat = x.reshape(-1).to(torch.float32).contiguous()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(n // 128, dtype=torch.float32, device=x.device)
    u = _draws_for(flat, generator, draws) if info.round_mode != N.RTN else None
    bias = max(float(bias_correction) if bias_correction is not None else 1.0, 1e-12)
    e = float(eps) if eps is not None else 1e-8
    N.check(N.lib().aw4_quantize_blocks(
        prepared(mode), int(bool(eden_correction)), N.ptr(flat), n, N.ptr(packed), N.ptr(scales),
        N.ptr(u), 0, 0, 0, float(np.float32(bias)), float(np.float32(e)), x.device.index,
        N.stream_handle(x.device)), "aw4_quantize_blocks")
    codes = unpack_4bit_codes(packed, numel=n).reshape(x.shape)
    qs = QuantState(absmax=scales, shape=x.shape, dtype=x.dtype, blocksize=block_size)
    if return_dequantized:
        deq = dequantize(packed, QuantState(scales, x.shape, x.dtype, block_size, packed=True),
                         mode=mode)
        return codes, qs, deq
    return codes, qs


def quantize(x, block_size: int = 128, mode: str = "nf4", use_bitsandbytes: bool = False,
             min_scale=None, eden_correction: bool = False, generator=None,
             bias_correction=None, eps=None, draws=None):
    """Block-wise 4-bit quantization on the GPU (quantization.py:715-745, 898-971).
    Returns unpacked logical-shape uint8 codes and their QuantState."""
    return _quantize_impl(x, block_size, mode, use_bitsandbytes, min_scale, eden_correction,
                          generator, bias_correction, eps, draws, False)


def quantize_with_dequantized(x, block_size: int = 128, mode: str = "nf4",
                              use_bitsandbytes: bool = False, min_scale=None,
                              eden_correction: bool = False, generator=None,
                              bias_correction=None, eps=None, draws=None):
    """quantization.py:748-776."""
    return _quantize_impl(x, block_size, mode, use_bitsandbytes, min_scale, eden_correction,
                          generator, bias_correction, eps, draws, True)


def dequantize(codes: torch.Tensor, quant_state: QuantState, mode: str = "nf4",
               use_bitsandbytes: bool = False) -> torch.Tensor:
    """cb[code] * absmax[block] on the GPU (quantization.py:975-1004)."""
    if use_bitsandbytes:
        raise NotImplementedError("bitsandbytes dequantization is outside adamw4bit_b200")
    scheme_info(mode)
    if quant_state.blocksize != 128:
        raise NotImplementedError("the B200 codec uses 128-value blocks")
    N.require_cuda(codes, "dequantize")
    n = _numel(quant_state.shape)
    if n % 128:
        raise NotImplementedError("numel must be a multiple of the 128-value block")
    packed = packed_codes(codes, quant_state).contiguous()
    scales = quant_state.absmax.to(device=codes.device, dtype=torch.float32).contiguous()
    out = torch.empty(n, dtype=torch.float32, device=codes.device)
    N.check(N.lib().aw4_dequantize_blocks(prepared(mode), N.ptr(packed), N.ptr(scales), n,
                                          N.ptr(out), codes.device.index,
                                          N.stream_handle(codes.device)), "aw4_dequantize_blocks")
    return out.reshape(quant_state.shape).to(quant_state.dtype)


def apply_eden_correction_to_quant_state(x, codes, quant_state, mode):
    raise NotImplementedError("store-EDEN schemes are outside adamw4bit_b200")
