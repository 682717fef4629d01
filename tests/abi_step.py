"""Test-side driver of the C ABI (aw4_step_quantized / aw4_step_fp32_state).

Builds the descriptor arrays by hand from torch CUDA tensors, so parity tests
exercise the exact boundary a foreign caller (C, cgo, JNI) would use.
"""

from __future__ import annotations

import numpy as np
import torch

from adamw4bit_b200 import _native as N
from adamw4bit_b200 import quantization as Q
from adamw4bit_b200.optimizer import hyper_scalars


class QTensorState:
    """Device buffers of one quantized tensor: param, grad, codes, scales."""

    def __init__(self, param: torch.Tensor, m1_scheme: str, m2_scheme: str, eden: bool):
        n = param.numel()
        self.param = param
        self.m1_codes = torch.empty(n // 2, dtype=torch.uint8, device=param.device)
        self.m2_codes = torch.empty(n // 2, dtype=torch.uint8, device=param.device)
        self.m1_scales = torch.empty(n // 128, dtype=torch.float32, device=param.device)
        self.m2_scales = torch.empty(n // 128, dtype=torch.float32, device=param.device)
        dev = param.device
        for codes, scales, scheme, e in ((self.m1_codes, self.m1_scales, m1_scheme, False),
                                         (self.m2_codes, self.m2_scales, m2_scheme, eden)):
            N.check(N.lib().aw4_init_zero_state(Q.prepared(scheme), int(e), N.ptr(codes),
                                                N.ptr(scales), n, dev.index,
                                                N.stream_handle(dev)), "init")


def hyper(step: int, *, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
          next_bias=False, m1_key=0, m2_key=0) -> N.Hyper:
    h = hyper_scalars(lr, betas[0], betas[1], eps, weight_decay, step, next_bias)
    return N.Hyper(h["w1"], h["w2"], h["decay"], h["neg_step"], h["sqrt_bc2"], h["eps"],
                   h["sr_bias"], step, m1_key, m2_key)


def step(states: list[QTensorState], grads: list[torch.Tensor], *, m1_scheme: str,
         m2_scheme: str, eden: bool, hypers: list[N.Hyper], hyper_index: list[int] | None = None,
         ordinals: list[int] | None = None, elem_offsets: list[int] | None = None,
         m1_draws=None, m2_draws=None) -> None:
    n = len(states)
    hyper_index = hyper_index or [0] * n
    ordinals = ordinals or list(range(n))
    elem_offsets = elem_offsets or [0] * n
    m1_draws = m1_draws or [None] * n
    m2_draws = m2_draws or [None] * n
    descs = []
    for i, s in enumerate(states):
        descs.append(N.QTensor(N.ptr(s.param), N.ptr(grads[i]), N.ptr(s.m1_codes),
                               N.ptr(s.m1_scales), N.ptr(s.m2_codes), N.ptr(s.m2_scales),
                               N.ptr(m1_draws[i]), N.ptr(m2_draws[i]), s.param.numel(),
                               elem_offsets[i], ordinals[i], hyper_index[i]))
    dev = states[0].param.device
    pdt = N.DTYPE_CODES[states[0].param.dtype]
    gdt = N.DTYPE_CODES[grads[0].dtype]
    arr = (N.QTensor * n)(*descs)
    harr = (N.Hyper * len(hypers))(*hypers)
    N.check(N.lib().aw4_step_quantized(Q.prepared(m1_scheme), Q.prepared(m2_scheme), int(eden),
                                       pdt, gdt, arr, n, harr, len(hypers), 0, dev.index,
                                       N.stream_handle(dev)), "aw4_step_quantized")


def step_fp32(params, grads, m1s, m2s, hypers: list[N.Hyper]) -> None:
    descs = [N.FTensor(N.ptr(p), N.ptr(g), N.ptr(a), N.ptr(b), p.numel(), 0, 0)
             for p, g, a, b in zip(params, grads, m1s, m2s)]
    dev = params[0].device
    arr = (N.FTensor * len(descs))(*descs)
    harr = (N.Hyper * len(hypers))(*hypers)
    N.check(N.lib().aw4_step_fp32_state(N.DTYPE_CODES[params[0].dtype], N.DTYPE_CODES[grads[0].dtype],
                                        arr, len(descs), harr, len(hypers), dev.index,
                                        N.stream_handle(dev)), "aw4_step_fp32_state")


def to_np_bits(t: torch.Tensor) -> np.ndarray:
    """Raw storage of a CUDA tensor as numpy (float32 or uint16 bits)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return t.numpy().reshape(-1).copy()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().reshape(-1).view(np.uint16).copy()
    return t.numpy().reshape(-1).copy()
