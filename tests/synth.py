"""Synthetic inputs of the large parity configurations, bit-identical on CPU and GPU.

BASELINE configurations 3-5 step hundreds of millions of values for tens of
steps.  Regenerating their gradients with ``torch.randn`` on the host of the
GPU box would take minutes per run, so every value here is a gather from one
fixed pool of normal deviates at an index given by an integer hash:

    value[i] = pool[hash(i ^ key(stream, step)) mod 2^22] * std

The pool (``torch.randn`` of 2^22 float32 from a seeded CPU generator) is made
once on the CPU and moved to the device; the hash uses int64 arithmetic whose
products stay below 2^63; the scale is one IEEE float32 multiply.  The same
values therefore come out of torch on the CPU (where the golden generator
feeds them to the reference) and on CUDA (where the tests feed them to the
fused step), and each 128-block is an i.i.d.-looking sample of N(0, std^2).

Outlier blocks (configuration 4: 1 % of 128-value blocks scaled by 100) are
chosen by the same hash over block indices.
"""

from __future__ import annotations

import hashlib

import torch

POOL_BITS = 22
POOL_SEED = 20260101
MASK32 = 0xFFFFFFFF
# multipliers below 2^31: an int64 product of a 32-bit value never overflows
_M = (0x7FEB352D, 0x5BD1E995, 0x2C1B3C6D)
KIND_PARAM, KIND_GRAD, KIND_OUTLIER = 1, 2, 3

_pools: dict[str, torch.Tensor] = {}


def pool(device) -> torch.Tensor:
    """The 2^22 standard normal deviates (float32), cached per device."""
    key = str(torch.device(device))
    if key not in _pools:
        if "cpu" not in _pools:
            g = torch.Generator().manual_seed(POOL_SEED)
            _pools["cpu"] = torch.randn(1 << POOL_BITS, generator=g, dtype=torch.float32)
        _pools[key] = _pools["cpu"].to(device)
    return _pools[key]


def pool_digest() -> str:
    return hashlib.sha256(pool("cpu").numpy().tobytes()).hexdigest()


def mix32_int(x: int) -> int:
    """The hash on a Python int (used for keys)."""
    x &= MASK32
    x = (x * _M[0]) & MASK32
    x ^= x >> 15
    x = (x * _M[1]) & MASK32
    x ^= x >> 13
    x = (x * _M[2]) & MASK32
    x ^= x >> 16
    return x


def mix32(x: torch.Tensor, tmp: torch.Tensor | None = None) -> torch.Tensor:
    """The same hash, in place, on an int64 tensor of values in [0, 2^32)."""
    tmp = torch.empty_like(x) if tmp is None else tmp[: x.numel()]
    for m, s in zip(_M, (15, 13, 16)):
        x.mul_(m).bitwise_and_(MASK32)
        torch.bitwise_right_shift(x, s, out=tmp)
        x.bitwise_xor_(tmp)
    return x


def key(stream: int, step: int, kind: int) -> int:
    return mix32_int(mix32_int(stream * 0x9E3779B1 + kind) ^ mix32_int(step * 0x85EBCA6B + 7))


def _chunk(device) -> int:
    # CPU: chunks small enough for the allocator to reuse their pages
    return (1 << 21) if torch.device(device).type == "cpu" else (1 << 26)


def normal(numel: int, stream: int, step: int, kind: int, std: float, device) -> torch.Tensor:
    """numel float32 values ~ N(0, std^2) (pool gather), identical on every device."""
    p = pool(device)
    out = torch.empty(numel, dtype=torch.float32, device=device)
    k = key(stream, step, kind)
    c = _chunk(device)
    x = torch.empty(min(c, max(numel, 1)), dtype=torch.int64, device=device)
    tmp = torch.empty_like(x)
    for a in range(0, numel, c):
        b = min(a + c, numel)
        xv = x[: b - a]
        torch.arange(a, b, dtype=torch.int64, device=device, out=xv)
        xv.bitwise_xor_(k)
        mix32(xv, tmp)
        xv.bitwise_and_((1 << POOL_BITS) - 1)
        torch.index_select(p, 0, xv, out=out[a:b])
    return out.mul_(std)


def outlier_mask(nblocks: int, stream: int, step: int, frac: float, device) -> torch.Tensor:
    """A boolean mask over 128-value blocks selecting about frac of them."""
    idx = torch.arange(nblocks, dtype=torch.int64, device=device) ^ key(stream, step, KIND_OUTLIER)
    return (mix32(idx).remainder_(1_000_000)) < int(round(frac * 1_000_000))


def init_param(shape, stream: int, dtype, device, std: float = 0.02) -> torch.Tensor:
    n = int(torch.Size(shape).numel())
    return normal(n, stream, 0, KIND_PARAM, std, device).view(shape).to(dtype)


def grad(shape, stream: int, step: int, std: float, dtype, device,
         outlier_frac: float = 0.0) -> torch.Tensor:
    n = int(torch.Size(shape).numel())
    g = normal(n, stream, step, KIND_GRAD, std, device)
    if outlier_frac > 0 and n % 128 == 0:
        flat = g.view(-1, 128)
        flat[outlier_mask(n // 128, stream, step, outlier_frac, device)] *= 100.0
    return g.view(shape).to(dtype)


def checksum(t: torch.Tensor) -> int:
    """Exact integer checksum of a tensor's bit patterns (sum of the 16- or
    32-bit words as int64, plus the same sum weighted by position mod 251),
    computed where the tensor lives."""
    t = t.detach().contiguous().reshape(-1)
    if t.dtype in (torch.bfloat16, torch.float16):
        t, mask = t.view(torch.int16), 0xFFFF
    elif t.dtype == torch.float32:
        t, mask = t.view(torch.int32), MASK32
    else:
        mask = None
    c = _chunk(t.device)
    s0 = torch.zeros((), dtype=torch.int64, device=t.device)
    s1 = torch.zeros((), dtype=torch.int64, device=t.device)
    w = torch.empty(min(c, max(t.numel(), 1)), dtype=torch.int64, device=t.device)
    pos = torch.empty_like(w)
    for a in range(0, t.numel(), c):
        b = min(a + c, t.numel())
        wv, pv = w[: b - a], pos[: b - a]
        wv.copy_(t[a:b])
        if mask is not None:
            wv.bitwise_and_(mask)
        s0 += wv.sum()
        torch.arange(a, b, dtype=torch.int64, device=t.device, out=pv)
        pv.remainder_(251)
        s1 += (wv.mul_(pv)).sum()
    return int(s0.item()) * 1000003 + int(s1.item())


# ---------------------------------------------------------------------------
# parameter sets of BASELINE configurations 3-5
# ---------------------------------------------------------------------------

def gpt2_small_shapes() -> list[tuple[int, ...]]:
    """GPT-2 small with an untied LM head (HF Conv1D weights are [in, out]):
    149 tensors, 163.0 M values, 51 of them with quantized state."""
    V, P, d = 50257, 1024, 768
    shapes: list[tuple[int, ...]] = [(V, d), (P, d)]
    for _ in range(12):
        shapes += [(d,), (d,), (d, 3 * d), (3 * d,), (d, d), (d,),
                   (d,), (d,), (d, 4 * d), (4 * d,), (4 * d, d), (d,)]
    shapes += [(d,), (d,), (d, V)]
    return shapes


def llama_1b_shapes() -> list[tuple[int, ...]]:
    """Llama-style 1B (vocab 32000, d 2048, 16 layers, ffn 5632, 32/8 heads,
    untied head): 147 tensors, 852.6 M values, 114 with quantized state."""
    V, d, L, ffn, kv = 32000, 2048, 16, 5632, 512
    shapes: list[tuple[int, ...]] = [(V, d)]
    for _ in range(L):
        shapes += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    shapes += [(d,), (V, d)]
    return shapes


def llama3_8b_subset_shapes() -> list[tuple[int, ...]]:
    """Llama-3-8B at real shapes, reduced to the embedding, one full decoder
    layer, the final norm and the head: 12 tensors, 1.27 G values."""
    V, d, ffn, kv = 128256, 4096, 14336, 1024
    return [(V, d), (d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,),
            (d,), (V, d)]
