"""Device arithmetic behind the step kernel's fast path, and the fast path's
edge values, against IEEE and the CPU oracle.

The fast denominator/update path builds RN(1/b) and RN(sqrt(x)) from the
hardware approximations, and divides by Markstein's method under per-lane
bounds.  These tests check the two functions on every float32 of their
domains, then push values at and beyond every bound through the fused step:
zero moments of both signs, signed-zero parameters, tiny and subnormal
moments, moments beyond the fast bounds, overflow to inf/NaN, and
hyper-parameters that switch the fast path off.  Codes, scales and parameters
must equal the oracle's bit for bit.
"""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from adamw4bit_b200 import _native as N
from adamw4bit_b200 import quantization as Q
from oracle import oracle as O
from tests import abi_step as A
from tests.test_gpu_parity import _assert_state_equal

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
_ODT = {torch.float32: O.F32, torch.bfloat16: O.BF16, torch.float16: O.F16}


def test_selfcheck_math_is_exact_on_every_float32():
    counts = torch.zeros(2, dtype=torch.int64, device=DEV)
    N.check(N.lib().aw4_selfcheck_math(N.ptr(counts), DEV.index, N.stream_handle(DEV)),
            "aw4_selfcheck_math")
    torch.cuda.synchronize()
    assert counts.tolist() == [0, 0], f"mismatches (reciprocal, square root): {counts.tolist()}"


def _edge_inputs(rng: np.random.Generator, n_blocks: int):
    """Parameters and one gradient pattern per 128-value block."""
    n = n_blocks * 128
    p = (rng.standard_normal(n) * 0.02).astype(np.float32)
    g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    blocks = g.reshape(n_blocks, 128)
    pb = p.reshape(n_blocks, 128)
    pattern = [
        lambda b, q: (b.fill(0.0), q.__setitem__(slice(0, 64), -0.0)),      # zero grads, -0 params
        lambda b, q: b.__imul__(1e-35),                                      # tiny m1, subnormal g^2
        lambda b, q: b.__imul__(1e-39),                                      # subnormal grads
        lambda b, q: b.__imul__(1e15),                                       # m2 beyond the fast bound
        lambda b, q: b.__imul__(1e23),                                       # g^2 overflows to inf
        lambda b, q: (b.__setitem__(slice(0, 128, 9), 0.0),                  # zeros among normals
                      b.__setitem__(slice(3, 128, 11), 1e-33)),              # and tiny values
        lambda b, q: (q.fill(0.0), q.__setitem__(slice(1, 128, 2), -0.0)),   # signed-zero params
        lambda b, q: (b.__setitem__(0, 50.0), q.__setitem__(slice(0, 128), 1e-40)),  # tiny params
        lambda b, q: b.__imul__(np.float32(np.exp(rng.standard_normal() * 4))),
    ]
    for k in range(n_blocks):
        pattern[k % len(pattern)](blocks[k], pb[k])
    return p, g


HYPERS = [
    # (lr, betas, eps, weight_decay)
    (1e-3, (0.9, 0.95), 1e-8, 0.1),
    (1e-3, (0.9, 0.999), 0.0, 0.0),          # eps = 0: fast path off
    (3e-2, (0.5, 0.99999), 1e-30, 0.01),     # eps below 2^-100: fast path off
    (1e-4, (0.9, 0.95), 1.0, 0.1),           # large eps
    (1e-3, (0.0, 0.0), 1e-8, 0.0),           # betas of zero: bc == 1
    (10.0, (0.9, 0.95), 1e-6, 0.5),          # large step
]


@pytest.mark.parametrize("p_dtype,g_dtype", [(torch.float32, torch.float32),
                                             (torch.float32, torch.bfloat16),
                                             (torch.bfloat16, torch.bfloat16),
                                             (torch.float16, torch.float16)])
@pytest.mark.parametrize("m1,m2,eden", [("nf4", "dyn4_nz", True),
                                         ("nf4", "dyn4_upd_sr_fp32read", False),
                                         ("nf4", "lin4", False)])
@pytest.mark.parametrize("hi", range(len(HYPERS)))
def test_update_edge_values_bit_exact(m1, m2, eden, p_dtype, g_dtype, hi):
    lr, betas, eps, wd = HYPERS[hi]
    rng = np.random.default_rng(zlib.crc32(f"{m1}/{m2}/{p_dtype}/{g_dtype}/{hi}".encode()))
    n_blocks = 18
    n = n_blocks * 128
    p_np, g_np = _edge_inputs(rng, n_blocks)
    p = torch.from_numpy(p_np).to(p_dtype)
    st = A.QTensorState(p.to(DEV), m1, m2, eden)
    c1, s1 = O.init_zero(m1, n)
    c2, s2 = O.init_zero(m2, n, eden=eden)
    pr = A.to_np_bits(p)
    keys = (O.stream_key(5, O.M1_OFFSET), O.stream_key(5, O.M2_OFFSET))
    next_bias = Q.SCHEMES[m2].next_bias
    for t in (1, 2, 3):
        g = torch.from_numpy(g_np * np.float32(1.0 + 0.25 * t)).to(g_dtype)
        hy = [A.hyper(t, lr=lr, betas=betas, eps=eps, weight_decay=wd, next_bias=next_bias,
                      m1_key=keys[0], m2_key=keys[1])]
        A.step([st], [g.to(DEV)], m1_scheme=m1, m2_scheme=m2, eden=eden, hypers=hy)
        cfg = O.make_cfg(m1_scheme=m1, m2_scheme=m2, eden=eden, lr=lr, betas=betas, eps=eps,
                         weight_decay=wd, step=t, param_dtype=_ODT[p_dtype],
                         grad_dtype=_ODT[g_dtype], m1_key=keys[0], m2_key=keys[1])
        O.step(cfg, pr, A.to_np_bits(g), c1, s1, c2, s2)
        torch.cuda.synchronize()
        _assert_state_equal(st, c1, s1, c2, s2, pr, what=f"step {t}")
