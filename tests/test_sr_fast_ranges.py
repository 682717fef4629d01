"""The range facts behind the fast update-SR encoder, checked on the CPU.

The step kernel computes the preconditioner-space SR rule (quantization.py:
336-377) with Markstein divisions and Newton-Raphson reciprocal and square
root instead of the IEEE operations.  That is exact only where the operands
stay in certain ranges, and the kernel then also drops the reference's clamp
of p to [0, 1].  The host enables the fast encoder only for bias in
[2^-40, 1], eps in [2^-60, 2^25] and block scales up to 2^26, with values 0
or >= 2^-100 (the warp vote).  This file draws many such configurations and
checks, with IEEE float32 arithmetic (numpy), every fact the exactness
argument uses:

* every level preconditioner f lies in [2^-34, 2^60];
* s*x is 0 or at least 2^-101;
* for an interval the reference treats as valid, the divisor f[l] - f[r] is
  at least 2^-57, and the numerator fx - f[r] lies in [0, divisor] and is 0
  or at least 2^-57, so p lies in [0, 1] before the clamp.

The GPU tests compare the kernel with the oracle bit for bit; this test pins
the premises of that design independently of the hardware.
"""

from __future__ import annotations

import numpy as np
import pytest

from adamw4bit_b200.quantization import SCHEMES

F = np.float32


def _precond(s, level, bias, eps):
    """1 / (sqrt(max(s * l / bias, 0)) + eps) in IEEE float32 (quantization.py:356-358)."""
    t = (F(s) * level.astype(F)).astype(F)
    t = (t / F(bias)).astype(F)
    t = np.maximum(t, F(0))
    r = np.sqrt(t).astype(F)
    return (F(1) / (r + F(eps)).astype(F)).astype(F)


@pytest.mark.parametrize("scheme", ["dyn4_upd_sr_fp32read", "lin4_upd_sr_fp32read"])
def test_fast_update_sr_ranges(scheme):
    cb = SCHEMES[scheme].codebook.astype(F)
    rng = np.random.default_rng(20261202)
    lo57 = F(2.0 ** -57)
    for _ in range(300):
        bias = F(2.0 ** rng.uniform(-40, 0))
        eps = F(2.0 ** rng.uniform(-60, 25))
        s = F(2.0 ** rng.uniform(np.log2(1e-12), 26))
        f = _precond(s, cb, bias, eps)
        assert (f >= F(2.0 ** -34)).all() and (f <= F(2.0 ** 60)).all()

        # values of one block: v = x0 * s, kept when 0 or >= 2^-100 (the vote),
        # plus the levels themselves and zeros; x = RN(v / s) as the kernel has it
        x0 = np.concatenate([rng.random(2048).astype(F), cb, np.zeros(4, F),
                             (2.0 ** rng.uniform(-60, 0, 256)).astype(F)])
        v = (x0 * s).astype(F)
        v = v[(v == 0) | (v >= F(2.0 ** -100))]
        x = (v / s).astype(F)
        t1 = (s * x).astype(F)
        assert ((t1 == 0) | (t1 >= F(2.0 ** -101))).all()

        idx = np.searchsorted(cb, x, side="left")
        lo, hi = np.maximum(idx - 1, 0), np.minimum(idx, 15)
        fx = _precond(s, x, bias, eps)
        den = (f[lo] - f[hi]).astype(F)
        valid = ((cb[hi] - cb[lo]).astype(F) > 0) & (den > 0)
        num = (fx - f[hi]).astype(F)
        assert (den[valid] >= lo57).all()
        nv = num[valid]
        assert ((nv == 0) | (nv >= lo57)).all()
        assert (nv >= 0).all() and (nv <= den[valid]).all()
        p = (nv / den[valid]).astype(F)
        assert ((p >= 0) & (p <= 1)).all()
