"""The C-ABI library loads, exports every symbol include/adamw4bit_b200.h
declares, and its host-only pieces (struct layouts, aw4_scheme_prepare) are
right.  No GPU needed: nothing here launches a kernel."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from adamw4bit_b200 import _native as N
from adamw4bit_b200 import quantization as Q
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "adamw4bit_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int32_t|uint64_t|const char\*)\s+(aw4_\w+)\s*\(",
                                 text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    names = declared_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
        assert name in N.SIGNATURES, f"{name} has no ctypes signature"
    assert set(N.SIGNATURES) == set(names)
    assert lib.aw4_abi_version() == N.ABI_VERSION


def test_struct_layouts_match_header():
    # sizes follow from the C declarations (natural alignment, x86-64)
    assert ctypes.sizeof(N.Scheme) == 64 + 12 + N.LUT_BINS + 72 + 8 + 4
    assert ctypes.sizeof(N.Hyper) == 56
    assert ctypes.sizeof(N.QTensor) == 104
    assert ctypes.sizeof(N.FTensor) == 48


def _lut_search(s: N.Scheme, x: np.ndarray) -> np.ndarray:
    """numpy copy of the kernels' table search: exact bin floor((x+1)*bins/2)."""
    nb = s.lut_bins
    half = np.float32(nb // 2)
    lut = np.frombuffer(bytes(s.lut), dtype=np.uint8)[:nb].astype(np.int64)
    thr = np.array(list(s.thr), dtype=np.float32)
    b = np.floor(x.astype(np.float32) * half).astype(np.int64) + nb // 2
    last = int(lut[nb - 1])
    lut = np.append(lut, last + int(thr[last + 1] <= 1.0))   # edge x == 1
    k = lut[b]
    return k + (x >= thr[k + 1]).astype(np.int64)


def _literal_rtn(cb: np.ndarray, x: np.ndarray) -> np.ndarray:
    i = np.searchsorted(cb, x, side="left")
    left = np.clip(i - 1, 0, 15)
    right = np.clip(i, 0, 15)
    dl = np.abs((x - cb[left]).astype(np.float32))
    dr = np.abs((cb[right] - x).astype(np.float32))
    return np.where(dl < dr, left, right)


def _sample(rng, n=1 << 20) -> np.ndarray:
    words = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32)
    x = words.view(np.float32)
    x = x[np.isfinite(x) & (np.abs(x) <= 1)]
    return np.concatenate([x, rng.uniform(-1, 1, n).astype(np.float32),
                           np.array([-1.0, -0.0, 0.0, 1.0], np.float32)])


@pytest.mark.parametrize("scheme", sorted(Q.SCHEMES))
def test_scheme_tables_reproduce_the_reference_rounding_rule(scheme):
    info = Q.SCHEMES[scheme]
    s = Q.prepared(scheme)
    assert list(s.codebook) == list(info.codebook)
    rng = np.random.default_rng(7)
    x = _sample(rng)
    # values right around every table threshold
    thr = np.array([t for t in s.thr if np.isfinite(t)], np.float32)
    near = (thr.view(np.int32)[:, None] + np.arange(-50, 51)[None, :]).astype(np.int32)
    x = np.concatenate([x, near.reshape(-1).view(np.float32)])
    x = x[np.abs(x) <= 1]
    got = _lut_search(s, x)
    if info.round_mode == N.RTN:
        want = _literal_rtn(info.codebook, x)
    else:
        want = np.searchsorted(info.codebook, x, side="left")
    np.testing.assert_array_equal(got, want)


def test_bin_counts_are_the_coarsest_valid():
    assert Q.prepared("nf4").lut_bins == 32
    assert Q.prepared("dyn4_nz").lut_bins == 1024
    for scheme in Q.SCHEMES:
        assert Q.prepared(scheme).lut_bins in (32, 64, 128, 256, 512, 1024)


def test_zero_state_matches_oracle_init():
    for scheme, eden in (("nf4", False), ("dyn4_nz", True), ("dyn4_upd_sr_fp32read", False),
                         ("nf4_sr", False)):
        s = Q.prepared(scheme)
        packed, scales = O.init_zero(scheme, 128, eden=eden)
        assert packed[0] == (s.zero_code | (s.zero_code << 4))
        want = s.zero_scale_eden if eden else s.zero_scale
        assert np.float32(want).view(np.uint32) == scales[0].view(np.uint32)


def test_prepare_rejects_bad_codebooks():
    bad = np.linspace(0, 1, 16, dtype=np.float32)[::-1].copy()
    with pytest.raises(N.NativeError, match="invalid argument"):
        N.prepare_scheme(bad, N.RTN, False)
    with pytest.raises(N.NativeError, match="bad round mode"):
        N.prepare_scheme(Q.NF4, 7, False)
    dense = np.concatenate([np.linspace(0, 1e-3, 15, dtype=np.float32), [1.0]]).astype(np.float32)
    with pytest.raises(N.NativeError, match="unsupported"):
        N.prepare_scheme(dense, N.RTN, False)


def test_step_entry_point_validates_before_touching_the_gpu():
    """Bad arguments are rejected by the host checks, before any CUDA call."""
    t = (N.QTensor * 1)(N.QTensor(16, 16, 4, 4, 4, 4, None, None, 100, 0, 0, 0))
    h = (N.Hyper * 1)(N.Hyper())
    s = Q.prepared("nf4")
    rc = N.lib().aw4_step_quantized(s, Q.prepared("dyn4_nz"), 1, N.F32, N.F32, t, 1, h, 1, 0, 0, None)
    assert rc == N.AW4_ERR_INVALID
    assert b"multiple of 128" in N.lib().aw4_last_error()
    rc = N.lib().aw4_step_quantized(Q.prepared("dyn4_upd_sr_fp32read"), s, 0, N.F32, N.F32, t, 1,
                                    h, 1, 0, 0, None)
    assert rc == N.AW4_ERR_UNSUPPORTED
    t[0].numel = 128
    t[0].hyper = 3
    rc = N.lib().aw4_step_quantized(s, s, 0, N.F32, N.F32, t, 1, h, 1, 0, 0, None)
    assert rc == N.AW4_ERR_INVALID and b"hyper index" in N.lib().aw4_last_error()
    rc = N.lib().aw4_step_quantized(s, s, 0, N.BF16, N.F32, t, 1, h, 1, 0, 0, None)
    assert rc == N.AW4_ERR_UNSUPPORTED
