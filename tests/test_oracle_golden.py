"""Pins the CPU oracle against the reference's own outputs (tests/golden/).

The oracle (oracle/aw4_oracle.c) is the checker for every GPU parity test, so
it is trusted only after matching what the reference produced on the same
inputs: codebooks, codec cases (RTN, value-SR and update-SR given the
reference's uniforms, EDEN, the zero floor and the scale floor) and optimizer
trajectories.  Codes and block scales must be bit-exact; parameters must agree
within rtol=1e-6 (the reference's CPU sqrt is MKL VML, not correctly rounded,
so the denominator may differ by one ulp in rare elements).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import golden_io as G

PARAM_RTOL = 1e-6
PARAM_ATOL = 1e-9


def test_codebooks_match_reference():
    with open(os.path.join(G.GOLDEN, "codebooks.json")) as f:
        ref = json.load(f)
    for scheme, words in ref.items():
        cb = O.SCHEMES[scheme][0]
        assert [int(w) for w in cb.view(np.uint32)] == words, scheme


def test_codec_cases_bit_exact():
    with open(os.path.join(G.GOLDEN, "codec_cases.json")) as f:
        meta = json.load(f)
    arrays = np.load(os.path.join(G.GOLDEN, "codec_cases.npz"))
    for case in meta:
        tag, scheme = case["tag"], case["scheme"]
        codes, scales = O.quantize(arrays[f"{tag}_x"], scheme, eden=case["eden"],
                                   draws=arrays[f"{tag}_draws"],
                                   bias_correction=case["bias_correction"], eps=case["eps"])
        np.testing.assert_array_equal(codes, arrays[f"{tag}_codes"], err_msg=tag + scheme)
        np.testing.assert_array_equal(scales.view(np.uint32),
                                      arrays[f"{tag}_scales"].view(np.uint32), err_msg=tag)


def test_nibble_order_kat():
    """tests/quantization/test_utils.py:92-101 of the reference: [1,2,15] -> [0x21, 0x0F]."""
    arrays = np.load(os.path.join(G.GOLDEN, "codec_cases.npz"))
    np.testing.assert_array_equal(O.pack(arrays["pack_in"]), arrays["pack_out"])
    np.testing.assert_array_equal(O.unpack(arrays["pack_out"], 3), arrays["pack_in"])


def _np_param(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.numpy().reshape(-1).copy()
    return t.view(torch.int16).numpy().reshape(-1).view(np.uint16).copy()


def _f32(a: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    if dtype == torch.float32:
        return a
    return torch.from_numpy(a.view(np.int16)).view(dtype).float().numpy()


_DT = {torch.float32: O.F32, torch.bfloat16: O.BF16, torch.float16: O.F16}


def run_oracle_trajectory(meta: dict, on_step=None):
    """Run the oracle over a fixture's replayed inputs; yields per-step state."""
    rep = G.Replay(meta)
    params = [_np_param(p) for p in rep.init_params()]
    state = []
    for p, s in zip(params, rep.shapes):
        n = int(np.prod(s))
        if G.eligible(n):
            c1, s1 = O.init_zero(rep.m1_scheme, n)
            c2, s2 = O.init_zero(rep.m2_scheme, n, eden=rep.eden)
            state.append({"m1_code": c1, "m1_absmax": s1, "m2_code": c2, "m2_absmax": s2})
        else:
            state.append({"m1": np.zeros(n, np.float32), "m2": np.zeros(n, np.float32)})
    for t in range(1, meta["steps"] + 1):
        inp = rep.next()
        for i, (p, st) in enumerate(zip(params, state)):
            g = _np_param(inp.grads[i])
            m1_scheme = inp.m1_scheme if i == 0 else rep.m1_scheme
            cfg = O.make_cfg(m1_scheme=m1_scheme, m2_scheme=rep.m2_scheme, eden=rep.eden,
                             lr=meta["lr"], betas=meta["betas"], eps=meta["eps"],
                             weight_decay=meta["weight_decay"], step=t,
                             param_dtype=_DT[rep.p_dtype], grad_dtype=_DT[rep.g_dtype])
            if "m1_code" in st:
                O.step(cfg, p, g, st["m1_code"], st["m1_absmax"], st["m2_code"], st["m2_absmax"],
                       inp.m1_draws[i], inp.m2_draws[i])
            else:
                O.step_fp32_state(cfg, p, g, st["m1"], st["m2"])
        if on_step is not None:
            on_step(t, inp, params, state)
    return params, state


TRAJS = ["zeeden_f32_small", "zipsr_f32_small", "zeeden_switch_small", "zipsr_bf16_outliers",
         "zeeden_f32p_bf16g", "zeeden_f16"]


@pytest.mark.parametrize("name", TRAJS)
def test_oracle_trajectory_matches_reference(name):
    meta, arrays = G.load_traj(name)
    rep_dtype = G.DTYPES[meta["p_dtype"]]

    def check(t, inp, params, state):
        rec = meta["per_step"][t - 1]
        for i, g in enumerate(inp.grads):
            assert G.sha(g) == rec["grad_sha"][i], f"gradient recipe drifted at step {t}"
        st = state[0]
        for key in ("m1_code", "m1_absmax", "m2_code", "m2_absmax"):
            assert G.sha_np(st[key]) == rec[key], f"{name} step {t} {key}"
        sample = _f32(params[0], rep_dtype)[::meta["sample_stride"]]
        np.testing.assert_allclose(sample, arrays[f"s{t}_param_sample"], rtol=PARAM_RTOL,
                                   atol=PARAM_ATOL, err_msg=f"{name} step {t}")
        if f"s{t}_param" in arrays:
            np.testing.assert_allclose(_f32(params[0], rep_dtype), arrays[f"s{t}_param"],
                                       rtol=PARAM_RTOL, atol=PARAM_ATOL)
        for i in range(1, len(params)):
            if f"s{t}_small{i}_param" in arrays:
                np.testing.assert_allclose(_f32(params[i], rep_dtype),
                                           arrays[f"s{t}_small{i}_param"], rtol=PARAM_RTOL,
                                           atol=PARAM_ATOL)
                np.testing.assert_allclose(state[i]["m1"], arrays[f"s{t}_small{i}_m1"],
                                           rtol=0, atol=0)
                np.testing.assert_allclose(state[i]["m2"], arrays[f"s{t}_small{i}_m2"],
                                           rtol=0, atol=0)

    run_oracle_trajectory(meta, on_step=check)


@pytest.mark.parametrize("name", ["zeeden_f32_c1", "zipsr_f32_c2"])
def test_oracle_full_size_trajectory_matches_reference(name):
    """BASELINE configs 1 and 2 at full size (16.8M values, 10 steps)."""
    if not G.exists(name):
        pytest.skip("full-size digests not generated")
    meta, arrays = G.load_traj(name)

    def check(t, inp, params, state):
        rec = meta["per_step"][t - 1]
        st = state[0]
        for key in ("m1_code", "m1_absmax", "m2_code", "m2_absmax"):
            assert G.sha_np(st[key]) == rec[key], f"{name} step {t} {key}"
        np.testing.assert_allclose(params[0][::meta["sample_stride"]], arrays[f"s{t}_param_sample"],
                                   rtol=PARAM_RTOL, atol=PARAM_ATOL)

    run_oracle_trajectory(meta, on_step=check)


@pytest.mark.parametrize("name", ["nf4_lookahead", "nf4_nextbc", "nf4_lin4_fp32read",
                                  "fp32m1_zipsr", "fp32m1_zeeden", "fp32m1_lookahead"])
def test_oracle_scheme_pairs_match_reference(name):
    """Scheme pairs through the reference's QuantizedAdamW, 6 steps
    (tests/golden/make_golden_configs.py): the fp32-read update-SR m2 schemes
    next to an nf4 m1 (dyn4_lookahead_sr and its nextbc alias store against
    the next step's bias correction c_{t+1}, lin4_upd_sr_fp32read against
    c_t; adamw.py:112-116, 655-683), and an FP32 m1 next to a 4-bit m2
    (adamw.py:510-521).  The oracle, fed the reference's m2 draws, must
    reproduce every digest of codes, scales and FP32 moments."""
    import hashlib

    from tests import synth as S
    with open(os.path.join(G.GOLDEN, f"mixed_{name}.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(G.GOLDEN, f"mixed_{name}.npz")))
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [S.init_param(s, i, torch.float32, "cpu").numpy().reshape(-1).copy()
              for i, s in enumerate(shapes)]
    fp32_m1 = meta["m1_scheme"] == "fp32"
    state = []
    for p in params:
        if G.eligible(p.size):
            c2, s2 = O.init_zero(meta["m2_scheme"], p.size, eden=meta["eden"])
            if fp32_m1:
                state.append({"m1": np.zeros(p.size, np.float32), "m2_code": c2, "m2_absmax": s2})
            else:
                c1, s1 = O.init_zero(meta["m1_scheme"], p.size)
                state.append({"m1_code": c1, "m1_absmax": s1, "m2_code": c2, "m2_absmax": s2})
        else:
            state.append({"m1": np.zeros(p.size, np.float32), "m2": np.zeros(p.size, np.float32)})
    sr = O.SCHEMES[meta["m2_scheme"]][1] != O.RTN
    seed = meta["quant_rng_seed"]
    gen = torch.Generator().manual_seed((seed + G.M2_OFFSET) % ((1 << 63) - 1)) if sr else None
    for t in range(1, meta["steps"] + 1):
        cfg = O.make_cfg(m1_scheme=meta["m1_scheme"], m2_scheme=meta["m2_scheme"],
                         eden=meta["eden"], lr=1e-3, betas=(0.9, 0.95), eps=1e-8,
                         weight_decay=0.1, step=t, param_dtype=O.F32, grad_dtype=O.F32)
        for i, (p, st) in enumerate(zip(params, state)):
            g = S.grad(shapes[i], i, t, meta["grad_std"], torch.float32, "cpu").numpy().reshape(-1)
            if "m2_code" in st:
                d2 = None
                if gen is not None:
                    rows = (p.size // 128, 128)
                    if t == 1:
                        torch.rand(rows, generator=gen)             # zero-state init
                    d2 = torch.rand(rows, generator=gen).numpy().reshape(-1).copy()
                if fp32_m1:
                    O.step_fp32_m1(cfg, p, g.copy(), st["m1"], st["m2_code"], st["m2_absmax"], d2)
                else:
                    O.step(cfg, p, g.copy(), st["m1_code"], st["m1_absmax"], st["m2_code"],
                           st["m2_absmax"], None, d2)
            else:
                O.step_fp32_state(cfg, p, g.copy(), st["m1"], st["m2"])
        hs = {k: hashlib.sha256() for k in ("m1_code", "m1_absmax", "m2_code", "m2_absmax",
                                            "f_m1", "f_m2")}
        for st in state:
            for key, arr in st.items():
                hs[key if "_" in key else f"f_{key}"].update(arr.tobytes())
        rec = meta["per_step"][t - 1]
        for k, h in hs.items():
            assert h.hexdigest() == rec[k], f"{name} step {t}: {k}"
    for i, p in enumerate(params):
        np.testing.assert_allclose(p, arrays[f"s{meta['steps']}_p{i}"].reshape(-1),
                                   rtol=PARAM_RTOL, atol=PARAM_ATOL)
