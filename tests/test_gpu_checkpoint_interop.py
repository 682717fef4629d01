"""Checkpoints exchanged with the reference itself (adamw.py:326-470).

Forward: the reference's own state_dict after 3 steps (saved by
tests/golden/make_golden_configs.py with the reference's eager step) loads
into this optimizer, which continues 3 steps on the GPU and must reproduce
the reference's digests of every packed code, block scale and FP32 moment at
every step, with parameters within rtol 1e-6.  For ZIP-SR the checkpoint's
version-1 RNG payload holds the reference's CPU generator states; the test
continues those generators in the reference's order and feeds the draws
through the optimizer's draws hook.

Reverse: this optimizer's state_dict after 3 GPU steps is loaded by the
reference (its offline install under baseline/_ref; skipped when absent),
which continues 3 steps on the CPU; its states must equal the reference's
own uninterrupted run.
"""

from __future__ import annotations

import hashlib
import io
import json
import os
import sys

import numpy as np
import pytest
import torch

from adamw4bit_b200 import ZEEDENAdamW4Bit, ZIPSRAdamW4Bit
from tests import synth as S

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
M2_OFFSET, MAX_SEED = 0x5E6F7789, (1 << 63) - 1
RECIPES = {"zeeden": ZEEDENAdamW4Bit, "zipsr": ZIPSRAdamW4Bit}


def _fixture(name):
    with open(os.path.join(GOLDEN, f"ckpt_{name}.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(GOLDEN, f"ckpt_{name}.npz")))
    sd = torch.load(os.path.join(GOLDEN, f"ckpt_{name}.pt"), map_location="cpu",
                    weights_only=True)
    return meta, arrays, sd


def _eligible(n):
    return n >= 4096 and n % 128 == 0


def _digests(state_of, params) -> dict:
    hs = {k: hashlib.sha256() for k in ("m1_code", "m1_absmax", "m2_code", "m2_absmax",
                                        "f_m1", "f_m2")}
    for p in params:
        st = state_of[p]
        if _eligible(p.numel()):
            parts = (("m1_code", st["m1_code"]), ("m1_absmax", st["m1_quant_state"].absmax),
                     ("m2_code", st["m2_code"]), ("m2_absmax", st["m2_quant_state"].absmax))
        else:
            parts = (("f_m1", st["m1"]), ("f_m2", st["m2"]))
        for k, t in parts:
            hs[k].update(t.detach().contiguous().cpu().numpy().tobytes())
    return {k: h.hexdigest() for k, h in hs.items()}


def _m2_draws(gen, params):
    """The reference's m2 update-SR uniforms of one step, in parameter order."""
    return {id(p): (None, torch.rand((p.numel() // 128, 128), generator=gen).reshape(-1).to(DEV))
            for p in params if _eligible(p.numel())}


@pytest.mark.parametrize("name", ["zeeden", "zipsr"])
def test_reference_checkpoint_loads_and_continues_bit_exact(name):
    meta, arrays, sd = _fixture(name)
    k, more = meta["k"], meta["more"]
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [torch.nn.Parameter(torch.from_numpy(arrays[f"s{k}_p{i}"]).to(DEV).view(s))
              for i, s in enumerate(shapes)]
    kw = {} if meta["quant_rng_seed"] is None else {"quant_rng_seed": meta["quant_rng_seed"]}
    opt = RECIPES[name](params, **kw)
    opt.load_state_dict(sd)
    gen = None
    if name == "zipsr":
        gen = torch.Generator()
        gen.set_state(sd["_quant_rng_state"]["states"]["m2"]["cpu"])
    for t in range(k + 1, k + more + 1):
        for i, p in enumerate(params):
            p.grad = S.grad(p.shape, i, t, meta["grad_std"], torch.float32, DEV)
        opt._draws_override = _m2_draws(gen, params) if gen is not None else None
        opt.step()
        rec = meta["per_step"][t - 1]
        got = _digests(opt.state, params)
        for key in got:
            assert got[key] == rec[key], f"{name} step {t}: {key}"
    for i, p in enumerate(params):
        np.testing.assert_allclose(p.detach().cpu().numpy(), arrays[f"s{k + more}_p{i}"],
                                   rtol=1e-6, atol=1e-9)


def _reference():
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "adamw4bit")):
        pytest.skip("the reference's offline install (baseline/_ref) is absent")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import adamw4bit
    return adamw4bit


@pytest.mark.parametrize("name", ["zeeden", "zipsr"])
def test_this_optimizers_checkpoint_continues_in_the_reference(name):
    """Our GPU state after k steps, saved with state_dict(), continues in the
    reference's own optimizer on the CPU exactly as the reference's
    uninterrupted run does.  ZIP-SR runs unseeded here: this optimizer's
    seeded checkpoints carry a Philox payload (version 2) that the reference
    refuses by design, so both sides draw from the global torch RNG."""
    ref = _reference()
    meta, arrays, _ = _fixture(name)
    k, more = meta["k"], meta["more"]
    shapes = [tuple(s) for s in meta["shapes"]]
    init = [S.init_param(s, i, torch.float32, "cpu") for i, s in enumerate(shapes)]
    ours = [torch.nn.Parameter(x.clone().to(DEV)) for x in init]
    theirs = [torch.nn.Parameter(x.clone()) for x in init]
    opt = RECIPES[name](ours)
    ref_cls = {"zeeden": ref.ZEEDENAdamW4Bit, "zipsr": ref.ZIPSRAdamW4Bit}[name]
    twin = ref_cls(theirs)                      # uninterrupted reference run
    torch.manual_seed(77)
    for t in range(1, k + 1):
        grads = [S.grad(s, i, t, meta["grad_std"], torch.float32, "cpu") for i, s in enumerate(shapes)]
        state = torch.get_rng_state()
        for p, g in zip(theirs, grads):
            p.grad = g
        twin.step()
        if name == "zipsr":   # the same global-RNG draws, in the reference's order
            after = torch.get_rng_state()
            torch.set_rng_state(state)
            draws = {}
            for p in ours:
                if _eligible(p.numel()):
                    if t == 1:
                        torch.rand((p.numel() // 128, 128))            # zero-state init
                    draws[id(p)] = (None, torch.rand((p.numel() // 128, 128)).reshape(-1).to(DEV))
            torch.set_rng_state(after)
            opt._draws_override = draws
        for p, g in zip(ours, grads):
            p.grad = g.to(DEV)
        opt.step()
    buf = io.BytesIO()
    torch.save(opt.state_dict(), buf)
    buf.seek(0)
    saved = torch.load(buf, map_location="cpu", weights_only=True)
    resumed = [torch.nn.Parameter(p.detach().cpu().clone()) for p in ours]
    cont = ref_cls(resumed)
    cont.load_state_dict(saved)
    assert _digests(cont.state, resumed) == _digests(twin.state, theirs)
    for t in range(k + 1, k + more + 1):
        grads = [S.grad(s, i, t, meta["grad_std"], torch.float32, "cpu") for i, s in enumerate(shapes)]
        state = torch.get_rng_state()
        for p, g in zip(theirs, grads):
            p.grad = g
        twin.step()
        torch.set_rng_state(state)
        for p, g in zip(resumed, grads):
            p.grad = g
        cont.step()
        assert _digests(cont.state, resumed) == _digests(twin.state, theirs), f"{name} step {t}"
        for a, b in zip(resumed, theirs):
            np.testing.assert_allclose(a.detach().numpy(), b.detach().numpy(), rtol=1e-6, atol=1e-9)
