"""Golden fixtures for BASELINE configurations 3, 4 and 5 and for checkpoint
interchange, made by running the REFERENCE (nubank/adamw4bit, eager path,
optimized=False) on the CPU.

    python tests/golden/make_golden_configs.py --reference <reference checkout> \
        [--only c3,c4,c5,ckpt,mixed] [--threads N]

Inputs come from tests/synth.py (hash-indexed pool gathers that are
bit-identical on the CPU and on CUDA), so the GPU tests rebuild every
gradient on the device.  Per step each fixture records:

  * SHA-256 of the m1/m2 packed codes and block scales of every quantized
    tensor (concatenated in parameter order), and of the FP32 moments of the
    other tensors;
  * an exact checksum of every gradient (drift guard for the input recipe);
  * per-tensor float64 sums of the parameters, and at a few steps a strided
    sample of all parameters.

ZIP-SR (configuration 4) also records SR flips.  The reference's CPU square
root (MKL VML, not correctly rounded) enters the preconditioner-space SR
probability; where that moves the probability across the uniform draw, the
reference's m2 code differs from the one IEEE arithmetic gives.  The
generator recomputes each SR call with the same torch operations but an IEEE
square root and lists every position whose code differs: (step, parameter,
element, reference code, IEEE code).  The GPU test checks that the kernel
gives the IEEE code there, then writes the reference's code back so the two
states stay identical.

``ckpt`` saves the reference's ``state_dict()`` after 3 steps of each recipe
(adamw.py:326-362) and the digests of 3 further steps, for the test that
loads a reference checkpoint into this optimizer.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from tests import synth as S  # noqa: E402

SAMPLES_PER_STEP = 16384


def eligible(n: int) -> bool:
    return n >= 4096 and n % 128 == 0


class Digest:
    """SHA-256 over several tensors' bytes, in order."""

    def __init__(self):
        self.h = hashlib.sha256()

    def add(self, t: torch.Tensor) -> None:
        t = t.detach().contiguous().cpu()
        if t.dtype in (torch.bfloat16, torch.float16):
            t = t.view(torch.int16)
        self.h.update(t.numpy().tobytes())

    def hex(self) -> str:
        return self.h.hexdigest()


def state_digests(opt, params, quantized) -> dict:
    d = {k: Digest() for k in ("m1_code", "m1_absmax", "m2_code", "m2_absmax", "f_m1", "f_m2")}
    for p, q in zip(params, quantized):
        st = opt.state[p]
        if q:
            d["m1_code"].add(st["m1_code"])
            d["m1_absmax"].add(st["m1_quant_state"].absmax)
            d["m2_code"].add(st["m2_code"])
            d["m2_absmax"].add(st["m2_quant_state"].absmax)
        else:
            d["f_m1"].add(st["m1"])
            d["f_m2"].add(st["m2"])
    return {k: v.hex() for k, v in d.items()}


class FlipRecorder:
    """Wraps the reference's preconditioner-space SR rule (quantization.py:327-377)
    to find the codes that an IEEE square root would round differently."""

    def __init__(self, quant_module):
        self.cls = quant_module._UpdateUnbiasedStochasticCodebookQuantizationStrategy
        self.orig = self.cls.quantize
        self.schedule: list[tuple[int, str]] = []
        self.calls = 0
        self.flips: list[tuple[int, int, int, int, int]] = []
        self.step = 0
        rec = self

        def wrapped(strategy, scaled_blocked, generator=None, *, block_scales=None,
                    bias_correction=None, eps=None):
            state = generator.get_state() if generator is not None else torch.get_rng_state()
            codes = rec.orig(strategy, scaled_blocked, generator, block_scales=block_scales,
                             bias_correction=bias_correction, eps=eps)
            rec.check(strategy, scaled_blocked, state, block_scales, bias_correction, eps, codes)
            return codes

        self.cls.quantize = wrapped

    def restore(self):
        self.cls.quantize = self.orig

    def begin_step(self, step: int, schedule: list[tuple[int, str]]) -> None:
        self.step, self.schedule, self.calls = step, schedule, 0

    def end_step(self) -> None:
        assert self.calls == len(self.schedule), (self.calls, len(self.schedule))

    def check(self, strategy, x, gen_state, block_scales, bias_correction, eps, codes):
        pidx, what = self.schedule[self.calls]
        self.calls += 1
        gen = torch.Generator()
        gen.set_state(gen_state)
        u = torch.rand(x.shape, generator=gen, dtype=torch.float32)
        cb = strategy._get_codebook(x.device)
        idx = torch.searchsorted(cb, x)
        left = (idx - 1).clamp_(min=0)
        right = idx.clamp_(max=cb.numel() - 1)
        lv, rv = cb[left], cb[right]
        width = rv - lv
        scales = block_scales.to(torch.float32).unsqueeze(1)
        bias = max(float(bias_correction) if bias_correction is not None else 1.0, 1e-12)
        adam_eps = float(eps) if eps is not None else 1e-8

        def pre(levels):
            v = (scales * levels.float() / bias).clamp_min(0.0)
            # IEEE float32 square root: the double root rounded to float32 is
            # correctly rounded for every float32 input
            return 1.0 / (v.double().sqrt().float() + adam_eps)

        fl, fr, fx = pre(lv), pre(rv), pre(x.float())
        denom = fl - fr
        prob = (fx - fr) / denom.clamp_min(1e-30)
        prob = torch.where((width > 0) & (denom > 0), prob, torch.ones_like(prob)).clamp_(0.0, 1.0)
        ieee = torch.where(u < prob, left, right).to(torch.uint8)
        diff = torch.nonzero(ieee.reshape(-1) != codes.reshape(-1)).reshape(-1)
        if diff.numel():
            assert what == "step", "flip while quantizing the zero state"
            ref = codes.reshape(-1)[diff]
            ie = ieee.reshape(-1)[diff]
            for e, r, i in zip(diff.tolist(), ref.tolist(), ie.tolist()):
                self.flips.append((self.step, pidx, e, r, i))


def run_config(ref, quant, name: str, *, shapes, recipe: str, p_dtype, g_dtype, steps: int,
               grad_std: float, quant_rng_seed, outlier_frac: float = 0.0, switch_at=None,
               head=None, sample_steps=(), lr=1e-3, betas=(0.9, 0.95), eps=1e-8, wd=0.1):
    cls = {"ze-eden": ref.ZEEDENAdamW4Bit, "zip-sr": ref.ZIPSRAdamW4Bit}[recipe]
    t0 = time.time()
    params = [torch.nn.Parameter(S.init_param(s, i, p_dtype, "cpu")) for i, s in enumerate(shapes)]
    if g_dtype != p_dtype:
        for p in params:
            p.grad_dtype = None   # torch >= 2.10: opt in to gradients of another dtype
    kw = dict(lr=lr, betas=betas, eps=eps, weight_decay=wd)
    if quant_rng_seed is not None:
        kw["quant_rng_seed"] = quant_rng_seed
    opt = cls(params, **kw)
    numels = [p.numel() for p in params]
    quantized = [eligible(n) for n in numels]
    total = sum(numels)
    stride = max(1, total // SAMPLES_PER_STEP) | 1
    meta = {
        "name": name, "recipe": recipe, "shapes": [list(s) for s in shapes],
        "p_dtype": str(p_dtype).replace("torch.", ""), "g_dtype": str(g_dtype).replace("torch.", ""),
        "steps": steps, "grad_std": grad_std, "outlier_frac": outlier_frac,
        "quant_rng_seed": quant_rng_seed, "switch_at": switch_at, "head": head,
        "lr": lr, "betas": list(betas), "eps": eps, "weight_decay": wd,
        "sample_steps": list(sample_steps), "sample_stride": stride,
        "synth": {"pool_bits": S.POOL_BITS, "pool_seed": S.POOL_SEED,
                  "pool_sha256": S.pool_digest(), "param_std": 0.02},
        "values": total, "tensors": len(shapes), "quantized_tensors": int(sum(quantized)),
        "reference": "adamw4bit eager step (optimized=False) on CPU, "
                     f"torch {torch.__version__}, {torch.get_num_threads()} threads",
        "per_step": [],
    }
    arrays = {"param_sums": np.zeros((steps, len(shapes)), np.float64),
              "param_abs_sums": np.zeros((steps, len(shapes)), np.float64)}
    flips = FlipRecorder(quant) if recipe == "zip-sr" else None
    try:
        for t in range(1, steps + 1):
            ts = time.time()
            if switch_at is not None and t == switch_at:
                opt.set_m1_quant_scheme_for_parameters([params[head]], "nf4_sr")
            gsum = 0
            for i, p in enumerate(params):
                p.grad = S.grad(p.shape, i, t, grad_std, g_dtype, "cpu", outlier_frac)
                gsum += (i + 1) * S.checksum(p.grad)
            if flips is not None:
                sched = []
                for i, q in enumerate(quantized):
                    if q:
                        sched += ([(i, "init")] if t == 1 else []) + [(i, "step")]
                flips.begin_step(t, sched)
            opt.step()
            if flips is not None:
                flips.end_step()
            rec = {"step": t, "grad_checksum": str(gsum)}
            rec.update(state_digests(opt, params, quantized))
            for i, p in enumerate(params):
                v = p.detach().double()
                arrays["param_sums"][t - 1, i] = float(v.sum())
                arrays["param_abs_sums"][t - 1, i] = float(v.abs().sum())
            if t in sample_steps:
                flat = torch.cat([p.detach().float().reshape(-1) for p in params])
                arrays[f"s{t}_param_sample"] = flat[::stride].numpy().copy()
                del flat
            meta["per_step"].append(rec)
            nfl = len(flips.flips) if flips is not None else 0
            print(f"  {name} step {t}/{steps} {time.time() - ts:.1f}s flips so far {nfl}",
                  flush=True)
    finally:
        if flips is not None:
            flips.restore()
    if flips is not None:
        f = np.array(flips.flips, dtype=np.int64).reshape(-1, 5)
        arrays["sr_flips"] = f
        meta["sr_flips"] = int(f.shape[0])
    meta["seconds"] = round(time.time() - t0, 1)
    with open(os.path.join(HERE, f"cfg_{name}.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    np.savez_compressed(os.path.join(HERE, f"cfg_{name}.npz"), **arrays)
    print(f"{name}: {steps} steps in {meta['seconds']} s", flush=True)


def checkpoint_fixture(ref, name: str, recipe: str, seed, k: int = 3, more: int = 3):
    """The reference's state_dict after k steps, then the digests of `more`
    further steps from that state (adamw.py:326-470)."""
    cls = {"ze-eden": ref.ZEEDENAdamW4Bit, "zip-sr": ref.ZIPSRAdamW4Bit}[recipe]
    shapes = [(64, 512), (768,), (96, 128)]
    params = [torch.nn.Parameter(S.init_param(s, i, torch.float32, "cpu"))
              for i, s in enumerate(shapes)]
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    if seed is not None:
        kw["quant_rng_seed"] = seed
    opt = cls(params, **kw)
    quantized = [eligible(p.numel()) for p in params]
    meta = {"name": name, "recipe": recipe, "shapes": [list(s) for s in shapes],
            "quant_rng_seed": seed, "k": k, "more": more, "grad_std": 1e-3, "per_step": []}
    arrays = {}
    for t in range(1, k + more + 1):
        for i, p in enumerate(params):
            p.grad = S.grad(p.shape, i, t, 1e-3, torch.float32, "cpu")
        opt.step()
        rec = {"step": t}
        rec.update(state_digests(opt, params, quantized))
        meta["per_step"].append(rec)
        if t in (k, k + more):
            for i, p in enumerate(params):
                arrays[f"s{t}_p{i}"] = p.detach().numpy().copy()
        if t == k:
            torch.save(opt.state_dict(), os.path.join(HERE, f"ckpt_{name}.pt"))
    with open(os.path.join(HERE, f"ckpt_{name}.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    np.savez_compressed(os.path.join(HERE, f"ckpt_{name}.npz"), **arrays)
    print(f"checkpoint fixture {name} written", flush=True)


def moment_digests(opt, params) -> dict:
    """Per moment: packed codes and scales when the moment is quantized,
    else its FP32 values (all tensors concatenated in parameter order)."""
    d = {k: Digest() for k in ("m1_code", "m1_absmax", "m2_code", "m2_absmax", "f_m1", "f_m2")}
    for p in params:
        st = opt.state[p]
        for m in ("m1", "m2"):
            if f"{m}_code" in st:
                d[f"{m}_code"].add(st[f"{m}_code"])
                d[f"{m}_absmax"].add(st[f"{m}_quant_state"].absmax)
            else:
                d[f"f_{m}"].add(st[m])
    return {k: v.hex() for k, v in d.items()}


def mixed_fixture(ref, name: str, m2_scheme: str, eden: bool, seed, steps: int = 6,
                  m1_scheme: str = "fp32"):
    """A scheme pair through QuantizedAdamW: FP32 first moments next to a
    4-bit second moment (the reference resolves each moment's scheme on its
    own, adamw.py:510-521), or a 4-bit m1 next to one of the fp32-read m2
    schemes whose storage bias is c_t or c_{t+1} (adamw.py:112-116, 655-683;
    quantization.py:581-582)."""
    shapes = [(64, 512), (768,), (32, 128)]
    params = [torch.nn.Parameter(S.init_param(s, i, torch.float32, "cpu"))
              for i, s in enumerate(shapes)]
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
              m1_quant_scheme=m1_scheme, m2_quant_scheme=m2_scheme, use_eden_m2=eden)
    if seed is not None:
        kw["quant_rng_seed"] = seed
    opt = ref.QuantizedAdamW(params, **kw)
    meta = {"name": name, "shapes": [list(s) for s in shapes], "m1_scheme": m1_scheme,
            "m2_scheme": m2_scheme, "eden": eden, "quant_rng_seed": seed, "steps": steps,
            "grad_std": 1e-3, "per_step": []}
    arrays = {}
    for t in range(1, steps + 1):
        for i, p in enumerate(params):
            p.grad = S.grad(p.shape, i, t, 1e-3, torch.float32, "cpu")
        opt.step()
        meta["per_step"].append({"step": t, **moment_digests(opt, params)})
    for i, p in enumerate(params):
        arrays[f"s{steps}_p{i}"] = p.detach().numpy().copy()
    with open(os.path.join(HERE, f"mixed_{name}.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    np.savez_compressed(os.path.join(HERE, f"mixed_{name}.npz"), **arrays)
    print(f"mixed fixture {name} written", flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--only", default="ckpt,c3,c5,c4")
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "src"))
    torch.set_num_threads(args.threads)
    import adamw4bit as ref
    import adamw4bit.quantization as quant

    f32, bf16 = torch.float32, torch.bfloat16
    for item in args.only.split(","):
        if item == "mixed":
            mixed_fixture(ref, "fp32m1_zipsr", "dyn4_upd_sr_fp32read", False, 11)
            mixed_fixture(ref, "fp32m1_zeeden", "dyn4_nz", True, None)
        elif item == "schemes":
            mixed_fixture(ref, "fp32m1_lookahead", "dyn4_lookahead_sr", False, 23)
            mixed_fixture(ref, "nf4_lookahead", "dyn4_lookahead_sr", False, 21, m1_scheme="nf4")
            mixed_fixture(ref, "nf4_nextbc", "dyn4_upd_sr_fp32read_nextbc", False, 22,
                          m1_scheme="nf4")
            mixed_fixture(ref, "nf4_lin4_fp32read", "lin4_upd_sr_fp32read", False, 24,
                          m1_scheme="nf4")
        elif item == "ckpt":
            checkpoint_fixture(ref, "zeeden", "ze-eden", None)
            checkpoint_fixture(ref, "zipsr", "zip-sr", 4321)
        elif item == "c3":
            shapes = S.gpt2_small_shapes()
            run_config(ref, quant, "c3_gpt2_zeeden", shapes=shapes, recipe="ze-eden",
                       p_dtype=f32, g_dtype=f32, steps=100, grad_std=1e-3, quant_rng_seed=1234,
                       switch_at=90, head=len(shapes) - 1,
                       sample_steps=(1, 10, 50, 89, 90, 91, 100))
        elif item == "c4":
            run_config(ref, quant, "c4_llama1b_zipsr", shapes=S.llama_1b_shapes(),
                       recipe="zip-sr", p_dtype=bf16, g_dtype=bf16, steps=50, grad_std=1e-4,
                       quant_rng_seed=1234, outlier_frac=0.01, sample_steps=(1, 10, 25, 50))
        elif item == "c5":
            run_config(ref, quant, "c5_llama8b_subset_zeeden", shapes=S.llama3_8b_subset_shapes(),
                       recipe="ze-eden", p_dtype=f32, g_dtype=bf16, steps=20, grad_std=1e-4,
                       quant_rng_seed=None, sample_steps=(1, 10, 20))
        else:
            raise SystemExit(f"unknown item {item}")


if __name__ == "__main__":
    main()
