"""Generate the golden fixtures in tests/golden/ by running the REFERENCE.

Run where a checkout of the reference (nubank/adamw4bit) exists, passing its
root as ``--reference``; the fixtures are committed so the tests never need
the reference at run time:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

Every optimizer trajectory uses the reference's eager path (optimized=False):
its optimized=True path draws a different number of SR uniforms at state
initialisation, so the eager path is the one parity is defined against.
Inputs are seeded synthetic tensors shaped like the benchmark configurations;
gradients are regenerated in the tests from the same torch CPU generator
recipe (recorded in each fixture, with a checksum of every step's gradient to
detect drift).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
SAMPLE_STRIDE = 4099  # parameter sample: every 4099th element


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def as_f32_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().reshape(-1)


def make_grad(ggen: torch.Generator, shape, std: float, dtype, outlier_frac: float = 0.0,
              outlier_gen: torch.Generator | None = None) -> torch.Tensor:
    """Gradient recipe shared with tests/golden_io.py: N(0, std) float32 from ggen,
    optional outlier blocks (a fraction of 128-blocks scaled by 100, chosen with
    outlier_gen), then cast to the gradient dtype."""
    g = torch.randn(shape, generator=ggen) * std
    if outlier_frac > 0:
        flat = g.view(-1, 128)
        mask = torch.rand(flat.shape[0], generator=outlier_gen) < outlier_frac
        flat[mask] *= 100.0
    return g.to(dtype)


def trajectory(ref, name: str, *, recipe: str, shape, p_dtype, g_dtype, steps: int,
               grad_std: float, quant_rng_seed, outlier_frac: float = 0.0, switch_at=None,
               extra_small_shapes=(), full_state_steps=(), lr=1e-3, wd=0.1,
               betas=(0.9, 0.95), eps=1e-8, weight_decay=None):
    """Run the reference optimizer and record per-step digests."""
    cls = {"ze-eden": ref.ZEEDENAdamW4Bit, "zip-sr": ref.ZIPSRAdamW4Bit}[recipe]
    init_gen = torch.Generator().manual_seed(1)
    params = [torch.nn.Parameter((torch.randn(shape, generator=init_gen) * 0.02).to(p_dtype))]
    for s in extra_small_shapes:
        params.append(torch.nn.Parameter((torch.randn(s, generator=init_gen) * 0.02).to(p_dtype)))
    kw = dict(lr=lr, betas=betas, eps=eps, weight_decay=wd if weight_decay is None else weight_decay)
    if quant_rng_seed is not None:
        kw["quant_rng_seed"] = quant_rng_seed
    if g_dtype != p_dtype:
        for p in params:
            p.grad_dtype = None  # torch >= 2.10 requires opting in to mixed grad dtypes
    opt = cls(params, **kw)
    ggen = torch.Generator().manual_seed(0)
    ogen = torch.Generator().manual_seed(2)
    record = {
        "name": name, "recipe": recipe, "shape": list(shape),
        "extra_small_shapes": [list(s) for s in extra_small_shapes],
        "p_dtype": str(p_dtype).replace("torch.", ""), "g_dtype": str(g_dtype).replace("torch.", ""),
        "steps": steps, "grad_std": grad_std, "outlier_frac": outlier_frac,
        "quant_rng_seed": quant_rng_seed, "switch_at": switch_at,
        "lr": lr, "betas": list(betas), "eps": eps, "weight_decay": kw["weight_decay"],
        "init": "params: torch.Generator().manual_seed(1), randn*0.02 per tensor in order; "
                "grads: torch.Generator().manual_seed(0), randn*grad_std per step per tensor; "
                "outlier blocks: torch.Generator().manual_seed(2)",
        "sample_stride": SAMPLE_STRIDE,
        "per_step": [],
    }
    arrays = {}
    for t in range(1, steps + 1):
        if switch_at is not None and t == switch_at:
            opt.set_m1_quant_scheme_for_parameters([params[0]], "nf4_sr")
        grad_shas = []
        for p in params:
            p.grad = make_grad(ggen, p.shape, grad_std, g_dtype, outlier_frac, ogen)
            grad_shas.append(sha(p.grad))
        opt.step()
        st = opt.state[params[0]]
        rec = {
            "step": t, "grad_sha": grad_shas,
            "m1_code": sha(st["m1_code"]), "m1_absmax": sha(st["m1_quant_state"].absmax),
            "m2_code": sha(st["m2_code"]), "m2_absmax": sha(st["m2_quant_state"].absmax),
            "param": sha(params[0]),
        }
        rec_small = []
        for i, p in enumerate(params[1:], start=1):
            s = opt.state[p]
            rec_small.append({k: sha(s[k]) for k in ("m1", "m2")} | {"param": sha(p)})
            if t in full_state_steps:
                arrays[f"s{t}_small{i}_param"] = as_f32_numpy(p)
                arrays[f"s{t}_small{i}_m1"] = as_f32_numpy(s["m1"])
                arrays[f"s{t}_small{i}_m2"] = as_f32_numpy(s["m2"])
        rec["small"] = rec_small
        arrays[f"s{t}_param_sample"] = as_f32_numpy(params[0])[::SAMPLE_STRIDE].copy()
        if t in full_state_steps:
            arrays[f"s{t}_param"] = as_f32_numpy(params[0])
            arrays[f"s{t}_m1_code"] = st["m1_code"].numpy().copy()
            arrays[f"s{t}_m2_code"] = st["m2_code"].numpy().copy()
            arrays[f"s{t}_m1_absmax"] = st["m1_quant_state"].absmax.numpy().copy()
            arrays[f"s{t}_m2_absmax"] = st["m2_quant_state"].absmax.numpy().copy()
        record["per_step"].append(rec)
        print(f"  {name} step {t} done", flush=True)
    with open(os.path.join(HERE, f"traj_{name}.json"), "w") as f:
        json.dump(record, f, indent=1)
    np.savez_compressed(os.path.join(HERE, f"traj_{name}.npz"), **arrays)


def codebooks(quant) -> None:
    out = {}
    for scheme in ("nf4", "nf4_sr", "sdyn4", "sdyn4_sr", "dyn4", "dyn4_nz", "dyn4_sr",
                   "dyn4_upd_sr_fp32read", "dyn4_lookahead_sr", "dyn4_upd_sr_fp32read_nextbc",
                   "lin4", "lin4_nz", "lin4_sr", "lin4_upd_sr_fp32read"):
        cb = quant._STRATEGIES[scheme]._get_codebook(torch.device("cpu")).numpy()
        out[scheme] = [int(w) for w in cb.view(np.uint32)]
    with open(os.path.join(HERE, "codebooks.json"), "w") as f:
        json.dump(out, f, indent=1)


def codec_inputs(n_blocks: int, signed: bool, seed: int) -> torch.Tensor:
    """Blocks with mixed magnitudes, exact codebook levels, midpoints, zeros."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n_blocks, 128, generator=g)
    x *= torch.exp(torch.randn(n_blocks, 1, generator=g) * 4.0)
    if not signed:
        x = x.square()
    x[0] = 0.0                                   # all-zero block -> 1e-12 scale floor
    x[1, :5] = torch.tensor([1e-30, 1e-20, 1e-13, 0.0, 0.0])
    x[2] = torch.linspace(-1.0 if signed else 0.0, 1.0, 128)
    return x.reshape(-1).contiguous()


def codec_cases(quant) -> None:
    arrays = {}
    meta = []
    cases = [
        ("nf4", False, True), ("sdyn4", False, True), ("dyn4", False, False),
        ("dyn4_nz", False, False), ("dyn4_nz", True, False), ("dyn4", True, False),
        ("lin4", False, False), ("lin4_nz", False, False), ("lin4_nz", True, False),
        ("nf4_sr", False, True), ("sdyn4_sr", False, True), ("dyn4_sr", False, False),
        ("lin4_sr", False, False), ("dyn4_upd_sr_fp32read", False, False),
        ("dyn4_upd_sr_fp32read", True, False), ("lin4_upd_sr_fp32read", False, False),
    ]
    for k, (scheme, eden, signed) in enumerate(cases):
        x = codec_inputs(32, signed, seed=100 + k)
        if signed and scheme in ("nf4", "sdyn4"):
            # exact levels and exact float32 midpoints of each codebook
            cb = quant._STRATEGIES[scheme]._get_codebook(torch.device("cpu"))
            mids = (cb[:-1] + cb[1:]) / 2
            x[3 * 128:3 * 128 + 16] = cb
            x[3 * 128 + 16:3 * 128 + 31] = mids
        gen = torch.Generator().manual_seed(500 + k)
        draws = torch.rand((x.numel() // 128, 128), generator=torch.Generator().manual_seed(500 + k))
        kwargs = dict(block_size=128, mode=scheme, eden_correction=eden)
        if "upd_sr" in scheme:
            kwargs.update(bias_correction=0.0975, eps=1e-8)
        codes, qs = quant.quantize(x, generator=gen, **kwargs)
        tag = f"c{k}"
        arrays[f"{tag}_x"] = x.numpy()
        arrays[f"{tag}_draws"] = draws.numpy().reshape(-1)
        arrays[f"{tag}_codes"] = codes.numpy().astype(np.uint8)
        arrays[f"{tag}_scales"] = qs.absmax.numpy()
        meta.append({"tag": tag, "scheme": scheme, "eden": eden,
                     "bias_correction": kwargs.get("bias_correction"), "eps": kwargs.get("eps")})
    # nibble packing KAT (tests/quantization/test_utils.py:92-101)
    arrays["pack_in"] = np.array([1, 2, 15], np.uint8)
    arrays["pack_out"] = quant.pack_4bit_codes(torch.tensor([1, 2, 15], dtype=torch.uint8)).numpy()
    np.savez_compressed(os.path.join(HERE, "codec_cases.npz"), **arrays)
    with open(os.path.join(HERE, "codec_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--skip-full", action="store_true", help="skip the 16.8M-element runs")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "src"))
    torch.set_num_threads(os.cpu_count() or 1)
    import adamw4bit as ref
    import adamw4bit.quantization as quant

    codebooks(quant)
    codec_cases(quant)
    f32, bf16, f16 = torch.float32, torch.bfloat16, torch.float16
    # config 1 / 2 shapes, reduced (full state kept for steps 1 and 10)
    trajectory(ref, "zeeden_f32_small", recipe="ze-eden", shape=(64, 512), p_dtype=f32,
               g_dtype=f32, steps=10, grad_std=1e-3, quant_rng_seed=None,
               full_state_steps=(10,))
    trajectory(ref, "zipsr_f32_small", recipe="zip-sr", shape=(64, 512), p_dtype=f32,
               g_dtype=f32, steps=10, grad_std=1e-3, quant_rng_seed=1234,
               full_state_steps=(10,))
    # config 3 flavour: head m1 switched to nf4_sr mid-run, plus FP32-state tensors
    trajectory(ref, "zeeden_switch_small", recipe="ze-eden", shape=(32, 768), p_dtype=f32,
               g_dtype=f32, steps=6, grad_std=1e-3, quant_rng_seed=7, switch_at=4,
               extra_small_shapes=((768,), (2304,), (4097,)), full_state_steps=(6,))
    # config 4 flavour: BF16 params/grads, ZIP-SR, 1% outlier blocks x100
    trajectory(ref, "zipsr_bf16_outliers", recipe="zip-sr", shape=(128, 512), p_dtype=bf16,
               g_dtype=bf16, steps=10, grad_std=1e-4, quant_rng_seed=99, outlier_frac=0.01,
               extra_small_shapes=((2048,),), full_state_steps=(10,))
    # config 5 flavour: FP32 master params, BF16 grads, ZE-EDEN
    trajectory(ref, "zeeden_f32p_bf16g", recipe="ze-eden", shape=(128, 512), p_dtype=f32,
               g_dtype=bf16, steps=5, grad_std=1e-4, quant_rng_seed=None, full_state_steps=(5,))
    trajectory(ref, "zeeden_f16", recipe="ze-eden", shape=(32, 512), p_dtype=f16, g_dtype=f16,
               steps=4, grad_std=1e-3, quant_rng_seed=None, full_state_steps=(4,))
    if not args.skip_full:
        # configs 1 and 2 at full size: digests of every step (no full state)
        trajectory(ref, "zeeden_f32_c1", recipe="ze-eden", shape=(4096, 4096), p_dtype=f32,
                   g_dtype=f32, steps=10, grad_std=1e-3, quant_rng_seed=None)
        trajectory(ref, "zipsr_f32_c2", recipe="zip-sr", shape=(4096, 4096), p_dtype=f32,
                   g_dtype=f32, steps=10, grad_std=1e-3, quant_rng_seed=1234)


if __name__ == "__main__":
    main()
