"""Replay of the golden fixtures' inputs (tests/golden/, made by make_golden.py).

Gradients, initial parameters and the reference's SR uniforms are regenerated
from torch CPU generators with the recipe recorded in each fixture; the
fixture's per-step gradient digests guard against any drift of that recipe.
"""

from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

M1_OFFSET = 0x1A2B3C4D  # adamw.py:122-125
M2_OFFSET = 0x5E6F7789
RECIPE_SCHEMES = {"ze-eden": ("nf4", "dyn4_nz", True),
                  "zip-sr": ("nf4", "dyn4_upd_sr_fp32read", False)}
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def sha_np(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_traj(name: str):
    with open(os.path.join(GOLDEN, f"traj_{name}.json")) as f:
        meta = json.load(f)
    path = os.path.join(GOLDEN, f"traj_{name}.npz")
    arrays = dict(np.load(path)) if os.path.exists(path) else {}
    return meta, arrays


def exists(name: str) -> bool:
    return os.path.exists(os.path.join(GOLDEN, f"traj_{name}.json"))


def eligible(numel: int) -> bool:
    """adamw.py:807-811: quantized state iff numel >= 4096 and numel % 128 == 0."""
    return numel >= 4096 and numel % 128 == 0


@dataclass
class StepInputs:
    step: int
    grads: list            # torch CPU tensors, one per parameter
    m1_draws: list         # per parameter: float32 numpy [n] or None
    m2_draws: list
    m1_scheme: str         # scheme of the main parameter's m1 at this step


class Replay:
    """Regenerates the inputs a fixture was produced with, step by step."""

    def __init__(self, meta: dict):
        self.meta = meta
        self.shapes = [tuple(meta["shape"])] + [tuple(s) for s in meta["extra_small_shapes"]]
        self.p_dtype = DTYPES[meta["p_dtype"]]
        self.g_dtype = DTYPES[meta["g_dtype"]]
        m1, m2, eden = RECIPE_SCHEMES[meta["recipe"]]
        self.m1_scheme, self.m2_scheme, self.eden = m1, m2, eden
        seed = meta["quant_rng_seed"]
        self.m1_gen = self.m2_gen = None
        if seed is not None:
            self.m1_gen = torch.Generator().manual_seed((seed + M1_OFFSET) % ((1 << 63) - 1))
            self.m2_gen = torch.Generator().manual_seed((seed + M2_OFFSET) % ((1 << 63) - 1))
        self.ggen = torch.Generator().manual_seed(0)
        self.ogen = torch.Generator().manual_seed(2)
        self.t = 0

    def init_params(self) -> list:
        g = torch.Generator().manual_seed(1)
        return [(torch.randn(s, generator=g) * 0.02).to(self.p_dtype) for s in self.shapes]

    def _grad(self, shape) -> torch.Tensor:
        g = torch.randn(shape, generator=self.ggen) * self.meta["grad_std"]
        if self.meta["outlier_frac"] > 0:
            flat = g.view(-1, 128)
            mask = torch.rand(flat.shape[0], generator=self.ogen) < self.meta["outlier_frac"]
            flat[mask] *= 100.0
        return g.to(self.g_dtype)

    def _draws(self, gen, n: int) -> np.ndarray:
        assert gen is not None, "SR stream without quant_rng_seed"
        return torch.rand((n // 128, 128), generator=gen).numpy().reshape(-1).copy()

    def next(self) -> StepInputs:
        """Inputs of the next step, drawing reference uniforms in reference order
        (adamw.py:524-545 init draws, then 675-683 m2 and 764-771 m1)."""
        self.t += 1
        t = self.t
        switch = self.meta.get("switch_at")
        m1_now = "nf4_sr" if (switch is not None and t >= switch) else self.m1_scheme
        grads = [self._grad(s) for s in self.shapes]
        m1d, m2d = [], []
        for i, s in enumerate(self.shapes):
            n = int(np.prod(s))
            if not eligible(n):
                m1d.append(None)
                m2d.append(None)
                continue
            m1_sr = (m1_now == "nf4_sr") if i == 0 else False
            m2_sr = "sr" in self.m2_scheme
            if t == 1:
                # state init quantizes zeros with the moment generators
                if m1_sr:
                    self._draws(self.m1_gen, n)
                if m2_sr:
                    self._draws(self.m2_gen, n)
            m2d.append(self._draws(self.m2_gen, n) if m2_sr else None)
            m1d.append(self._draws(self.m1_gen, n) if m1_sr else None)
        return StepInputs(t, grads, m1d, m2d, m1_now)
