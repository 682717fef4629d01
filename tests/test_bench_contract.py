"""bench.py's contract, checked without a GPU: the benchmark's parameter set
is Llama-3-8B as the workload names it, and the CPU reference arm prints one
JSON line with the keys the measurement driver reads."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_llama3_8b_parameter_set():
    shapes = bench.llama3_8b_shapes()
    assert len(shapes) == 291
    assert sum(int(torch.Size(s).numel()) for s in shapes) == 8_030_261_248
    # every tensor qualifies for 4-bit state (numel >= 4096, multiple of 128)
    assert all(torch.Size(s).numel() >= 4096 and torch.Size(s).numel() % 128 == 0 for s in shapes)


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
         "--cpu-sample", str(1 << 20)],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["impl"] == "reference" and rec["metric"] == bench.METRIC
    assert rec["value"] > 0 and rec["higher_is_better"] is True
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["e2e"]["d2h_bytes_per_step"] == 0
    assert rec["cpu_baseline"]["kind"] in ("port", "reference")


def test_algorithmic_bytes_per_value():
    """The roofline's bytes per value: parameter read + write, gradient read,
    m1/m2 packed codes read + write (0.5 B each way each) and block scales
    (2 moments x 4 B read + write per 128 values), plus the BF16 model copy
    when FP32 master weights are kept."""
    assert bench.B_STATE == 2.125
    assert bench.bytes_per_value(4, 4, False) == 14.125      # configs 1-3
    assert bench.bytes_per_value(2, 2, False) == 8.125       # config 4
    assert bench.bytes_per_value(4, 2, False) == 12.125      # config 5, drop-in API
    assert bench.bytes_per_value(4, 2, True) == bench.B_PER_ELEM == 14.125   # bench value
    assert len(bench.llama_1b_shapes()) == 147
    assert sum(int(torch.Size(s).numel()) for s in bench.llama_1b_shapes()) == 852_559_872


def test_multi_gpu_nvlink_accounting():
    """NVLink bytes per GPU and step for config 5 (8.03 G values): NCCL's
    gather brings (W-1)/W of the BF16 model, the multicast stores the whole
    model (the switch delivers a rank's own shard back to it), and the fused
    ZeRO-2 step moves 2 (1 + 1/W) B per value each way; --gather auto picks
    multicast from 4 ranks up."""
    n = 8_030_261_248
    assert bench.gather_ingress_bytes(8, n, True, False) == 7 / 8 * n * 2
    assert bench.gather_ingress_bytes(8, n, True, True) == n * 2
    assert bench.gather_ingress_bytes(2, n, False, False) == n * 2      # FP32, half the model
    assert round(bench.zero2_nvlink_bytes(2, n) / 1e9, 2) == 24.09
    assert [bench.resolve_gather("auto", w) for w in (2, 4, 8)] == ["bf16", "multicast", "multicast"]
    assert bench.resolve_gather("bf16", 8) == "bf16"
