"""Benchmark of the fused 4-bit AdamW step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1)

Workload (``value``, every N): the Llama-3-8B parameter set (vocab 128256,
d 4096, 32 layers, ffn 14336, 32/8 heads, untied head: 291 tensors, 8.03 B
values, all quantized), FP32 master weights, BF16 gradients N(0, 1e-4),
ZE-EDEN (NF4 m1 + zero-exclusive Dyn4 m2 with EDEN), stepped by
ZeRO1AdamW4Bit: the update kernel updates the FP32 masters and writes the BF16
model copy the next forward pass reads.  At N=1 one GPU owns every value; at
N>1 the masters and moments are sharded ZeRO-1 style and the BF16 model is
all-gathered (NCCL, or the kernel's own NVSwitch multicast stores with
``--gather multicast``), so every N does the same work per step.
Synthetic data, random-init weights.

A step is one pass of the optimizer over every parameter.  ``value`` is the
whole-job elements/s with everything resident in HBM (the working set is far
larger than the 126 MB L2, so no flush is needed between steps); ``e2e`` is
the same metric with each rank's gradients copied in from pinned host memory
and its updated BF16 model shard copied back every step.

N=1 also reports, as extra keys:
  * ``drop_in``: the reference's own API, ZEEDENAdamW4Bit with FP32
    parameters and BF16 gradients (no model copy), on the same parameter set;
  * ``zip_sr``: ZIPSRAdamW4Bit on BASELINE configuration 4's Llama-1B set,
    BF16 parameters and gradients, and FP32 parameters with BF16 gradients;
  * ``cpu_baseline``: the C/OpenMP port of the reference algorithm on a
    2^27-value sample, and the reference's own CPU step (from the offline
    install under baseline/_ref), eager (optimized=False) and chunked
    (optimized=True), on one 4096x4096 FP32 tensor, all host threads.

``--impl reference`` times the CPU port of the reference algorithm on the
host's cores on a bounded sample of the same workload (the reference itself
is Python on PyTorch).  ``--impl reference-gpu`` / ``reference-gpu-eager`` /
``reference-cpu`` / ``reference-cpu-eager`` time the reference's own
implementation on the GPU or on the host cores, for comparison only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "optimizer-step elements/s"
UNIT = "elements/s"
B_STATE = 2 * (0.5 + 0.5) + 2 * 2 * 4 / 128   # m1/m2 packed codes and block scales, read + write
WORKLOAD = ("llama3-8b ZE-EDEN: FP32 master weights + BF16 model copy, BF16 grads "
            "(BASELINE config 5)")


def bytes_per_value(p_bytes: int, g_bytes: int, model_copy: bool) -> float:
    """Algorithmic HBM bytes of one value's step: parameter read + write,
    gradient read, moment state, and the BF16 model-copy write."""
    return 2 * p_bytes + g_bytes + B_STATE + (2 if model_copy else 0)


B_PER_ELEM = bytes_per_value(4, 2, True)   # the config-5 workload: 14.125 B/value


def llama3_8b_shapes() -> list[tuple[int, ...]]:
    V, d, L, ffn, kv = 128256, 4096, 32, 14336, 1024
    shapes = [(V, d)]
    for _ in range(L):
        shapes += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    shapes += [(d,), (V, d)]
    return shapes


def llama_1b_shapes() -> list[tuple[int, ...]]:
    """vocab 32000, d 2048, 16 layers, ffn 5632,
    32/8 heads (kv dim 512), untied head: 147 tensors, 852.6 M values."""
    V, d, L, ffn, kv = 32000, 2048, 16, 5632, 512
    shapes = [(V, d)]
    for _ in range(L):
        shapes += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    shapes += [(d,), (V, d)]
    return shapes


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def traffic_record() -> dict | None:
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def resolve_gather(gather: str, world: int) -> str:
    """--gather auto: NVSwitch multicast stores from 4 ranks up (measured
    faster than NCCL's gather there), NCCL's BF16 gather below."""
    if gather != "auto":
        return gather
    return "multicast" if world >= 4 else "bf16"


def gather_ingress_bytes(world: int, total: int, master: bool, multicast: bool) -> float:
    """Model bytes each GPU receives per step.  NCCL's all-gather brings the
    other ranks' shards, (W-1)/W of the model.  A multimem store goes through
    the switch to every replica, this rank's own included, so the multicast
    gather brings the whole model in."""
    share = 1.0 if multicast else (world - 1) / world
    return share * total * (2 if master else 4)


def zero2_nvlink_bytes(world: int, total: int) -> float:
    """Bytes per NVLink direction per GPU and step of the fused ZeRO-2 step
    (BF16 gradients and model): 2 (1 + 1/W) per value.  Out: the switch
    reads every rank's copy of a shard for its owner's ld_reduce, this rank's
    own copy included, so all of its local gradients (2 B), plus its shard's
    multicast model stores (2/W).  In: its shard's reduced sums (2/W) and
    every shard of the model, its own included (2).  Measured with ld_reduce
    alone (BF16, 2 and 4 GPUs): each GPU's egress is its whole buffer, at
    670-708 GB/s."""
    return 2.0 * total * (1.0 + 1.0 / world)


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def make_workload(dev, shapes, seed=0, param_dtype=torch.float32):
    g = torch.Generator(device=dev).manual_seed(seed)
    params, grads = [], []
    for s in shapes:
        p = torch.nn.Parameter((torch.randn(s, device=dev, generator=g) * 0.02).to(param_dtype))
        gr = (torch.randn(s, device=dev, generator=g) * 1e-4).to(torch.bfloat16)
        p.grad_dtype = None  # FP32 parameter, BF16 gradient
        params.append(p)
        grads.append(gr)
    return params, grads


def cpu_oracle_rate(sample_elems: int, steps: int, threads: int | None = None) -> dict:
    """Time the oracle port of the reference algorithm on the host cores."""
    import numpy as np

    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    n = sample_elems
    rng = np.random.default_rng(0)
    p = (rng.standard_normal(n, dtype=np.float32) * 0.02).astype(np.float32)
    g32 = (rng.standard_normal(n, dtype=np.float32) * 1e-4).astype(np.float32)
    g = (g32.view(np.uint32) >> 16).astype(np.uint16)   # bf16 (truncated; values only)
    c1, s1 = O.init_zero("nf4", n)
    c2, s2 = O.init_zero("dyn4_nz", n, eden=True)
    times = []
    for t in range(1, steps + 2):
        cfg = O.make_cfg(m1_scheme="nf4", m2_scheme="dyn4_nz", eden=True, lr=1e-3,
                         betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, step=t,
                         grad_dtype=O.BF16)
        t0 = time.perf_counter()
        O.step(cfg, p, g, c1, s1, c2, s2)
        dt = time.perf_counter() - t0
        if t > 1:
            times.append(dt)
    med = statistics.median(times)
    return {"value": n / med, "unit": UNIT, "cores": O.max_threads(), "kind": "port",
            "sample": f"{n} values (FP32 params, BF16 grads, ZE-EDEN), median of {steps} steps "
                      f"after 1 warm-up step, C oracle (OpenMP)",
            "seconds_per_step": med}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    sample = args.cpu_sample
    base = cpu_oracle_rate(sample, max(1, args.steps), threads)
    line = {"metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": base["seconds_per_step"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample_values": sample, "l2": "inputs > L2"},
            "impl": "reference",
            "cpu_baseline": {**{k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
                             **{k: ({kk: vv for kk, vv in v.items() if kk != "seconds_per_step"}
                                    if isinstance(v, dict) else v)
                                for k, v in reference_cpu_rates(max(1, min(args.steps, 3))).items()}},
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_torch(args, rank, device: str, eager: bool):
    """The reference's own implementation (its ZEEDENAdamW4Bit), for
    comparison only: on CUDA (the "GPU bar") with optimized=True
    (torch.compile per 512 Ki chunk) or its eager path; on the host CPU with
    all threads, eager or chunked (optimized=True).  Imported from the offline
    install under baseline/_ref; not part of the product.  The CPU runs
    default to config 1's tensor (4096 x 4096)."""
    if rank != 0:
        return
    ref = os.path.join(ROOT, "baseline", "_ref")
    impl = f"reference-{'gpu' if device == 'cuda' else 'cpu'}{'-eager' if eager else ''}"
    if not os.path.isdir(os.path.join(ref, "adamw4bit")):
        print(json.dumps({"impl": impl, "unavailable": "baseline/_ref is not installed"}))
        return
    sys.path.insert(0, ref)
    from adamw4bit import ZEEDENAdamW4Bit as RefZE

    if device == "cuda":
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        shapes = llama3_8b_shapes()
        if args.layers is not None:
            shapes = shapes[:1 + 9 * args.layers] + shapes[-2:]
    else:
        dev = torch.device("cpu")
        torch.set_num_threads(os.cpu_count() or 1)
        shapes = [(4096, 4096)]
    if args.values:
        shapes = [(args.values,)]
    total = sum(int(torch.Size(s).numel()) for s in shapes)
    params, grads = make_workload(dev, shapes)
    compat = None
    if args.compile_compat and not eager:
        # the reference passes torch.compile(isolate_recompiles=True)
        # (_optimized.py:244-246), a keyword this torch lacks; dropping it
        # keeps every other argument and the reference's code unchanged
        orig_compile = torch.compile

        def compile_without_isolation(*a, **kw):
            kw.pop("isolate_recompiles", None)
            return orig_compile(*a, **kw)
        torch.compile = compile_without_isolation
        compat = "torch.compile called without isolate_recompiles (absent from torch " \
                 f"{torch.__version__})"
    opt = RefZE(params, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                optimized=not eager)
    for p_, g_ in zip(params, grads):
        p_.grad = g_
    t0 = time.perf_counter()
    try:
        for _ in range(args.warmup):
            opt.step()
    except TypeError as exc:   # the reference needs torch >= 2.13 for its compiled path
        print(json.dumps({"impl": impl, "unavailable": f"reference step failed on torch "
                                                        f"{torch.__version__}: {exc}"}))
        return
    if device == "cuda":
        torch.cuda.synchronize()
        warm_s = time.perf_counter() - t0
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            opt.step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        extra = {}
    else:
        warm_s = time.perf_counter() - t0
        times = []
        for _ in range(args.steps):
            t1 = time.perf_counter()
            opt.step()
            times.append(time.perf_counter() - t1)
        ms = statistics.median(times) * 1e3
        extra = {"cores": torch.get_num_threads(), "timing": "median wall time per step"}
    print(json.dumps({"metric": METRIC, "value": total / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "impl": impl, "dtype": "f32",
                      "data": "synthetic",
                      "config": {"workload": "llama3-8b, FP32 params updated in place, BF16 "
                                             "grads, ZE-EDEN (BASELINE config 5 through the "
                                             "reference's API)" if device == "cuda" else
                                 "4096x4096 FP32 param, BF16 grads, ZE-EDEN",
                                 "values": total, "tensors": len(shapes)},
                      "warmup_seconds": warm_s, **({"compat": compat} if compat else {}),
                      **extra}), flush=True)


def reference_cpu_rates(steps: int) -> dict:
    """The reference's own ZEEDENAdamW4Bit.step on the host cores (all
    threads), eager (optimized=False, adamw.py:472-805) and chunked
    (optimized=True, _optimized.py:145-247), on one 4096x4096 FP32 tensor
    with BF16 gradients: median wall time of `steps` steps after one warm-up
    step.  Imported from the offline install under baseline/_ref."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "adamw4bit")):
        return {"unavailable": "baseline/_ref is not installed"}
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from adamw4bit import ZEEDENAdamW4Bit as RefZE

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    init = torch.randn(4096, 4096, generator=gen) * 0.02
    grad = (torch.randn(4096, 4096, generator=gen) * 1e-4).to(torch.bfloat16)
    out = {}
    for key, optimized in (("reference_eager", False), ("reference_optimized", True)):
        p = torch.nn.Parameter(init.clone())
        p.grad_dtype = None   # FP32 parameter, BF16 gradient
        opt = RefZE([p], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                    optimized=optimized)
        p.grad = grad
        opt.step()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            opt.step()
            times.append(time.perf_counter() - t0)
        med = statistics.median(times)
        out[key] = {"value": p.numel() / med, "unit": UNIT, "cores": threads,
                    "kind": "reference",
                    "sample": f"4096x4096 FP32 param, BF16 grads, ZEEDENAdamW4Bit "
                              f"optimized={optimized}, median of {steps} steps after 1 "
                              "warm-up step (baseline/_ref, CPU)",
                    "seconds_per_step": med}
    return out


def rank_identities(world: int, dev) -> list | None:
    """Each rank's GPU (name, PCI bus id) and the NCCL version, gathered over
    the process group: the line shows which devices took part."""
    if world == 1:
        return None
    import torch.distributed as dist
    props = torch.cuda.get_device_properties(dev)
    me = {"rank": dist.get_rank(), "device": props.name,
          "pci_bus_id": f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}",
          "nccl": ".".join(str(v) for v in torch.cuda.nccl.version()),
          "nccl_nvls_enable": os.environ.get("NCCL_NVLS_ENABLE", "default")}
    out = [None] * world
    dist.all_gather_object(out, me)
    return out


def timed_steps(opt, steps: int, warmup: int) -> tuple[float, float, float]:
    """Runs warm-up then `steps` optimizer steps; returns (device ms per step,
    fused-kernel ms per step, values updated per step)."""
    for _ in range(warmup):
        opt.step()
    torch.cuda.synchronize()
    opt.launch_timings = []
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        opt.step()
    e1.record()
    torch.cuda.synchronize()
    t = opt.launch_timings
    opt.launch_timings = None
    kms = sum(a.elapsed_time(b) for a, b, *_ in t) / steps
    vals = sum(x[2] for x in t) / steps
    return e0.elapsed_time(e1) / steps, kms, vals


def leg_record(kernel_ms: float, values: float, bpv: float, peak: float, step_ms: float) -> dict:
    gbs = values * bpv / (kernel_ms / 1e3) / 1e9
    return {"values": int(values), "step_ms": round(step_ms, 4), "launch_ms": round(kernel_ms, 4),
            "elements_per_s": values / (kernel_ms / 1e3), "bytes_per_value": bpv,
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}


def run_legs(args, dev, peak: float) -> dict:
    """N=1 extra keys: the drop-in API on config 5 and the ZIP-SR legs."""
    from adamw4bit_b200 import ZEEDENAdamW4Bit, ZIPSRAdamW4Bit

    out = {}
    params, grads = make_workload(dev, llama3_8b_shapes(), param_dtype=torch.float32)
    for p, g in zip(params, grads):
        p.grad = g
    opt = ZEEDENAdamW4Bit(params, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    step_ms, kms, vals = timed_steps(opt, args.steps, args.warmup)
    out["drop_in"] = {"api": "ZEEDENAdamW4Bit", "workload": "llama3-8b, FP32 params updated in "
                      "place, BF16 grads (BASELINE config 5 through the reference's API)",
                      **leg_record(kms, vals, bytes_per_value(4, 2, False), peak, step_ms)}
    del opt, params, grads
    torch.cuda.empty_cache()
    zs = {"api": "ZIPSRAdamW4Bit", "workload": "llama-1b (BASELINE config 4 parameter set), "
          "quant_rng_seed=1234, in-kernel Philox draws"}
    for key, pdt in (("bf16_params_bf16_grads", torch.bfloat16),
                     ("fp32_params_bf16_grads", torch.float32)):
        params, grads = make_workload(dev, llama_1b_shapes(), param_dtype=pdt)
        for p, g in zip(params, grads):
            p.grad = g
        opt = ZIPSRAdamW4Bit(params, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                             quant_rng_seed=1234)
        step_ms, kms, vals = timed_steps(opt, args.steps, args.warmup)
        zs[key] = leg_record(kms, vals, bytes_per_value(pdt.itemsize, 2, False), peak, step_ms)
        del opt, params, grads
        torch.cuda.empty_cache()
    out["zip_sr"] = zs
    return out


def run_ours(args, rank, world, local):
    from adamw4bit_b200 import _native
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shapes = llama3_8b_shapes()
    if args.layers is not None:
        shapes = shapes[:1 + 9 * args.layers] + shapes[-2:]
    if args.values:
        shapes = [(args.values,)]   # single-tensor case (profiling)
    total = sum(int(torch.Size(s).numel()) for s in shapes)
    args.gather = resolve_gather(args.gather, world)
    master = args.gather != "fp32"
    params, grads = make_workload(dev, shapes,
                                  param_dtype=torch.bfloat16 if master else torch.float32)
    # FP32 masters (sharded over the ranks at N>1) and the BF16 model copy
    # written by the update kernel; at N>1 the model is all-gathered
    opt = ZeRO1AdamW4Bit(params, recipe=args.recipe, rounds=args.rounds,
                         master_weights=master, reserve_sms=args.reserve_sms,
                         gather="multicast" if args.gather == "multicast" else "nccl",
                         grad_reduce=args.grad_reduce, quant_rng_seed=1234)
    step_fn = opt.step
    updated_per_rank = opt.owned_numel()
    b_per_elem = bytes_per_value(4, 2, master)
    zero2 = world > 1 and args.grad_reduce == "multicast"
    for p, g in zip(params, grads):
        if zero2:   # this rank's unreduced gradients, in the bound symmetric buffer
            p.grad.copy_(g)
        else:
            p.grad = g
    for _ in range(args.warmup):
        step_fn()
    barrier(world)

    sampler = ClockSampler(torch.cuda.current_device() if world == 1 else local)
    sampler.start()
    opt.launch_timings = []
    launches0 = _native.launch_count()
    barrier(world)
    cur = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        step_fn()
    e1.record(cur)
    barrier(world)
    launches = _native.launch_count() - launches0
    clocks = sampler.stop()
    elapsed_ms = e0.elapsed_time(e1)
    timings = opt.launch_timings
    opt.launch_timings = None
    kernel_ms = sum(a.elapsed_time(b) for a, b, *_ in timings)
    kernel_elems = sum(n for _, _, n, *_ in timings)
    elapsed_ms = max_over_ranks(elapsed_ms, world)
    kernel_ms_max = max_over_ranks(kernel_ms, world)
    ms_per_step = elapsed_ms / args.steps
    value = total * args.steps / (elapsed_ms / 1e3)

    peaks = measured_peaks()
    hbm_peak = peaks.get("hbm_gbs")
    peak_src = "measured"
    if hbm_peak is None:
        hbm_peak, peak_src = 6650.0, "fallback"
    per_launch_ms = kernel_ms / max(1, len(timings))
    per_launch_elems = kernel_elems / max(1, len(timings))
    achieved = per_launch_elems * b_per_elem / (per_launch_ms / 1e3) / 1e9
    tr = traffic_record()
    traffic = None
    if tr and tr.get("bytes_per_value") and tr.get("bytes_per_value_algorithmic") == b_per_elem:
        traffic = tr["bytes_per_value"] * per_launch_elems
    kname = "aw4::step_kernel<F32,BF16,RTN,%s> (fused decode+AdamW+encode+BF16 model copy)" % (
        "RTN" if args.recipe == "ze-eden" else "SR_UPDATE")
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                "peak_source": peak_src, "algorithmic_bytes_per_value": b_per_elem,
                "kernel": kname, "launch_ms": round(per_launch_ms, 4),
                "values_per_launch": int(per_launch_elems)}

    e2e = run_e2e(args, opt, dev, world, total) if args.e2e_steps > 0 else None
    ranks = rank_identities(world, dev)
    gather_mode = opt.gather_mode
    del opt, params, grads
    torch.cuda.empty_cache()
    legs = run_legs(args, dev, hbm_peak) if (world == 1 and args.legs) else {}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD if args.recipe == "ze-eden" else
                           WORKLOAD.replace("ZE-EDEN", "ZIP-SR").replace(" (BASELINE config 5)", ""),
                           "values": total, "tensors": len(shapes),
                           "param_dtype": "fp32 master + bf16 model copy" if master else "fp32",
                           "grad_dtype": "bf16", "recipe": args.recipe.upper(),
                           "parallelism": "single GPU" if world == 1 else
                           f"{'zero2' if zero2 else 'zero1'}-dp{world}, "
                           f"{'bf16 model' if master else 'fp32'} gather "
                           f"({gather_mode})"
                           + (", gradient reduce-scatter fused into the update "
                              "(multimem.ld_reduce)" if zero2 else
                              ", gradients already reduced"),
                           "l2": "no flush: 72 GB working set >> 126 MB L2"},
                "roofline": roofline,
                "update_only": {"values_per_rank": updated_per_rank,
                                "kernel_ms_per_step_max_rank": kernel_ms_max / args.steps,
                                "elements_per_s_per_rank":
                                    updated_per_rank * args.steps / (kernel_ms_max / 1e3)},
                "clocks": clocks, "gpu_launches": int(launches),
                "e2e": e2e}
        if world > 1:
            line["ranks"] = ranks
            nv = gather_ingress_bytes(world, total, master, gather_mode == "multicast")
            line["gather"] = {"ingress_bytes_per_gpu": nv,
                              "ingress_gbs": round(nv / (ms_per_step / 1e3) / 1e9, 1),
                              "peak_gbs": 770.0,
                              "peak_source": "measured peer copy, per direction",
                              "floor_ms": round(nv / 770e9 * 1e3, 2)}
        if zero2:
            nv = zero2_nvlink_bytes(world, total)
            line["nvlink"] = {"bytes_per_direction_per_gpu": nv,
                              "achieved_gbs": round(nv / (ms_per_step / 1e3) / 1e9, 1),
                              "peak_gbs": 770.0, "peak_source": "measured peer copy, per direction",
                              "frac": round(nv / (ms_per_step / 1e3) / 1e9 / 770.0, 4)}
        line.update(legs)
        if world == 1 and args.cpu_sample > 0:
            cb = {k: v for k, v in cpu_oracle_rate(
                args.cpu_sample, args.cpu_steps).items() if k != "seconds_per_step"}
            for k, v in reference_cpu_rates(args.cpu_steps).items():
                cb[k] = {kk: vv for kk, vv in v.items() if kk != "seconds_per_step"} \
                    if isinstance(v, dict) else v
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)


def run_e2e(args, opt, dev, world, total):
    """End to end through the optimizer with host buffers: each rank copies in
    its gradients from pinned host memory (its owned segments; with the
    ZeRO-2 reduction, its full local gradients), steps, and copies its updated
    BF16 model shard back to pinned host memory, all inside the timed region.

    The copies are pipelined per round of the step (ZeRO1AdamW4Bit.step's
    round hooks): gradients upload on a copy stream, round after round, each
    round once the previous step's update has consumed that round's
    gradients; round r's update waits for its upload and for the previous
    step's read-back of its model values; round r's values download on a
    second stream while round r+1 updates.  PCIe then carries both directions
    at once and the updates hide under the copies.  With the ZeRO-2 reduction
    every rank's full gradients must be in place before any rank's first
    round, so there the upload precedes the step.  The timed region ends
    after the last read-back; afterwards a strided sample of the host copy is
    compared with the device model."""
    cur = torch.cuda.current_stream(dev)
    up = torch.cuda.Stream(dev)
    side = torch.cuda.Stream(dev)
    R = len(opt.segments)
    zero2 = opt.grad_reduce == "multicast"
    if zero2:
        seg_rounds = [[(ti, 0, p.numel(), 0) for ti, p in enumerate(opt.params)]]
    else:
        seg_rounds = [list(opt.segments[r]) for r in range(R)]
    host_g = [[opt.params[ti].grad.reshape(-1)[s:s + n].to("cpu").pin_memory()
               for ti, s, n, _ in segs] for segs in seg_rounds]
    small = [opt.all_params[i] for i in opt.sindex]
    host_gs = [p.grad.to("cpu").pin_memory() for p in small]
    owned = list(opt.owned)
    host_p = [torch.empty(b - a, dtype=opt.flat.dtype, pin_memory=True) if b > a else None
              for a, b in owned]
    h2d = sum(h.numel() * h.element_size() for hs in host_g for h in hs)
    h2d += sum(h.numel() * h.element_size() for h in host_gs)
    d2h = sum(h.numel() * h.element_size() for h in host_p if h is not None)

    def ev():
        e = torch.cuda.Event()
        e.record(cur)   # complete: nothing to wait for yet
        return e
    consumed = [ev() for _ in seg_rounds]   # the update has read these gradients
    read_back = [ev() for _ in owned]       # these model values are on the host
    stepped = ev()
    uploaded = [torch.cuda.Event() for _ in seg_rounds]
    small_up = torch.cuda.Event()

    def one():
        with torch.cuda.stream(up):
            if zero2:   # other ranks read these gradients until the step ends
                up.wait_event(stepped)
            for r, (segs, hs) in enumerate(zip(seg_rounds, host_g)):
                up.wait_event(consumed[r])
                for (ti, s, n, _), hg in zip(segs, hs):
                    opt.params[ti].grad.reshape(-1)[s:s + n].copy_(hg, non_blocking=True)
                uploaded[r].record(up)
            up.wait_event(stepped)          # the FP32-state tensors read theirs last
            for p, hg in zip(small, host_gs):
                p.grad.copy_(hg, non_blocking=True)
            small_up.record(up)

        def begin(r):
            cur.wait_event(uploaded[0] if zero2 else uploaded[r])
            cur.wait_event(read_back[r])

        def end(r):
            consumed[0 if zero2 else r].record(cur)
            side.wait_event(consumed[0 if zero2 else r])
            (a, b), hp = owned[r], host_p[r]
            if hp is not None:
                with torch.cuda.stream(side):
                    hp.copy_(opt.flat[a:b], non_blocking=True)
            read_back[r].record(side)
            if r == R - 1:   # the FP32-state update follows the last round
                cur.wait_event(small_up)

        if zero2:   # every rank's gradients in place before the step's first round
            cur.wait_event(uploaded[0])
            cur.wait_event(small_up)
        opt.step(round_begin=begin, round_end=end)
        stepped.record(cur)

    one()
    cur.wait_stream(side)           # the timed region starts with idle copy streams
    cur.wait_stream(up)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.e2e_steps):
        one()
    cur.wait_stream(side)           # the last read-back is inside the timed region
    cur.wait_stream(up)
    e1.record(cur)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    torch.cuda.synchronize()
    for (a, b), hp in zip(owned, host_p):
        if hp is None:
            continue
        stride = max(1, (b - a) // 4099)
        if not torch.equal(hp[::stride].to(dev), opt.flat[a:b][::stride]):
            raise RuntimeError("e2e: the host copy does not hold the stepped model")
    del host_g, host_gs, host_p
    return {"value": total * args.e2e_steps / (ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "bytes_are_per_rank": world > 1, "ms_per_step": ms / args.e2e_steps,
            "steps": args.e2e_steps, "pipelined_rounds": 1 if zero2 else R,
            "readback_checked": True}


def probe_pcie(args) -> None:
    """Pinned host <-> device copy rates of the GPU box (the floor of `e2e`):
    one 4 GB BF16 buffer each way, upload alone, download alone and both at
    once on two streams; best of 3, GB/s per direction."""
    dev = torch.device("cuda", 0)
    n = (4 << 30) // 2
    hg = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    hp = torch.empty(n, dtype=torch.bfloat16).pin_memory()
    hg.fill_(1.0)
    dg = torch.empty(n, dtype=torch.bfloat16, device=dev)
    dp = torch.ones(n, dtype=torch.bfloat16, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    out = {"probe": "pcie", "bytes_per_direction": 2 * n}
    for name, up, down in (("h2d_gbs", True, False), ("d2h_gbs", False, True),
                           ("both_gbs_each_way", True, True)):
        best = 0.0
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if up:
                with torch.cuda.stream(s1):
                    dg.copy_(hg, non_blocking=True)
            if down:
                with torch.cuda.stream(s2):
                    hp.copy_(dp, non_blocking=True)
            torch.cuda.synchronize()
            best = max(best, 2 * n / (time.perf_counter() - t0) / 1e9)
        out[name] = round(best, 1)
    print(json.dumps(out), flush=True)


def probe_ld_reduce(args, rank: int, world: int, local: int) -> None:
    """multimem.ld_reduce through NVSwitch against NCCL's reduce-scatter
    (torchrun, one rank per GPU).  Each rank reduces its shard of a 2 GB
    symmetric buffer into a local FP32 buffer with aw4_reduce_multicast (the
    FP32-state path of the ZeRO-2 step), BF16 and FP32; NCCL's
    reduce_scatter_tensor runs on the same bytes.  10 launches after 3
    warm-ups, max over ranks.  A rank's egress is its whole buffer: the
    switch reads every rank's copy of a shard, the owner's own included."""
    import ctypes

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    from adamw4bit_b200 import _native as N
    dev = torch.device("cuda", local)
    if symm_mem.get_backend(dev) is None:
        symm_mem.set_backend("CUDA")
    lib = N.lib()
    cur = torch.cuda.current_stream(dev)
    reps = 10
    for dt, n in ((torch.bfloat16, 1 << 30), (torch.float32, 1 << 29)):
        buf = symm_mem.empty(n, dtype=dt, device=dev)
        mc = int(symm_mem.rendezvous(buf, dist.group.WORLD).multicast_ptr)
        buf.fill_(float(rank + 1))
        shard, esz = n // world, buf.element_size()
        res = torch.empty(shard, dtype=torch.float32, device=dev)

        def reduce():
            N.check(lib.aw4_reduce_multicast(ctypes.c_void_p(mc + rank * shard * esz),
                                             N.DTYPE_CODES[dt], shard, 1.0,
                                             ctypes.c_void_p(res.data_ptr()), local,
                                             ctypes.c_void_p(cur.cuda_stream)),
                    "aw4_reduce_multicast")
        src = torch.full((n,), float(rank + 1), dtype=dt, device=dev)
        dst = torch.empty(shard, dtype=dt, device=dev)

        def timed(fn) -> float:
            for _ in range(3):
                fn()
            barrier(world)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            for _ in range(reps):
                fn()
            e1.record(cur)
            barrier(world)
            return max_over_ranks(e0.elapsed_time(e1) / reps, world)
        ms = timed(reduce)
        correct = bool(torch.all(res == world * (world + 1) / 2).item())
        ms_nccl = timed(lambda: dist.reduce_scatter_tensor(dst, src))
        if rank == 0:
            print(json.dumps({"probe": "ld_reduce", "dtype": str(dt).replace("torch.", ""),
                              "world": world, "buffer_bytes": n * esz,
                              "ld_reduce_ms": round(ms, 3),
                              "shard_sums_in_gbs": round(shard * esz / ms / 1e6, 1),
                              "egress_gbs": round(n * esz / ms / 1e6, 1),
                              "nccl_reduce_scatter_ms": round(ms_nccl, 3),
                              "correct": correct}), flush=True)
        del buf, res, src, dst
        barrier(world)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu", "reference-gpu-eager",
                                       "reference-cpu", "reference-cpu-eager",
                                       "probe-pcie", "probe-ld-reduce"],
                    default="ours",
                    help="probe-pcie / probe-ld-reduce: the copy and NVSwitch-reduction "
                         "rates that bound e2e and the ZeRO-2 step (not bench lines)")
    ap.add_argument("--rounds", type=int, default=4,
                    help="rounds per step: one update launch each (and, at N>1, one gather)")
    ap.add_argument("--recipe", choices=["ze-eden", "zip-sr"], default="ze-eden",
                    help="the optimizer recipe (BASELINE config 5 is ZE-EDEN)")
    ap.add_argument("--grad-reduce", choices=["local", "multicast"], default="local",
                    help="N>1: gradients already reduced (local), or ZeRO-2 with the "
                         "reduce-scatter fused into the update through NVSwitch (multicast)")
    ap.add_argument("--reserve-sms", type=int, default=16,
                    help="N>1: SMs the update grid leaves to the concurrent all-gather")
    ap.add_argument("--gather", choices=["auto", "multicast", "bf16", "fp32"], default="auto",
                    help="N>1: the BF16 model copy of the FP32 masters written to every "
                         "replica by the update kernel through NVSwitch multicast, or "
                         "all-gathered by NCCL (bf16), or the FP32 parameters "
                         "all-gathered by NCCL; auto (default): multicast from 4 ranks "
                         "up, bf16 below (multicast falls back to NCCL where the "
                         "platform has none)")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--compile-compat", action="store_true",
                    help="--impl reference-gpu/-cpu: let the reference's optimized path "
                         "run on this torch by dropping the isolate_recompiles keyword "
                         "it passes to torch.compile")
    ap.add_argument("--no-legs", dest="legs", action="store_false",
                    help="N=1: skip the drop-in and ZIP-SR legs")
    ap.add_argument("--cpu-sample", type=int, default=1 << 27,
                    help="values in the CPU-oracle sample (0: skip)")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=None, help="fewer decoder layers (smaller case)")
    ap.add_argument("--values", type=int, default=0,
                    help="one tensor of this many values instead of the Llama-3-8B set "
                         "(small profiling case)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl.startswith("reference-"):
        run_reference_torch(args, int(os.environ.get("RANK", "0")),
                            "cuda" if "gpu" in args.impl else "cpu",
                            eager=args.impl.endswith("-eager"))
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, rank, int(os.environ.get("WORLD_SIZE", "1")))
        return
    if args.impl == "probe-pcie":
        probe_pcie(args)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "probe-ld-reduce":
            probe_ld_reduce(args, rank, world, local)
            return
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
