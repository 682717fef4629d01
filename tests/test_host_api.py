"""Host-side logic of the drop-in optimizer API, without a GPU: constructor
validation (the reference's messages), the scope checks, the per-step float32
scalars, checkpoint payload handling and the ZeRO-1 shard plan (also across
two gloo ranks)."""

from __future__ import annotations

import copy
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adamw4bit_b200 import AdamW8bit, QuantizedAdamW, ZEEDENAdamW4Bit, ZIPSRAdamW4Bit
from adamw4bit_b200.optimizer import _overlapping_pairs, byte_range, hyper_scalars
from adamw4bit_b200.quantization import QuantState, default_block_size, is_4bit_scheme
from adamw4bit_b200.zero import ShardPlan, grad_layout


def _p(n=4096):
    return torch.nn.Parameter(torch.linspace(-1.0, 1.0, n))


@pytest.mark.parametrize("kwargs,match", [
    (dict(lr=-1.0), "Invalid learning rate"),
    (dict(eps=-1.0), "Invalid epsilon value"),
    (dict(betas=(1.0, 0.9)), "Invalid beta parameter at index 0"),
    (dict(betas=(0.9, 1.0)), "Invalid beta parameter at index 1"),
    (dict(weight_decay=-0.1), "Invalid weight_decay value"),
    (dict(quant_rng_seed=-1), "quant_rng_seed must be a non-negative integer"),
    (dict(quant_rng_seed=True), "quant_rng_seed must be a non-negative integer"),
    (dict(m1_quant_scheme="nope"), "m1_quant_scheme must be one of"),
    (dict(m2_quant_scheme="dyn4_sr", use_eden_m2=True), "Vanilla stochastic-rounding"),
    (dict(m1_quant_scheme="fp32", m2_quant_scheme="dyn4_upd_sr_store_eden", use_eden_m2=True),
     "EDEN is built into the store path"),
    (dict(m1_quant_scheme="sdyn4", m2_quant_scheme="dyn4_la_upd_sr"), "supports m1_quant_scheme"),
    (dict(update_sign_clip=1.0, update_norm_clip=1.0), "Set at most one"),
])
def test_constructor_validation_matches_reference_messages(kwargs, match):
    """Messages of adamw.py:148-208 (and the reference tests that match them)."""
    with pytest.raises(ValueError, match=match):
        QuantizedAdamW([_p()], **kwargs)


@pytest.mark.parametrize("kwargs", [
    dict(telemetry=lambda *a: None, m1_quant_scheme="nf4", m2_quant_scheme="dyn4_nz"),
    dict(update_sign_clip=0.5, m1_quant_scheme="nf4", m2_quant_scheme="dyn4_nz"),
    dict(record_preconditioner_steps=[1], m1_quant_scheme="nf4", m2_quant_scheme="dyn4_nz"),
    dict(m1_quant_scheme="linear", m2_quant_scheme="linear"),
    dict(m1_quant_scheme="nf4", m2_quant_scheme="dyn4_upd_sr"),
    dict(m1_quant_scheme="nf4", m2_quant_scheme="fp32"),
    dict(m1_quant_scheme="nf4", m2_quant_scheme="dyn4_nz", block_size=64),
])
def test_out_of_scope_options_fail_loudly(kwargs):
    with pytest.raises(NotImplementedError):
        QuantizedAdamW([_p()], **kwargs)


def test_fp32_m1_next_to_a_4bit_m2_is_accepted():
    """The reference resolves each moment's scheme on its own (adamw.py:510-521)."""
    opt = QuantizedAdamW([_p()], m1_quant_scheme="fp32", m2_quant_scheme="dyn4_upd_sr_fp32read")
    assert opt.param_groups[0]["m1_quant_scheme"] == "fp32"


def test_recipes_fix_the_paper_schemes():
    ze = ZEEDENAdamW4Bit([_p()])
    zs = ZIPSRAdamW4Bit([_p()])
    assert (ze.param_groups[0]["m1_quant_scheme"], ze.param_groups[0]["m2_quant_scheme"],
            ze.param_groups[0]["use_eden_m2"]) == ("nf4", "dyn4_nz", True)
    assert (zs.param_groups[0]["m1_quant_scheme"], zs.param_groups[0]["m2_quant_scheme"],
            zs.param_groups[0]["use_eden_m2"]) == ("nf4", "dyn4_upd_sr_fp32read", False)
    a8 = AdamW8bit([_p()], m1_quant_scheme="sdyn4", m2_quant_scheme="lin4_nz")
    assert a8.param_groups[0]["m2_quant_scheme"] == "lin4_nz"


def test_runtime_m1_retargeting_validation():
    p, q = _p(), _p()
    opt = ZEEDENAdamW4Bit([p])
    with pytest.raises(ValueError, match="supports only nf4 and nf4_sr"):
        opt.set_m1_quant_scheme_for_parameters([p], "sdyn4")
    with pytest.raises(ValueError, match="requires parameters"):
        opt.set_m1_quant_scheme_for_parameters([], "nf4_sr")
    with pytest.raises(ValueError, match="outside optimizer"):
        opt.set_m1_quant_scheme_for_parameters([q], "nf4_sr")
    opt.set_m1_quant_scheme_for_parameters([p], "nf4_sr")
    assert opt._m1_scheme_for(p, "nf4") == "nf4_sr"


def test_step_on_cpu_tensors_fails_loudly():
    p = _p()
    opt = ZEEDENAdamW4Bit([p])
    p.grad = torch.ones_like(p)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        opt.step()


def test_byte_range_overlap_sweep():
    """Overlap detection of the pre-launch alias checks (the reference's
    tensor_byte_range / overlaps, _moment_buffer.py:13-24): views of one
    buffer overlap exactly when their byte ranges intersect, non-contiguous
    views count their whole storage, and empty tensors never overlap."""
    base = torch.zeros(1024)
    a, b, c = base[0:512], base[511:600], base[600:700]
    other = torch.zeros(64)
    whole = torch.zeros(64, 4)
    strided = whole[:, 1]
    regions = [(*byte_range(a), 0, "param"), (*byte_range(b), 1, "param"),
               (*byte_range(c), 2, "grad"), (*byte_range(other), 3, "m1_code"),
               (*byte_range(torch.zeros(0)), 4, "m2_code")]
    pairs = {frozenset(p) for p in _overlapping_pairs(regions)}
    assert pairs == {frozenset({(0, "param"), (1, "param")})}
    d, s0, e0 = byte_range(strided)
    assert e0 - s0 == 64 * 4 * 4   # the whole storage
    regions += [(d, s0, e0, 5, "m2_absmax"), (*byte_range(whole[0, :1]), 6, "param")]
    pairs = {frozenset(p) for p in _overlapping_pairs(regions)}
    assert frozenset({(5, "m2_absmax"), (6, "param")}) in pairs


def test_eligibility_mirrors_torchao_rule():
    f = QuantizedAdamW._eligible_for_quantized_state
    assert f(torch.empty(4096), 128) and f(torch.empty(50257 * 768), 128)
    assert not f(torch.empty(768), 128) and not f(torch.empty(4097), 128)
    assert not f(torch.empty(2048), 128)


def test_scheme_helpers():
    assert is_4bit_scheme("nf4") and is_4bit_scheme("dyn4_nz") and not is_4bit_scheme("linear")
    assert default_block_size("dyn4_upd_sr_fp32read") == 128
    assert default_block_size("dynamic") == 256


def test_hyper_scalars_are_float32_roundings_of_float64_math():
    h = hyper_scalars(1e-3, 0.9, 0.95, 1e-8, 0.1, 3, False)
    bc1, bc2 = 1 - 0.9 ** 3, 1 - 0.95 ** 3
    assert h["w1"] == float(np.float32(1 - 0.9)) and h["w2"] == float(np.float32(1 - 0.95))
    assert h["neg_step"] == float(np.float32(-(1e-3 / bc1)))
    assert h["sqrt_bc2"] == float(np.float32(bc2 ** 0.5))
    assert h["decay"] == float(np.float32(1 - 1e-3 * 0.1))
    assert h["sr_bias"] == float(np.float32(bc2))
    h2 = hyper_scalars(1e-3, 0.9, 0.95, 1e-8, 0.1, 3, True)
    assert h2["sr_bias"] == float(np.float32(1 - 0.95 ** 4))


@pytest.mark.parametrize("scheme,bias_step", [
    ("lin4_upd_sr_fp32read", 1), ("dyn4_upd_sr_fp32read", 1),
    ("dyn4_lookahead_sr", 2), ("dyn4_upd_sr_fp32read_nextbc", 2)])
def test_update_sr_storage_bias_correction(scheme, bias_step):
    """Reference tests/quantization/test_dyn4_la_upd_sr.py:240-275: at t = 1
    the fp32-read schemes store against c_t = 1 - beta2^t, the lookahead SR
    scheme and its nextbc alias against c_{t+1}; the kernel receives that
    value as the float32 sr_bias of the step's scalars."""
    from adamw4bit_b200.quantization import SCHEMES
    h = hyper_scalars(1e-3, 0.9, 0.95, 1e-8, 0.0, 1, SCHEMES[scheme].next_bias)
    assert h["sr_bias"] == float(np.float32(1 - 0.95 ** bias_step))


def _fake_state(opt, p):
    n = p.numel()
    opt.state[p] = {
        "step": 2,
        "m1_code": torch.full((n // 2,), 0x77, dtype=torch.uint8),
        "m1_quant_state": QuantState(torch.full((n // 128,), 0.5), p.shape, torch.float32, 128, True),
        "m2_code": torch.full((n // 2,), 0x11, dtype=torch.uint8),
        "m2_quant_state": QuantState(torch.full((n // 128,), 0.25), p.shape, torch.float32, 128, True),
    }


def test_state_dict_layout_and_roundtrip_without_stepping():
    p = _p()
    opt = ZIPSRAdamW4Bit([p], quant_rng_seed=43)
    _fake_state(opt, p)
    sd = opt.state_dict()
    assert isinstance(sd["state"][0]["m1_quant_state"], dict)
    assert set(sd["state"][0]["m1_quant_state"]) == {"absmax", "shape", "dtype", "blocksize", "packed"}
    assert sd["_quant_rng_state"] == {"version": 2, "seed": 43, "stream": "philox4x32-10"}
    q = torch.nn.Parameter(p.detach().clone())
    opt2 = ZIPSRAdamW4Bit([q], quant_rng_seed=43)
    opt2.load_state_dict(copy.deepcopy(sd))
    st = opt2.state[q]
    assert isinstance(st["m1_quant_state"], QuantState) and st["m1_quant_state"].packed
    assert st["m1_code"].dtype == torch.uint8
    torch.testing.assert_close(st["m2_quant_state"].absmax, torch.full((32,), 0.25), rtol=0, atol=0)


def test_reference_v1_rng_payload_loads_and_bad_payloads_fail():
    p = _p()
    opt = ZIPSRAdamW4Bit([p], quant_rng_seed=43)
    _fake_state(opt, p)
    sd = opt.state_dict()
    v1 = dict(sd)
    v1["_quant_rng_state"] = {"version": 1, "seed": 43,
                              "states": {"m1": {"cpu": torch.Generator().get_state()}, "m2": {}}}
    ZIPSRAdamW4Bit([torch.nn.Parameter(p.detach().clone())], quant_rng_seed=43).load_state_dict(v1)
    torch_mode = ZIPSRAdamW4Bit([torch.nn.Parameter(p.detach().clone())], quant_rng_seed=43,
                                quant_rng="torch")
    torch_mode.load_state_dict(copy.deepcopy(v1))
    assert "cpu" in torch_mode._pending_quant_rng_states["m1"]
    bad = dict(sd)
    bad["_quant_rng_state"] = {"version": 9, "seed": 43}
    with pytest.raises(ValueError, match="Unsupported quantization RNG checkpoint version"):
        ZIPSRAdamW4Bit([torch.nn.Parameter(p.detach().clone())], quant_rng_seed=43).load_state_dict(bad)
    with pytest.raises(ValueError, match="seed mismatch"):
        ZIPSRAdamW4Bit([torch.nn.Parameter(p.detach().clone())], quant_rng_seed=44).load_state_dict(
            copy.deepcopy(sd))
    with pytest.raises(ValueError, match="quant_rng_seed is disabled"):
        ZIPSRAdamW4Bit([torch.nn.Parameter(p.detach().clone())]).load_state_dict(copy.deepcopy(sd))


def test_torch_stream_mode_writes_reference_v1_payload():
    p = _p()
    opt = ZIPSRAdamW4Bit([p], quant_rng_seed=43, quant_rng="torch")
    opt._quant_generator("m2", torch.device("cpu"))
    sd = opt.state_dict()
    assert sd["_quant_rng_state"]["version"] == 1
    assert "cpu" in sd["_quant_rng_state"]["states"]["m2"]


@pytest.mark.parametrize("world,rounds", [(1, 1), (2, 1), (2, 4), (8, 3)])
def test_shard_plan_covers_every_value_once(world, rounds):
    sizes = [128256 * 4, 4096 * 4096 // 64, 4096, 1024 * 4096 // 16, 4096]
    seen = np.zeros(sum(sizes), np.int32)
    starts = np.cumsum([0] + sizes[:-1])
    for r in range(world):
        plan = ShardPlan(sizes, world, r, rounds)
        assert plan.chunk % 128 == 0
        offs = set()
        for segs in plan.segments:
            for ti, s, n, so in segs:
                assert s % 128 == 0 and n % 128 == 0 and so % 128 == 0
                seen[starts[ti] + s: starts[ti] + s + n] += 1
                offs.add(so)
                assert so + n <= plan.state_numel()
    assert (seen == 1).all()


def test_zero2_grad_layout_is_disjoint_and_aligned():
    """ZeRO-2 gradient buffer: sharded tensors at their flat-model offsets,
    the FP32-state tensors after the padded model, each at a 16-byte
    (8-value) boundary, no overlaps."""
    sizes = [4096, 128 * 96, 8192]
    plan = ShardPlan(sizes, 2, 0, 2)
    small = [768, 300, 5, 8]
    qoffs, soffs, total = grad_layout(plan.starts, plan.padded, small)
    assert qoffs == plan.starts
    spans = [(o, o + n) for o, n in zip(qoffs, sizes)] + [(o, o + n) for o, n in zip(soffs, small)]
    spans.sort()
    assert all(a[1] <= b[0] for a, b in zip(spans, spans[1:]))
    assert all(o % 8 == 0 for o in soffs) and soffs[0] >= plan.padded
    assert total % 8 == 0 and total >= soffs[-1] + small[-1]


def _gloo_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sizes = [4096 * 3, 128 * 40, 8192, 4096]
        plan = ShardPlan(sizes, world, rank, 3)
        owned = torch.zeros(sum(sizes), dtype=torch.int32)
        starts = np.cumsum([0] + sizes[:-1])
        for segs in plan.segments:
            for ti, s, n, _ in segs:
                owned[starts[ti] + s: starts[ti] + s + n] += 1
        dist.all_reduce(owned)
        # emulate the in-place all-gather of each round on CPU
        flat = torch.full((plan.padded,), -1.0)
        for a, b in plan.owned:
            flat[a:b] = float(rank)
        for i in range(plan.rounds):
            base = i * world * plan.chunk
            region = flat[base:base + world * plan.chunk]
            parts = list(region.chunk(world))
            mine = parts[rank].clone()
            gathered = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(gathered, mine)
            region.copy_(torch.cat(gathered))
        ok = bool((owned == 1).all()) and bool((flat[: plan.total] >= 0).all())
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_shard_plan_with_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    results = [q.get(timeout=120) for _ in procs]
    for pr in procs:
        pr.join(timeout=60)
    assert all(ok for _, ok in results), results
