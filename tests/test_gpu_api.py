"""The drop-in Python API on the GPU: the reference's optimizer behaviours
(checkpoint resume, legacy state, the m1 switch, eligibility) and the
codec, plus the distributional bar for Philox stochastic rounding."""

from __future__ import annotations

import copy
import io

import numpy as np
import pytest
import torch

from adamw4bit_b200 import AdamW8bit, QuantizedAdamW, ZEEDENAdamW4Bit, ZIPSRAdamW4Bit, _native
from adamw4bit_b200 import quantization as Q
from adamw4bit_b200.quantization import QuantState
from oracle import oracle as O
from tests import golden_io as G

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
RECIPES = [ZEEDENAdamW4Bit, ZIPSRAdamW4Bit]


def _step(optimizer, parameter, step):
    generator = torch.Generator().manual_seed(123 + step)
    parameter.grad = torch.randn(parameter.shape, generator=generator).to(parameter)
    optimizer.step()


def _assert_state_equal(first, second):
    assert first.keys() == second.keys()
    for key, value in first.items():
        other = second[key]
        if isinstance(value, QuantState):
            assert isinstance(other, QuantState)
            assert (value.shape, value.dtype, value.blocksize, value.packed) == \
                (other.shape, other.dtype, other.blocksize, other.packed)
            torch.testing.assert_close(value.absmax, other.absmax, rtol=0, atol=0)
        elif torch.is_tensor(value):
            torch.testing.assert_close(value, other, rtol=0, atol=0, equal_nan=True)
        else:
            assert value == other


@pytest.mark.parametrize("optimizer_class", RECIPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("numel", [768, 4096])
@pytest.mark.parametrize("quant_rng", ["philox", "torch"])
def test_serialized_checkpoint_resumes_exactly(optimizer_class, dtype, numel, quant_rng):
    """Reference tests/adamw/test_checkpoint_io.py:38-74 on the GPU."""
    parameter = torch.nn.Parameter(torch.ones(numel, device=DEV, dtype=dtype))
    optimizer = optimizer_class([parameter], quant_rng_seed=43, quant_rng=quant_rng)
    optimizer.set_m1_quant_scheme_for_parameters([parameter], "nf4_sr")
    for step in range(3):
        _step(optimizer, parameter, step)
    buffer = io.BytesIO()
    torch.save(optimizer.state_dict(), buffer)
    buffer.seek(0)
    checkpoint = torch.load(buffer, map_location="cpu")
    if numel == 4096:
        assert isinstance(checkpoint["state"][0]["m1_quant_state"], dict)
    resumed_parameter = torch.nn.Parameter(parameter.detach().clone())
    resumed = optimizer_class([resumed_parameter], quant_rng_seed=43, quant_rng=quant_rng)
    resumed.set_m1_quant_scheme_for_parameters([resumed_parameter], "nf4_sr")
    resumed.load_state_dict(checkpoint)
    _assert_state_equal(optimizer.state[parameter], resumed.state[resumed_parameter])
    for step in range(3, 5):
        _step(optimizer, parameter, step)
        _step(resumed, resumed_parameter, step)
        torch.testing.assert_close(parameter, resumed_parameter, rtol=0, atol=0)
        _assert_state_equal(optimizer.state[parameter], resumed.state[resumed_parameter])


def test_cpu_checkpoint_moves_scales_to_cuda():
    """Reference tests/adamw/test_checkpoint_io.py:100-122: a checkpoint whose
    tensors live on the CPU loads onto the parameter's CUDA device."""
    parameter = torch.nn.Parameter(torch.ones(4096, device=DEV))
    optimizer = ZEEDENAdamW4Bit([parameter])
    _step(optimizer, parameter, 0)
    checkpoint = copy.deepcopy(optimizer.state_dict())
    for st in checkpoint["state"].values():
        for k, v in list(st.items()):
            if torch.is_tensor(v):
                st[k] = v.cpu()
            elif isinstance(v, dict):
                v["absmax"] = v["absmax"].cpu()
    resumed_parameter = torch.nn.Parameter(parameter.detach().clone())
    resumed = ZEEDENAdamW4Bit([resumed_parameter])
    resumed.load_state_dict(checkpoint)
    for moment in ("m1", "m2"):
        st = resumed.state[resumed_parameter]
        assert st[f"{moment}_code"].device == DEV
        assert st[f"{moment}_quant_state"].absmax.device == DEV
    _step(resumed, resumed_parameter, 1)
    _step(optimizer, parameter, 1)
    torch.testing.assert_close(parameter, resumed_parameter, rtol=0, atol=0)


def test_legacy_unpacked_state_is_read_and_repacked():
    """Reference tests/adamw/test_packed_state.py:54-78."""
    parameter = torch.nn.Parameter(torch.linspace(-1.0, 1.0, 4096, device=DEV))
    twin = torch.nn.Parameter(parameter.detach().clone())
    kw = dict(lr=1e-3, weight_decay=0.0, betas=(0.9, 0.95), m1_quant_scheme="sdyn4",
              m2_quant_scheme="dyn4_nz")
    optimizer, reference = AdamW8bit([parameter], **kw), AdamW8bit([twin], **kw)
    for opt, p in ((optimizer, parameter), (reference, twin)):
        p.grad = torch.linspace(-0.5, 0.5, 4096, device=DEV)
        opt.step()
    state = optimizer.state[parameter]
    for key in ("m1", "m2"):
        qs = state[f"{key}_quant_state"]
        state[f"{key}_code"] = Q.unpack_4bit_codes(state[f"{key}_code"], numel=4096).reshape(4096)
        qs.packed = False
    for opt, p in ((optimizer, parameter), (reference, twin)):
        p.grad = torch.linspace(-0.25, 0.25, 4096, device=DEV)
        opt.step()
    assert state["m1_code"].numel() == 2048 and state["m1_quant_state"].packed is True
    torch.testing.assert_close(parameter, twin, rtol=0, atol=0)
    torch.testing.assert_close(state["m2_code"], reference.state[twin]["m2_code"], rtol=0, atol=0)


def test_zeeden_golden_trajectory_through_public_api():
    """The reference's ZE-EDEN trajectory (RTN: no draws involved) reproduced by
    ZEEDENAdamW4Bit.step() on the GPU: codes/scales bit-exact every step."""
    meta, arrays = G.load_traj("zeeden_switch_small")
    rep = G.Replay(meta)
    params = [torch.nn.Parameter(p.to(DEV)) for p in rep.init_params()]
    opt = ZEEDENAdamW4Bit(params, lr=meta["lr"], betas=tuple(meta["betas"]), eps=meta["eps"],
                          weight_decay=meta["weight_decay"], quant_rng_seed=meta["quant_rng_seed"],
                          quant_rng="torch")
    # torch mode draws from CUDA generators; for the CPU fixture, feed the
    # reference's CPU draws through the same hook the optimizer uses
    for t in range(1, meta["steps"] + 1):
        inp = rep.next()
        if meta["switch_at"] is not None and t == meta["switch_at"]:
            opt.set_m1_quant_scheme_for_parameters([params[0]], "nf4_sr")
        for p, g in zip(params, inp.grads):
            p.grad = g.to(DEV)
        if inp.m1_draws[0] is not None:
            d1 = torch.from_numpy(inp.m1_draws[0]).to(DEV)
            opt._draws_override = {id(params[0]): (d1, None)}
        else:
            opt._draws_override = None
        opt.step()
        rec = meta["per_step"][t - 1]
        st = opt.state[params[0]]
        assert G.sha(st["m1_code"].cpu()) == rec["m1_code"], t
        assert G.sha(st["m2_code"].cpu()) == rec["m2_code"], t
        assert G.sha(st["m1_quant_state"].absmax.cpu()) == rec["m1_absmax"], t
        assert G.sha(st["m2_quant_state"].absmax.cpu()) == rec["m2_absmax"], t
        np.testing.assert_allclose(params[0].detach().cpu().numpy().reshape(-1)[::meta["sample_stride"]],
                                   arrays[f"s{t}_param_sample"], rtol=1e-6, atol=1e-9)
        for i, p in enumerate(params[1:], start=1):
            if f"s{t}_small{i}_param" in arrays:
                np.testing.assert_allclose(p.detach().cpu().numpy(), arrays[f"s{t}_small{i}_param"],
                                           rtol=1e-6, atol=1e-9)


def test_torch_stream_mode_matches_oracle_fed_the_same_cuda_draws():
    """quant_rng='torch' draws in the reference's order from per-moment CUDA
    generators; the oracle fed those same uniforms gives identical state."""
    n = 128 * 64
    seed = 17
    p0 = torch.randn(n, generator=torch.Generator().manual_seed(0)) * 0.02
    param = torch.nn.Parameter(p0.to(DEV))
    opt = ZIPSRAdamW4Bit([param], quant_rng_seed=seed, quant_rng="torch")
    g1 = torch.Generator(device=DEV).manual_seed((seed + O.M1_OFFSET) % ((1 << 63) - 1))
    g2 = torch.Generator(device=DEV).manual_seed((seed + O.M2_OFFSET) % ((1 << 63) - 1))
    pr = p0.numpy().copy()
    c1, s1 = O.init_zero("nf4", n)
    c2, s2 = O.init_zero("dyn4_upd_sr_fp32read", n)
    for t in range(1, 4):
        grad = torch.randn(n, generator=torch.Generator().manual_seed(t)) * 1e-3
        param.grad = grad.to(DEV)
        opt.step()
        if t == 1:
            torch.rand((n // 128, 128), device=DEV, generator=g2)  # init draw (adamw.py:537-545)
        d2 = torch.rand((n // 128, 128), device=DEV, generator=g2).reshape(-1).cpu().numpy()
        cfg = O.make_cfg(m1_scheme="nf4", m2_scheme="dyn4_upd_sr_fp32read", eden=False, lr=1e-3,
                         betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, step=t)
        O.step(cfg, pr, grad.numpy().copy(), c1, s1, c2, s2, None, d2)
        st = opt.state[param]
        np.testing.assert_array_equal(st["m2_code"].cpu().numpy(), c2)
        np.testing.assert_array_equal(st["m1_code"].cpu().numpy(), c1)
        np.testing.assert_array_equal(param.detach().cpu().numpy().view(np.uint32), pr.view(np.uint32))
    del g1


@pytest.mark.parametrize("scheme", ["dyn4_upd_sr_fp32read", "nf4_sr", "dyn4_sr"])
def test_philox_sr_is_distributionally_equal_to_reference_draws(scheme):
    """North-star bar for SR under Philox: the dequantized moments have the
    same mean and variance as with torch.rand uniforms (the reference's draws),
    and the codes' frequencies agree, over many independent streams."""
    n = 128 * 512
    rng = np.random.default_rng(5)
    x = np.abs(rng.standard_normal(n)).astype(np.float32) * np.float32(1e-6)
    if Q.SCHEMES[scheme].signed:
        x *= np.sign(rng.standard_normal(n)).astype(np.float32)
    xt = torch.from_numpy(x).to(DEV)
    kw = dict(bias_correction=0.0975, eps=1e-8) if "upd" in scheme else {}
    prep = Q.prepared(scheme)
    means_p, means_t, hist_p, hist_t = [], [], np.zeros(16), np.zeros(16)
    for k in range(16):
        codes = torch.empty(n // 2, dtype=torch.uint8, device=DEV)
        scales = torch.empty(n // 128, dtype=torch.float32, device=DEV)
        _native.check(_native.lib().aw4_quantize_blocks(
            prep, 0, xt.data_ptr(), n, codes.data_ptr(), scales.data_ptr(), None, 1000 + k, 1, 0,
            float(np.float32(kw.get("bias_correction", 1.0))), float(np.float32(1e-8)), 0,
            torch.cuda.current_stream().cuda_stream), "quantize")
        deq_p = Q.dequantize(codes, QuantState(scales, (n,), torch.float32, 128, True), mode=scheme)
        u = torch.rand(n, device=DEV, generator=torch.Generator(device=DEV).manual_seed(k))
        ct, qt = Q.quantize(xt, mode=scheme, draws=u, **kw)
        deq_t = Q.dequantize(ct, qt, mode=scheme)
        means_p.append(deq_p.double().mean().item())
        means_t.append(deq_t.double().mean().item())
        hist_p += np.bincount(Q.unpack_4bit_codes(codes, numel=n).cpu().numpy(), minlength=16)
        hist_t += np.bincount(ct.reshape(-1).cpu().numpy(), minlength=16)
    mp, mt = np.mean(means_p), np.mean(means_t)
    sp, st = np.std(means_p), np.std(means_t)
    assert abs(mp - mt) <= 4 * max(sp, st) / np.sqrt(16) + 1e-12 * abs(mt), (mp, mt, sp, st)
    assert 0.5 < (sp + 1e-30) / (st + 1e-30) < 2.0
    # code frequencies within 4 sigma of a binomial around the torch-draw frequencies
    tot = hist_t.sum()
    pf = hist_t / tot
    sigma = np.sqrt(np.maximum(pf * (1 - pf) * tot, 1.0))
    assert np.all(np.abs(hist_p - hist_t) <= 5 * np.sqrt(2) * sigma + 5), (hist_p, hist_t)


def test_codec_api_matches_reference_codec_cases():
    """adamw4bit_b200.quantization.quantize/dequantize on the GPU reproduce the
    reference's codec golden cases (uniforms fed for SR)."""
    import json
    import os
    with open(os.path.join(G.GOLDEN, "codec_cases.json")) as f:
        meta = json.load(f)
    arrays = np.load(os.path.join(G.GOLDEN, "codec_cases.npz"))
    for case in meta:
        tag, scheme = case["tag"], case["scheme"]
        x = torch.from_numpy(arrays[f"{tag}_x"]).to(DEV)
        kw = {}
        if case["bias_correction"] is not None:
            kw = dict(bias_correction=case["bias_correction"], eps=case["eps"])
        draws = torch.from_numpy(arrays[f"{tag}_draws"]).to(DEV)
        codes, qs = Q.quantize(x, block_size=128, mode=scheme, eden_correction=case["eden"],
                               draws=draws, **kw)
        np.testing.assert_array_equal(codes.cpu().numpy(), arrays[f"{tag}_codes"], err_msg=tag)
        np.testing.assert_array_equal(qs.absmax.cpu().numpy().view(np.uint32),
                                      arrays[f"{tag}_scales"].view(np.uint32), err_msg=tag)
        deq = Q.dequantize(codes, qs, mode=scheme).cpu().numpy()
        want = O.dequantize(arrays[f"{tag}_codes"], arrays[f"{tag}_scales"], scheme)
        np.testing.assert_array_equal(deq.view(np.uint32), want.view(np.uint32))
    packed = Q.pack_4bit_codes(torch.tensor([1, 2, 15], dtype=torch.uint8, device=DEV))
    assert packed.cpu().tolist() == [0x21, 0x0F]   # reference test_utils.py:92-101


def test_one_fused_launch_per_step_for_a_many_tensor_model():
    """Quantized tensors of one dtype/scheme group step in a single launch;
    FP32-state tensors in one more; parameters without gradients are skipped."""
    params = [torch.nn.Parameter(torch.randn(s, device=DEV) * 0.02)
              for s in [(768, 64), (4096,), (128, 96), (768,), (2304,), (64, 64), (5000,)]]
    opt = ZEEDENAdamW4Bit(params)
    for p in params[:-1]:
        p.grad = torch.randn_like(p) * 1e-3
    opt.step()   # first step also launches the state initialisation
    before = _native.launch_count()
    for p in params[:-1]:
        p.grad = torch.randn_like(p) * 1e-3
    opt.step()
    assert _native.launch_count() - before == 2
    assert params[-1] not in opt.state
    assert "m1_code" in opt.state[params[0]] and "m1" in opt.state[params[3]]
    assert opt.state[params[0]]["step"] == 2


def test_unseeded_zipsr_steps_all_tensors_in_one_launch():
    """Without quant_rng_seed (the reference's default) the Philox keys are
    drawn once per step() call, not per parameter: a many-tensor ZIP-SR model
    still takes one quantized launch per step, and re-seeding the global RNG
    reproduces the codes."""
    shapes = [(256, 64)] * 40 + [(4096,), (128, 128)]

    def run():
        torch.manual_seed(123)
        params = [torch.nn.Parameter(torch.full(s, 0.01, device=DEV)) for s in shapes]
        opt = ZIPSRAdamW4Bit(params)
        gen = torch.Generator(device=DEV).manual_seed(5)
        counts = []
        for _ in range(3):
            for p in params:
                p.grad = torch.randn(p.shape, device=DEV, generator=gen) * 1e-3
            before = _native.launch_count()
            opt.step()
            counts.append(_native.launch_count() - before)
        return counts, torch.cat([opt.state[p]["m2_code"] for p in params])

    counts, codes_a = run()
    assert counts[1:] == [1, 1], counts          # step 1 also initialises the state
    _, codes_b = run()
    assert torch.equal(codes_a, codes_b)


def test_group_hyperparameters_and_mixed_dtypes_in_one_step():
    """Two parameter groups (different lr / weight decay) and BF16 next to
    FP32 parameters: each tensor matches the oracle with its own scalars."""
    a = torch.nn.Parameter((torch.randn(8192, generator=torch.Generator().manual_seed(1)) * 0.02).to(DEV))
    b = torch.nn.Parameter((torch.randn(4096, generator=torch.Generator().manual_seed(2)) * 0.02)
                           .to(DEV, torch.bfloat16))
    opt = ZEEDENAdamW4Bit([{"params": [a]}, {"params": [b], "lr": 3e-4, "weight_decay": 0.0}])
    oracles = []
    for p, lr, wd in ((a, 1e-3, 0.1), (b, 3e-4, 0.0)):
        n = p.numel()
        bits = p.detach().cpu().view(torch.int16).numpy().view(np.uint16).copy() \
            if p.dtype == torch.bfloat16 else p.detach().cpu().numpy().copy()
        oracles.append([bits, *O.init_zero("nf4", n), *O.init_zero("dyn4_nz", n, eden=True), lr, wd])
    for t in (1, 2):
        gs = [torch.randn(p.shape, generator=torch.Generator().manual_seed(10 * t + i)) * 1e-3
              for i, p in enumerate((a, b))]
        for p, g in zip((a, b), gs):
            p.grad = g.to(DEV, p.dtype)
        opt.step()
        for (bits, c1, s1, c2, s2, lr, wd), p, g in zip(oracles, (a, b), gs):
            dt = O.BF16 if p.dtype == torch.bfloat16 else O.F32
            gbits = g.to(p.dtype).view(torch.int16).numpy().view(np.uint16).copy() \
                if p.dtype == torch.bfloat16 else g.numpy().copy()
            cfg = O.make_cfg(m1_scheme="nf4", m2_scheme="dyn4_nz", eden=True, lr=lr,
                             betas=(0.9, 0.95), eps=1e-8, weight_decay=wd, step=t,
                             param_dtype=dt, grad_dtype=dt)
            O.step(cfg, bits, gbits, c1, s1, c2, s2)
            st = opt.state[p]
            np.testing.assert_array_equal(st["m2_code"].cpu().numpy(), c2)
            got = p.detach().cpu()
            got = got.view(torch.int16).numpy().view(np.uint16) if p.dtype == torch.bfloat16 \
                else got.numpy().view(np.uint32)
            np.testing.assert_array_equal(got, bits if p.dtype == torch.bfloat16 else bits.view(np.uint32))


def test_gradient_aliasing_its_parameter_is_read_before_the_update():
    """p.grad sharing p's storage: the step reads the whole gradient before
    writing the parameter, as the reference's eager step does (its GPU
    backend refuses such storage, _optimized.py:110-113)."""
    base = (torch.randn(4096, 8, generator=torch.Generator().manual_seed(3)) * 1e-3).to(DEV)
    a = torch.nn.Parameter(base.clone())
    b = torch.nn.Parameter(base.clone())
    opt_a, opt_b = ZEEDENAdamW4Bit([a]), ZEEDENAdamW4Bit([b])
    for _ in range(2):
        a.grad = a.detach()                 # same storage as the parameter
        b.grad = b.detach().clone()
        opt_a.step()
        opt_b.step()
    assert torch.equal(a.detach(), b.detach())
    assert torch.equal(opt_a.state[a]["m2_code"], opt_b.state[b]["m2_code"])


def test_overlapping_parameters_are_refused():
    """Two parameters over overlapping bytes cannot be updated by one
    concurrent launch the way eager updates them one after the other."""
    storage = torch.zeros(8192 + 128, device=DEV)
    p1 = torch.nn.Parameter(storage[:8192])
    p2 = torch.nn.Parameter(storage[128:])
    opt = ZEEDENAdamW4Bit([p1, p2])
    p1.grad = torch.ones_like(p1)
    p2.grad = torch.ones_like(p2)
    with pytest.raises(RuntimeError, match="overlaps another parameter"):
        opt.step()


def test_aliased_moment_state_after_load_is_detached():
    """A checkpoint whose two parameters share moment storage (the reference
    marks such state, _optimized.py:53-83): each parameter decodes the shared
    bytes, then writes its own storage, like the reference's eager step."""
    gen = torch.Generator().manual_seed(9)
    init = [torch.randn(64, 128, generator=gen) * 0.02 for _ in range(2)]
    grads = [[torch.randn(64, 128, generator=gen) * 1e-3 for _ in range(2)] for _ in range(3)]

    def run(alias):
        ps = [torch.nn.Parameter(x.clone().to(DEV)) for x in init]
        opt = ZEEDENAdamW4Bit(ps)
        for p, g in zip(ps, grads[0]):
            p.grad = g.to(DEV)
        opt.step()
        src = opt.state[ps[0]]
        for key in ("m1_code", "m2_code"):
            opt.state[ps[1]][key] = src[key] if alias else src[key].clone()
        for key in ("m1_quant_state", "m2_quant_state"):
            qs = copy.copy(src[key])
            qs.absmax = src[key].absmax if alias else src[key].absmax.clone()
            opt.state[ps[1]][key] = qs
        for t in (1, 2):
            for p, g in zip(ps, grads[t]):
                p.grad = g.to(DEV)
            opt.step()
        return ps, opt

    ps_a, opt_a = run(alias=True)
    ps_b, opt_b = run(alias=False)
    assert opt_a.state[ps_a[0]]["m1_code"].data_ptr() != opt_a.state[ps_a[1]]["m1_code"].data_ptr()
    for pa, pb in zip(ps_a, ps_b):
        assert torch.equal(pa.detach(), pb.detach())
        for key in ("m1_code", "m2_code"):
            assert torch.equal(opt_a.state[pa][key], opt_b.state[pb][key])


@pytest.mark.parametrize("scheme", ["lin4_upd_sr_fp32read", "dyn4_upd_sr_fp32read",
                                    "dyn4_lookahead_sr", "dyn4_upd_sr_fp32read_nextbc"])
def test_fp32_m1_first_step_matches_adamw_and_stores_quantized_m2(scheme):
    """Reference KAT tests/quantization/test_dyn4_la_upd_sr.py:151-191: an FP32
    m1 next to a 4-bit fp32read m2; the first step equals torch's AdamW, m2 is
    stored packed and decodes to finite values."""
    values = torch.linspace(-1.0, 1.0, steps=4096, device=DEV)
    grad = torch.linspace(-0.5, 0.5, steps=4096, device=DEV)
    p_q = torch.nn.Parameter(values.clone())
    p_f = torch.nn.Parameter(values.clone())
    kwargs = {"lr": 1e-3, "weight_decay": 0.0, "betas": (0.9, 0.95), "eps": 1e-8}
    opt_q = AdamW8bit([p_q], **kwargs, m1_quant_scheme="fp32", m2_quant_scheme=scheme,
                      block_size=128)
    opt_f = torch.optim.AdamW([p_f], **kwargs)
    p_q.grad = grad.clone()
    p_f.grad = grad.clone()
    opt_q.step()
    opt_f.step()
    torch.testing.assert_close(p_q, p_f, rtol=1e-6, atol=1e-6)
    state = opt_q.state[p_q]
    assert "m2_code" in state and "m2_quant_state" in state and "m2" not in state
    assert state["m1"].dtype == torch.float32 and "m1_code" not in state
    saved = Q.dequantize(state["m2_code"], state["m2_quant_state"], mode=scheme)
    assert saved.shape == p_q.shape and torch.isfinite(saved).all()


@pytest.mark.parametrize("name", ["fp32m1_zipsr", "fp32m1_zeeden", "fp32m1_lookahead",
                                  "nf4_lookahead", "nf4_nextbc", "nf4_lin4_fp32read"])
def test_scheme_pair_matches_reference_trajectory(name):
    """Scheme pairs through QuantizedAdamW, 6 steps against the reference's own
    run (its draws for the SR schemes): an FP32 m1 next to a 4-bit m2 (the
    reference resolves each moment's scheme on its own, adamw.py:510-521), and
    an nf4 m1 next to the fp32-read update-SR m2 schemes, whose storage bias is
    the next step's c_{t+1} (dyn4_lookahead_sr, dyn4_upd_sr_fp32read_nextbc)
    or c_t (lin4_upd_sr_fp32read; adamw.py:112-116, 655-683).  Codes, scales
    and FP32 moments bit-exact, parameters within rtol 1e-6."""
    import hashlib
    import json
    import os

    from tests import synth as S
    golden = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    with open(os.path.join(golden, f"mixed_{name}.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(golden, f"mixed_{name}.npz")))
    shapes = [tuple(s) for s in meta["shapes"]]
    params = [torch.nn.Parameter(S.init_param(s, i, torch.float32, DEV)) for i, s in enumerate(shapes)]
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
              m1_quant_scheme=meta["m1_scheme"], m2_quant_scheme=meta["m2_scheme"],
              use_eden_m2=meta["eden"])
    seed = meta["quant_rng_seed"]
    if seed is not None:
        kw["quant_rng_seed"] = seed
    opt = QuantizedAdamW(params, **kw)
    sr = Q.SCHEMES[meta["m2_scheme"]].round_mode != _native.RTN
    gen = torch.Generator().manual_seed((seed + G.M2_OFFSET) % ((1 << 63) - 1)) if sr else None
    for t in range(1, meta["steps"] + 1):
        for i, p in enumerate(params):
            p.grad = S.grad(p.shape, i, t, meta["grad_std"], torch.float32, DEV)
        if gen is not None:
            draws = {}
            for p in params:
                if p.numel() >= 4096 and p.numel() % 128 == 0:
                    rows = (p.numel() // 128, 128)
                    if t == 1:
                        torch.rand(rows, generator=gen)            # zero-state init
                    draws[id(p)] = (None, torch.rand(rows, generator=gen).reshape(-1).to(DEV))
            opt._draws_override = draws
        opt.step()
        hs = {k: hashlib.sha256() for k in ("m1_code", "m1_absmax", "m2_code", "m2_absmax",
                                            "f_m1", "f_m2")}
        for p in params:
            st = opt.state[p]
            for m in ("m1", "m2"):
                if f"{m}_code" in st:
                    hs[f"{m}_code"].update(st[f"{m}_code"].cpu().numpy().tobytes())
                    hs[f"{m}_absmax"].update(st[f"{m}_quant_state"].absmax.cpu().numpy().tobytes())
                else:
                    hs[f"f_{m}"].update(st[m].cpu().numpy().tobytes())
        rec = meta["per_step"][t - 1]
        for k, h in hs.items():
            assert h.hexdigest() == rec[k], f"{name} step {t}: {k}"
    for i, p in enumerate(params):
        np.testing.assert_allclose(p.detach().cpu().numpy(), arrays[f"s{meta['steps']}_p{i}"],
                                   rtol=1e-6, atol=1e-9)


def test_philox_trajectory_is_distributionally_equal_to_reference_draws():
    """The north star's bar for SR under Philox, at trajectory level: BASELINE
    configuration 2 (one 4096x4096 FP32 tensor, ZIP-SR, 10 steps) under 16
    seeds, once with the in-kernel Philox stream and once with the
    reference's own draws (its CPU generator seeded (seed + 0x5E6F7789),
    adamw.py:281-324, fed through the draws hook).  Per seed: the mean and
    variance of the dequantized m2 and the mean Adam preconditioner
    1/(sqrt(m2/bc2) + eps).  The two samples of 16 must agree: a two-sample
    t statistic below 4 for each statistic, and variances across seeds
    within a factor 6.5 of each other (F(15, 15) at 0.05 %).  The seeds are
    fixed, so the outcome is the same on every run."""
    import math

    from tests import synth as S
    shape, steps, seeds = (4096, 4096), 10, range(100, 116)
    n = shape[0] * shape[1]
    bc2 = 1 - 0.95 ** steps
    stats = {"philox": [], "reference": []}
    for mode in stats:
        for seed in seeds:
            p = torch.nn.Parameter(S.init_param(shape, 0, torch.float32, DEV))
            opt = ZIPSRAdamW4Bit([p], quant_rng_seed=seed)
            gen = (torch.Generator().manual_seed((seed + G.M2_OFFSET) % ((1 << 63) - 1))
                   if mode == "reference" else None)
            for t in range(1, steps + 1):
                p.grad = S.grad(shape, 0, t, 1e-3, torch.float32, DEV)
                if gen is not None:
                    if t == 1:
                        torch.rand((n // 128, 128), generator=gen)      # zero-state init
                    d2 = torch.rand((n // 128, 128), generator=gen).reshape(-1).to(DEV)
                    opt._draws_override = {id(p): (None, d2)}
                opt.step()
            st = opt.state[p]
            m2 = Q.dequantize(st["m2_code"], st["m2_quant_state"],
                              mode="dyn4_upd_sr_fp32read").double()
            pre = 1.0 / (torch.sqrt(m2 / bc2) + 1e-8)
            stats[mode].append([m2.mean().item(), m2.var().item(), pre.mean().item()])
    a, b = np.array(stats["philox"]), np.array(stats["reference"])
    for k, what in enumerate(("mean of m2", "variance of m2", "mean preconditioner")):
        va, vb = a[:, k].var(ddof=1), b[:, k].var(ddof=1)
        tstat = abs(a[:, k].mean() - b[:, k].mean()) / math.sqrt(va / len(a) + vb / len(b))
        assert tstat < 4.0, (what, tstat, a[:, k].mean(), b[:, k].mean())
        assert 1 / 6.5 < va / vb < 6.5, (what, va, vb)
