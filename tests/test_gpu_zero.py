"""ZeRO-1 sharded step on 2 GPUs (NCCL): every rank's parameters after the
sharded update + all-gather are bit-identical to the unsharded single-GPU
step.  Runs as two spawned child processes; skipped with fewer than 2 GPUs.
NVLS is off for the test (NCCL_NVLS_ENABLE=0)."""

from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# two tensors below the 4-bit threshold (FP32 moments, replicated on every rank)
SHAPES = [(4096,), (128, 96), (768,), (1024, 64), (8192,), (100, 3), (384, 256)]


def _make(dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    params = [(torch.randn(s, generator=g) * 0.02).to(dev) for s in SHAPES]
    grads = [[(torch.randn(s, generator=g) * 1e-3).to(dev, torch.bfloat16) for s in SHAPES]
             for _ in range(3)]
    return params, grads


def _same_state(cons: dict, ref: dict) -> bool:
    """Bitwise equality of a consolidated ZeRO state and a single-GPU one."""
    for i, want in ref["state"].items():
        got = cons["state"][i]
        for key, val in want.items():
            if key == "step":
                if int(got[key]) != int(val):
                    return False
            elif key.endswith("_quant_state"):
                if not torch.equal(got[key]["absmax"].view(torch.int32),
                                   val["absmax"].cpu().view(torch.int32)):
                    return False
            elif not torch.equal(got[key].cpu().reshape(-1).view(torch.uint8),
                                 val.cpu().reshape(-1).view(torch.uint8)):
                return False
    return True


def _worker(rank, world, port, recipe, rounds, q, master=False, gather="nccl"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from adamw4bit_b200 import ZEEDENAdamW4Bit, ZIPSRAdamW4Bit
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        vals, grads = _make(dev)
        if master:   # a BF16 model; FP32 masters start from its values
            vals = [v.to(torch.bfloat16).float() for v in vals]
        model_dtype = torch.bfloat16 if master else torch.float32
        params = [torch.nn.Parameter(v.clone().to(model_dtype)) for v in vals]
        for p in params:
            p.grad_dtype = None
        opt = ZeRO1AdamW4Bit(params, recipe=recipe, rounds=rounds, quant_rng_seed=9,
                             master_weights=master, gather=gather)
        if opt.gather_mode != gather:
            q.put((rank, True, "skip: no NVSwitch multicast on this platform"))
            return
        for step_grads in grads:
            for p, g in zip(params, step_grads):
                p.grad = g
            opt.step()
        torch.cuda.synchronize()
        dist.barrier()
        # single-GPU reference on this rank's device: the same kernels, unsharded
        ref = [torch.nn.Parameter(v.clone()) for v in vals]
        for p in ref:
            p.grad_dtype = None
        cls = ZEEDENAdamW4Bit if recipe == "ze-eden" else ZIPSRAdamW4Bit
        single = cls(ref, quant_rng_seed=9)
        for step_grads in grads:
            for p, g in zip(ref, step_grads):
                p.grad = g
            single.step()
        torch.cuda.synchronize()
        # the consolidated checkpoint gathers every rank's shard: it must hold
        # the single-GPU optimizer's codes and scales bit for bit
        cons = opt.state_dict(consolidated=True)
        sref = single.state_dict()
        if not _same_state(cons, sref):
            raise AssertionError("consolidated state differs from the single-GPU state")
        if master:
            # the gathered BF16 model is bf16(the unsharded FP32 params) everywhere,
            # and this rank's FP32 masters equal the unsharded params it owns
            ok = all(torch.equal(a.detach().view(torch.int16),
                                 b.detach().to(torch.bfloat16).view(torch.int16))
                     for a, b in zip(params, ref))
            for segs in opt.plan.segments:
                for ti, s0, n, so in segs:
                    want = ref[opt.qindex[ti]].detach().reshape(-1)[s0:s0 + n]
                    ok = ok and torch.equal(opt.master[so:so + n].view(torch.int32),
                                            want.view(torch.int32))
        else:
            ok = all(torch.equal(a.detach().view(torch.int32), b.detach().view(torch.int32))
                     for a, b in zip(params, ref))
        # both ranks finish all device work (multicast stores included) before
        # either exits
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, ok, None))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            torch.cuda.synchronize()
            dist.destroy_process_group()


@pytest.mark.parametrize("recipe,rounds,master,gather", [
    ("ze-eden", 1, False, "nccl"), ("ze-eden", 3, False, "nccl"), ("zip-sr", 2, False, "nccl"),
    ("ze-eden", 2, True, "nccl"), ("ze-eden", 2, True, "multicast"),
    ("zip-sr", 3, True, "multicast")])
def test_zero1_two_gpus_matches_single_gpu_bit_exact(recipe, rounds, master, gather):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() % 400) + (7 if master else 0) + (13 if gather != "nccl" else 0)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, recipe, rounds, q, master, gather))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    if all(msg and str(msg).startswith("skip") for _, _, msg in results):
        pytest.skip(results[0][2])
    assert all(ok for _, ok, _ in results), results


def test_zero1_master_weights_on_one_gpu_matches_fp32_step():
    """master_weights without a process group (one rank): FP32 masters equal
    the FP32 optimizer's params and the BF16 model equals their bf16 cast."""
    from adamw4bit_b200 import ZEEDENAdamW4Bit
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    dev = torch.device("cuda", 0)
    vals, grads = _make(dev, seed=3)
    vals = [v.to(torch.bfloat16).float() for v in vals]
    model = [torch.nn.Parameter(v.to(torch.bfloat16)) for v in vals]
    fp32 = [torch.nn.Parameter(v.clone()) for v in vals]
    for p in fp32:
        p.grad_dtype = None
    opt = ZeRO1AdamW4Bit(model, recipe="ze-eden", rounds=2, master_weights=True)
    ref = ZEEDENAdamW4Bit(fp32)
    for step_grads in grads:
        for a, b, g in zip(model, fp32, step_grads):
            a.grad = g
            b.grad = g
        opt.step()
        ref.step()
    torch.cuda.synchronize()
    for a, b in zip(model, fp32):
        assert torch.equal(a.detach().view(torch.int16), b.detach().to(torch.bfloat16).view(torch.int16))
    for segs in opt.plan.segments:
        for ti, s0, n, so in segs:
            want = fp32[opt.qindex[ti]].detach().reshape(-1)[s0:s0 + n]
            assert torch.equal(opt.master[so:so + n].view(torch.int32), want.view(torch.int32))


def test_round_hooks_stream_gradients_in_and_model_out_per_round():
    """step(round_begin, round_end) on one rank: the hooks run once per round
    in order, and gradients uploaded from pinned host memory round by round
    on a copy stream, with each round's BF16 values downloaded on another
    stream while the next round updates, give the plain step's model and
    masters bit for bit."""
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    dev = torch.device("cuda", 0)
    vals, grads = _make(dev, seed=5)

    def build():
        model = [torch.nn.Parameter(v.to(torch.bfloat16)) for v in vals]
        return model, ZeRO1AdamW4Bit(model, recipe="zip-sr", rounds=3, master_weights=True,
                                     quant_rng_seed=9)

    plain_model, plain = build()
    _run(plain, plain_model, grads)
    model, opt = build()
    for p, g in zip(model, grads[0]):
        p.grad = torch.zeros_like(g)
    cur = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    R = len(opt.segments)
    calls, host_models = [], []
    for step_grads in grads:
        host = [g.cpu().pin_memory() for g in step_grads]
        for i in opt.sindex:
            opt.all_params[i].grad.copy_(host[i], non_blocking=True)
        uploaded = []
        with torch.cuda.stream(up):
            up.wait_stream(cur)
            for r in range(R):
                for ti, s, n, _ in opt.segments[r]:
                    q = opt.qindex[ti]
                    opt.params[ti].grad.reshape(-1)[s:s + n].copy_(
                        host[q].reshape(-1)[s:s + n], non_blocking=True)
                e = torch.cuda.Event()
                e.record(up)
                uploaded.append(e)
        out = [torch.empty(b - a, dtype=torch.bfloat16, pin_memory=True) for a, b in opt.owned]

        def begin(r):
            calls.append(("begin", r))
            cur.wait_event(uploaded[r])

        def end(r):
            calls.append(("end", r))
            done = torch.cuda.Event()
            done.record(cur)
            down.wait_event(done)
            a, b = opt.owned[r]
            with torch.cuda.stream(down):
                out[r].copy_(opt.flat[a:b], non_blocking=True)

        opt.step(round_begin=begin, round_end=end)
        cur.wait_stream(down)
        host_models.append(out)
    torch.cuda.synchronize()
    assert calls == [(k, r) for _ in grads for r in range(R) for k in ("begin", "end")]
    for a, b in zip(model, plain_model):
        assert torch.equal(a.detach().view(torch.int16), b.detach().view(torch.int16))
    assert torch.equal(opt.master.view(torch.int32), plain.master.view(torch.int32))
    for (a, b), h in zip(opt.owned, host_models[-1]):
        assert torch.equal(h.view(torch.int16), plain.flat[a:b].cpu().view(torch.int16))


def _run(opt, params, grads):
    for step_grads in grads:
        for p, g in zip(params, step_grads):
            p.grad = g
        opt.step()


def test_zero1_consolidated_state_dict_resumes_on_the_single_gpu_optimizer():
    """ZeRO-1 (one rank) -> consolidated state dict -> the single-GPU
    optimizer continues bit-identically, and the other way round."""
    from adamw4bit_b200 import ZEEDENAdamW4Bit
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    dev = torch.device("cuda", 0)
    vals, grads = _make(dev, seed=5)
    za = [torch.nn.Parameter(v.clone()) for v in vals]
    sa = [torch.nn.Parameter(v.clone()) for v in vals]
    for p in za + sa:
        p.grad_dtype = None
    zopt = ZeRO1AdamW4Bit(za, recipe="ze-eden", rounds=3)
    sopt = ZEEDENAdamW4Bit(sa)
    _run(zopt, za, grads[:2])
    _run(sopt, sa, grads[:2])
    sd = zopt.state_dict(consolidated=True)
    ref = sopt.state_dict()
    assert _same_state(sd, ref)
    # ZeRO -> single GPU
    sb = [torch.nn.Parameter(p.detach().clone()) for p in za]
    for p in sb:
        p.grad_dtype = None
    sopt_b = ZEEDENAdamW4Bit(sb)
    sopt_b.load_state_dict(sd)
    # single GPU -> ZeRO
    zb = [torch.nn.Parameter(p.detach().clone()) for p in sa]
    for p in zb:
        p.grad_dtype = None
    zopt_b = ZeRO1AdamW4Bit(zb, recipe="ze-eden", rounds=2)
    zopt_b.load_state_dict(ref)
    _run(zopt, za, grads[2:])
    _run(sopt_b, sb, grads[2:])
    _run(zopt_b, zb, grads[2:])
    torch.cuda.synchronize()
    for a, b, c in zip(za, sb, zb):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
        assert torch.equal(a.view(torch.int32), c.view(torch.int32))


def test_zero1_shard_state_dict_round_trip_with_master_weights():
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    dev = torch.device("cuda", 0)
    vals, grads = _make(dev, seed=6)
    a = [torch.nn.Parameter(v.to(torch.bfloat16)) for v in vals]
    b = [torch.nn.Parameter(v.to(torch.bfloat16)) for v in vals]
    opt_a = ZeRO1AdamW4Bit(a, recipe="zip-sr", rounds=2, master_weights=True, quant_rng_seed=4)
    _run(opt_a, a, grads[:2])
    sd = opt_a.state_dict()
    opt_b = ZeRO1AdamW4Bit(b, recipe="zip-sr", rounds=2, master_weights=True, quant_rng_seed=4)
    for pa, pb in zip(a, b):
        pb.data.copy_(pa.data)
    opt_b.load_state_dict(sd)
    _run(opt_a, a, grads[2:])
    _run(opt_b, b, grads[2:])
    torch.cuda.synchronize()
    for pa, pb in zip(a, b):
        assert torch.equal(pa.view(torch.int16), pb.view(torch.int16))
    assert torch.equal(opt_a.master.view(torch.int32), opt_b.master.view(torch.int32))
    bad = ZeRO1AdamW4Bit([torch.nn.Parameter(v.to(torch.bfloat16)) for v in vals], recipe="zip-sr",
                         rounds=3, master_weights=True, quant_rng_seed=4)
    with pytest.raises(ValueError, match="different sharding"):
        bad.load_state_dict(sd)


def _rank_grad(shape, step, index, rank):
    """Rank `rank`'s BF16 gradient of parameter `index` at `step`: integers
    in [-63, 63] times 2^-12.  The sum over 2 ranks has at most 7 significant
    bits, so it is exact in BF16 whatever order or rounding the switch uses."""
    g = torch.Generator().manual_seed(100_000 * step + 100 * index + rank)
    k = torch.randint(-63, 64, shape, generator=g).float()
    return (k * 2.0 ** -12).to(torch.bfloat16)


def _worker_reduce(rank, world, port, recipe, master, gather, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    from adamw4bit_b200 import ZEEDENAdamW4Bit, ZIPSRAdamW4Bit
    from adamw4bit_b200.zero import ZeRO1AdamW4Bit
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        vals, _ = _make(dev)
        if master:
            vals = [v.to(torch.bfloat16).float() for v in vals]
        model_dtype = torch.bfloat16 if master else torch.float32
        params = [torch.nn.Parameter(v.clone().to(model_dtype)) for v in vals]
        for p in params:
            p.grad_dtype = None
        try:
            opt = ZeRO1AdamW4Bit(params, recipe=recipe, rounds=2, quant_rng_seed=9,
                                 master_weights=master, gather=gather, grad_reduce="multicast")
        except RuntimeError as e:
            if "multicast" in str(e):
                q.put((rank, True, "skip: no NVSwitch multicast on this platform"))
                return
            raise
        if opt.gather_mode != gather:
            q.put((rank, True, "skip: no NVSwitch multicast on this platform"))
            return
        steps = 3
        for t in range(steps):
            opt.zero_grad()
            for i, p in enumerate(params):
                p.grad.copy_(_rank_grad(p.shape, t, i, rank).to(dev))
            opt.step()
        torch.cuda.synchronize()
        dist.barrier()
        # single-GPU reference fed the FP32 gradients the fused read defines:
        # f32(bf16(sum over ranks)) / world
        ref = [torch.nn.Parameter(v.clone()) for v in vals]
        cls = ZEEDENAdamW4Bit if recipe == "ze-eden" else ZIPSRAdamW4Bit
        single = cls(ref, quant_rng_seed=9)
        for t in range(steps):
            for i, p in enumerate(ref):
                s = sum(_rank_grad(p.shape, t, i, r).float() for r in range(world))
                p.grad = (s.to(torch.bfloat16).float() * (1.0 / world)).to(dev)
            single.step()
        torch.cuda.synchronize()
        cons = opt.state_dict(consolidated=True)
        ok = _same_state(cons, single.state_dict())
        why = None if ok else "state"
        if master:
            okp = all(torch.equal(a.detach().view(torch.int16),
                                  b.detach().to(torch.bfloat16).view(torch.int16))
                      for a, b in zip(params, ref))
        else:
            okp = all(torch.equal(a.detach().view(torch.int32), b.detach().view(torch.int32))
                      for a, b in zip(params, ref))
        if not okp:
            why = (why or "") + " params"
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, ok and okp, why))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            torch.cuda.synchronize()
            dist.destroy_process_group()


@pytest.mark.parametrize("recipe,master,gather", [
    ("ze-eden", True, "multicast"), ("zip-sr", True, "multicast"), ("ze-eden", False, "nccl")])
def test_zero2_fused_reduce_two_gpus_matches_single_gpu(recipe, master, gather):
    """ZeRO-2: the update kernel reads the gradient sum over ranks through
    NVSwitch (multimem.ld_reduce) and must equal the single-GPU step fed
    sum / W, bit for bit (the sums are exact in BF16)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30100 + (os.getpid() % 400) + (7 if master else 0) + (3 if recipe == "zip-sr" else 0)
    procs = [ctx.Process(target=_worker_reduce, args=(r, 2, port, recipe, master, gather, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    if all(msg and str(msg).startswith("skip") for _, _, msg in results):
        pytest.skip(results[0][2])
    assert all(ok for _, ok, _ in results), results
