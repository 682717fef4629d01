"""ZeRO-1 sharding of the fused 4-bit AdamW step across the GPUs of one node.

Every rank keeps a full replica of the parameters (one flat buffer the
parameters are re-homed into) and of the already-reduced gradients, but
optimizer state -- packed 4-bit m1/m2 codes and block scales -- only for the
elements it owns.  A step is:

  1. the fused kernel updates the owned elements in place (one multi-tensor
     launch per gather round; a shard segment is an ``aw4_qtensor`` whose
     pointers start inside the tensor and whose ``elem_offset`` keeps the
     Philox counter equal to the unsharded one, so results do not depend on
     the number of ranks);
  2. NCCL all-gathers the updated parameters over NVLink, in place.

With ``master_weights=True`` the parameters are a BF16 model and each rank
keeps FP32 master weights for the elements it owns only: the fused kernel
updates the masters and writes bf16(master) into the model in the same pass,
and the all-gather moves the BF16 model (2 bytes per value instead of 4).

With ``gather="multicast"`` (BF16 model only) there is no separate
all-gather: the model lives in symmetric memory bound to an NVSwitch
multicast object, and the update kernel writes each new BF16 value once to
the multicast address (``multimem`` stores), which delivers it to every
rank's replica while the kernel runs.  A symmetric-memory barrier ends the
step.  Without multicast support the optimizer falls back to NCCL.

With ``grad_reduce="multicast"`` (ZeRO-2) the gradients are not reduced
beforehand: every rank's backward writes its local gradients into a buffer in
symmetric memory (the optimizer binds each ``p.grad`` to a view of it), and
the update kernel reads the sum over ranks of its own shard straight from
the NVSwitch (``multimem.ld_reduce``: the switch adds the ranks' values), times
``grad_scale`` (default 1/W, the mean).  The reduce-scatter is fused into the
update: no reduced gradient is ever written to memory.  Together with
``gather="multicast"`` one kernel per round does reduce-scatter, update and
all-gather; the two collectives load opposite NVLink directions (the
reduction reads from every GPU, the multicast stores write to every GPU).
Symmetric-memory barriers before the update (all gradients written) and
after it (all reads done before the next backward) bracket the step.

Ownership is block-cyclic over ``rounds`` rounds: round i covers the flat
range [i*W*c, (i+1)*W*c) and rank r owns its r-th c-element slice, so each
round's all-gather writes one contiguous range and can run while the kernel
updates the next round.  c is a multiple of 128, so shards never split a
quantization block.

The reference has no sharding (its optimizer is rank-local); this module is
the data-parallel layer the build adds around the fused step.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _native as N
from .optimizer import hyper_scalars
from .quantization import SCHEMES, prepared

_RECIPES = {"ze-eden": ("nf4", "dyn4_nz", True), "zip-sr": ("nf4", "dyn4_upd_sr_fp32read", False)}
_M1_OFFSET = 0x1A2B3C4D
_M2_OFFSET = 0x5E6F7789
_MAX_SEED = (1 << 63) - 1


def _multicast_buffer(n: int, dtype, dev, group):
    """A flat model buffer in symmetric memory with an NVSwitch multicast
    address, or (None, None, 0) when the platform offers no multicast."""
    try:
        import torch.distributed._symmetric_memory as symm_mem
        if symm_mem.get_backend(dev) is None:
            symm_mem.set_backend("CUDA")
        buf = symm_mem.empty(n, dtype=dtype, device=dev)
        handle = symm_mem.rendezvous(buf, group if group is not None else dist.group.WORLD)
        mc = int(handle.multicast_ptr)
    except (RuntimeError, AttributeError, TypeError):
        return None, None, 0
    if not mc:
        return None, None, 0
    return buf, handle, mc


def grad_layout(plan_starts: list[int], padded: int, small_sizes: list[int]):
    """Offsets of every gradient in the ZeRO-2 gradient buffer: the sharded
    tensors at their flat-model offsets (plan_starts, inside [0, padded)),
    the FP32-state tensors after them, each at an 8-value boundary (16 bytes,
    the multimem.ld_reduce width).  Returns (sharded offsets, small offsets,
    buffer length in values)."""
    offs, off = [], padded
    for n in small_sizes:
        offs.append(off)
        off += -(-n // 8) * 8
    return list(plan_starts), offs, off


class ShardPlan:
    """Block-cyclic ownership of a flat index space of tensors (pure host logic).

    ``chunk`` (c) is a multiple of 128; round i covers [i*W*c, (i+1)*W*c) and
    rank r owns [i*W*c + r*c, i*W*c + (r+1)*c) clipped to the real data.  For
    each round a rank's segments are (tensor index, start within the tensor,
    length, offset within the rank's state buffers)."""

    def __init__(self, sizes: list[int], world: int, rank: int, rounds: int):
        if any(n % 128 for n in sizes):
            raise ValueError("tensor sizes must be multiples of 128")
        self.sizes = list(sizes)
        self.world, self.rank = world, rank
        self.rounds = max(1, int(rounds))
        self.total = sum(sizes)
        c = math.ceil(self.total / (world * self.rounds) / 128) * 128
        self.chunk = max(c, 128)
        self.padded = self.chunk * world * self.rounds
        self.starts = []
        off = 0
        for n in sizes:
            self.starts.append(off)
            off += n
        self.owned = []
        for i in range(self.rounds):
            a = i * world * self.chunk + rank * self.chunk
            self.owned.append((a, max(a, min(a + self.chunk, self.total))))
        self.segments = []
        state_off = 0
        for a, b in self.owned:
            segs = []
            for ti, (n, s0) in enumerate(zip(self.sizes, self.starts)):
                lo, hi = max(a, s0), min(b, s0 + n)
                if lo < hi:
                    segs.append((ti, lo - s0, hi - lo, state_off + (lo - a)))
            self.segments.append(segs)
            state_off += self.chunk

    def owned_numel(self) -> int:
        return sum(b - a for a, b in self.owned)

    def state_numel(self) -> int:
        return self.chunk * self.rounds


class ZeRO1AdamW4Bit:
    """Sharded fused step over a model's parameters.  Tensors eligible for
    4-bit state (numel a multiple of 128 and at least 4096, adamw.py:807-811)
    are sharded; the others keep FP32 moments replicated on every rank, which
    all run the same FP32-state update (bit-identical replicas, no exchange).

    Args:
        params: CUDA parameters of one dtype, all on this rank's device.
        recipe: ``"ze-eden"`` or ``"zip-sr"``.
        process_group: NCCL group (default: the world).
        rounds: number of pipelined gather rounds.
        quant_rng_seed: Philox seed for SR recipes.
        reserve_sms: SMs the update grid leaves to the concurrent all-gather.
        master_weights: the parameters are a BF16 model; keep FP32 master
            weights for the owned elements and gather the BF16 model.
        gather: ``"nccl"`` (all-gather on a side stream) or ``"multicast"``
            (the update kernel writes every replica through NVSwitch; needs
            ``master_weights`` and a process group of 2+ ranks).
        grad_reduce: ``"local"`` (``p.grad`` holds already-reduced gradients)
            or ``"multicast"`` (ZeRO-2: each ``p.grad`` is bound to this rank's
            unreduced gradients in symmetric memory and the update reads the
            sum over ranks through NVSwitch; needs 2+ ranks and multicast).
        grad_dtype: dtype of the bound gradients (``grad_reduce="multicast"``;
            default BF16).
        grad_scale: factor on the summed gradients (default 1/W).
    """

    def __init__(self, params, *, recipe: str = "ze-eden", lr: float = 1e-3,
                 betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.1,
                 process_group=None, rounds: int = 4, quant_rng_seed: int = 0,
                 reserve_sms: int = 16, master_weights: bool = False,
                 gather: str = "nccl", grad_reduce: str = "local", grad_dtype=torch.bfloat16,
                 grad_scale: float | None = None):
        self.all_params = [p for p in params]
        if not self.all_params:
            raise ValueError("ZeRO1AdamW4Bit needs parameters")
        eligible = [p.numel() >= 4096 and p.numel() % 128 == 0 for p in self.all_params]
        self.qindex = [i for i, e in enumerate(eligible) if e]        # sharded, 4-bit state
        self.sindex = [i for i, e in enumerate(eligible) if not e]    # replicated, FP32 state
        self.params = [self.all_params[i] for i in self.qindex]
        if not self.params:
            raise ValueError("ZeRO1AdamW4Bit needs at least one tensor of >= 4096 values")
        self.m1, self.m2, self.eden = _RECIPES[recipe]
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        dev = self.params[0].device
        dtype = self.params[0].dtype
        for p in self.all_params:
            N.require_cuda(p, "ZeRO1AdamW4Bit")
            if p.device != dev or p.dtype != dtype:
                raise ValueError("all parameters must share one device and dtype")
        if master_weights and dtype != torch.bfloat16:
            raise ValueError("master_weights=True needs BF16 parameters (the model copy)")
        self.master_weights = master_weights
        self.device, self.dtype = dev, dtype
        self.quant_rng_seed = quant_rng_seed
        self.keys = ((quant_rng_seed + _M1_OFFSET) % _MAX_SEED,
                     (quant_rng_seed + _M2_OFFSET) % _MAX_SEED)
        W = self.world
        plan = ShardPlan([p.numel() for p in self.params], W, self.rank, rounds)
        self.plan = plan
        self.chunk, self.padded, self.total = plan.chunk, plan.padded, plan.total
        if gather not in ("nccl", "multicast"):
            raise ValueError(f"unknown gather mode {gather!r}")
        if gather == "multicast" and not master_weights:
            raise ValueError('gather="multicast" needs master_weights=True (a BF16 model)')
        self.symm = None
        self.mc_base = 0
        flat = None
        if gather == "multicast" and W > 1:
            flat, self.symm, self.mc_base = _multicast_buffer(plan.padded, dtype, dev,
                                                              self.group)
        self.gather_mode = "multicast" if self.mc_base else "nccl"
        # re-home parameters into one flat buffer (zero padding at the end)
        if flat is None:
            flat = torch.zeros(plan.padded, dtype=dtype, device=dev)
        else:
            flat.zero_()
        for p, off in zip(self.params, plan.starts):
            n = p.numel()
            flat[off:off + n].copy_(p.detach().reshape(-1))
            p.data = flat[off:off + n].view(p.shape)
        self.flat = flat
        self.owned = plan.owned
        # state for the owned elements, one flat buffer per kind
        n_own = plan.state_numel()
        self.master = None
        if master_weights:
            # FP32 masters of the owned elements, laid out like the state buffers
            self.master = torch.zeros(n_own, dtype=torch.float32, device=dev)
            for segs in plan.segments:
                for ti, s, n, so in segs:
                    src = self.params[ti].detach().reshape(-1)[s:s + n]
                    self.master[so:so + n].copy_(src.float())
        self.m1_codes = torch.empty(n_own // 2, dtype=torch.uint8, device=dev)
        self.m2_codes = torch.empty(n_own // 2, dtype=torch.uint8, device=dev)
        self.m1_scales = torch.empty(n_own // 128, dtype=torch.float32, device=dev)
        self.m2_scales = torch.empty(n_own // 128, dtype=torch.float32, device=dev)
        stream = N.stream_handle(dev)
        for codes, scales, scheme, e in ((self.m1_codes, self.m1_scales, self.m1, False),
                                         (self.m2_codes, self.m2_scales, self.m2, self.eden)):
            N.check(N.lib().aw4_init_zero_state(prepared(scheme), int(e), N.ptr(codes),
                                                N.ptr(scales), n_own, dev.index, stream),
                    "aw4_init_zero_state")
        # FP32-state tensors, replicated: moments (and masters) per tensor
        self.small = []
        for i in self.sindex:
            p = self.all_params[i]
            entry = {"m1": torch.zeros(p.numel(), dtype=torch.float32, device=dev),
                     "m2": torch.zeros(p.numel(), dtype=torch.float32, device=dev)}
            if master_weights:
                entry["master"] = p.detach().reshape(-1).float().clone()
            self.small.append(entry)
        self.step_count = 0
        self.segments = plan.segments
        if grad_reduce not in ("local", "multicast"):
            raise ValueError(f"unknown grad_reduce mode {grad_reduce!r}")
        self.grad_reduce = grad_reduce
        self.grad_scale = float(1.0 / W if grad_scale is None else grad_scale)
        self.gsymm = None
        if grad_reduce == "multicast":
            self._bind_gradients(grad_dtype)
        nccl = W > 1 and self.gather_mode == "nccl"
        self.gather_stream = torch.cuda.Stream(dev) if nccl else None
        # With a concurrent all-gather, leave `reserve_sms` SMs free so NCCL's
        # kernels can run beside the persistent update grid (4 CTAs per SM).
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.max_ctas = max(1, (sms - reserve_sms) * 4) if nccl else 0
        if self.symm is not None:
            self.symm.barrier(channel=0)   # every replica holds the initial model
        self.launch_timings: list | None = None

    def _bind_gradients(self, grad_dtype) -> None:
        """ZeRO-2: one symmetric-memory gradient buffer with a multicast
        address, laid out by grad_layout; every p.grad becomes a view of it."""
        if self.world < 2:
            raise ValueError('grad_reduce="multicast" needs a process group of 2+ ranks')
        if grad_dtype not in (torch.float32, torch.bfloat16, torch.float16):
            raise ValueError(f"unsupported gradient dtype {grad_dtype}")
        _, offs, off = grad_layout(self.plan.starts, self.padded,
                                   [self.all_params[i].numel() for i in self.sindex])
        gbuf, self.gsymm, self.gmc = _multicast_buffer(off, grad_dtype, self.device, self.group)
        if not self.gmc:
            raise RuntimeError('grad_reduce="multicast" needs NVSwitch multicast (symmetric '
                               'memory with a multicast address), which this platform lacks')
        gbuf.zero_()
        self.gbuf, self.small_goff = gbuf, offs
        self.small_gtotal = off - self.padded
        self.small_g = torch.zeros(max(self.small_gtotal, 8), dtype=torch.float32,
                                   device=self.device)
        views = {}
        for ti, i in enumerate(self.qindex):
            s0 = self.plan.starts[ti]
            views[i] = gbuf[s0:s0 + self.all_params[i].numel()]
        for k, i in enumerate(self.sindex):
            views[i] = gbuf[offs[k]:offs[k] + self.all_params[i].numel()]
        for i, p in enumerate(self.all_params):
            if p.dtype != grad_dtype and hasattr(p, "grad_dtype"):
                p.grad_dtype = None   # a gradient dtype other than the parameter's
            p.grad = views[i].view(p.shape)
        self.grad_ptrs = [p.grad.data_ptr() for p in self.all_params]
        self.gsymm.barrier(channel=0)

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Zero the gradients.  With grad_reduce="multicast" the bound
        buffer is zeroed in place (the bindings stay); otherwise the grads are
        dropped (or zeroed when set_to_none is False)."""
        if self.grad_reduce == "multicast":
            self.gbuf.zero_()
            return
        for p in self.all_params:
            if p.grad is None:
                continue
            if set_to_none:
                p.grad = None
            else:
                p.grad.zero_()

    @torch.no_grad()
    def step(self, round_begin=None, round_end=None) -> None:
        """One optimizer step: per gather round, one fused update launch over
        this rank's owned segments (then that round's gather), then the
        FP32-state tensors.

        round_begin(r) / round_end(r), when given, are called on the host just
        before and just after round r's update launch is enqueued on the
        current stream.  A caller that streams gradients in and the model out
        per round orders its copies there: round r reads the gradients of
        ``segments[r]`` and writes this rank's values ``owned[r]`` of the flat
        model, so the next round's gradients can upload while round r
        updates, and round r's values can download while round r+1 updates."""
        if self.grad_reduce == "multicast" and any(
                p.grad is None or p.grad.data_ptr() != ptr
                for p, ptr in zip(self.all_params, self.grad_ptrs)):
            # a p.grad replaced or set to None (e.g. by module.zero_grad())
            # no longer lands in the buffer the kernel reads
            raise RuntimeError('grad_reduce="multicast": a parameter\'s .grad is no longer '
                               'the bound view; zero gradients with the optimizer\'s '
                               'zero_grad(), not by setting them to None')
        self.step_count += 1
        t = self.step_count
        hy = hyper_scalars(self.lr, self.betas[0], self.betas[1], self.eps, self.wd, t,
                           SCHEMES[self.m2].next_bias)
        harr = (N.Hyper * 1)(N.Hyper(hy["w1"], hy["w2"], hy["decay"], hy["neg_step"],
                                     hy["sqrt_bc2"], hy["eps"], hy["sr_bias"], t, self.keys[0],
                                     self.keys[1], self.grad_scale))
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        pdt = N.DTYPE_CODES[torch.float32 if self.master_weights else self.dtype]
        esz_p = self.flat.element_size()
        reduce_mc = self.grad_reduce == "multicast"
        grads = [p.grad for p in self.params]
        if any(g is None for g in grads) or any(self.all_params[i].grad is None
                                                for i in self.sindex):
            raise RuntimeError("ZeRO1AdamW4Bit.step needs a gradient for every parameter")
        gdt = N.DTYPE_CODES[self.gbuf.dtype if reduce_mc else grads[0].dtype]
        W = self.world
        if reduce_mc:
            self.gsymm.barrier(channel=0)   # every rank's gradients are written
        for r, segs in enumerate(self.segments):
            descs = []
            for ti, s, n, so in segs:
                p, g = self.params[ti], grads[ti]
                model = p.data_ptr() + s * esz_p
                multicast = 0
                if self.gather_mode == "multicast":   # every rank's replica, via NVSwitch
                    model = self.mc_base + (self.plan.starts[ti] + s) * esz_p
                    multicast = 1
                if self.master_weights:   # update the FP32 master, write the BF16 model
                    target, copy = self.master.data_ptr() + so * 4, model
                else:
                    target, copy = model, None
                if reduce_mc:   # the sum over ranks, read through NVSwitch
                    gptr = self.gmc + (self.plan.starts[ti] + s) * self.gbuf.element_size()
                else:
                    gptr = g.data_ptr() + s * g.element_size()
                descs.append(N.QTensor(
                    target, gptr,
                    self.m1_codes.data_ptr() + so // 2, self.m1_scales.data_ptr() + (so // 128) * 4,
                    self.m2_codes.data_ptr() + so // 2, self.m2_scales.data_ptr() + (so // 128) * 4,
                    # Philox ordinal: the position among all parameters, as in
                    # the single-GPU optimizer, so SR draws do not depend on sharding
                    None, None, n, s, self.qindex[ti], 0, copy, multicast, int(reduce_mc)))
            if round_begin is not None:
                round_begin(r)
            if descs:
                arr = (N.QTensor * len(descs))(*descs)
                if self.launch_timings is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(cur)
                N.check(N.lib().aw4_step_quantized(prepared(self.m1), prepared(self.m2),
                                                   int(self.eden), pdt, gdt, arr, len(descs), harr,
                                                   1, self.max_ctas, dev.index, cur.cuda_stream),
                        "aw4_step_quantized")
                if self.launch_timings is not None:
                    e1.record(cur)
                    self.launch_timings.append((e0, e1, sum(d.numel for d in descs), pdt, gdt))
            if round_end is not None:
                round_end(r)
            if W > 1 and self.gather_mode == "nccl":
                base = r * W * self.chunk
                region = self.flat[base:base + W * self.chunk]
                mine = region[self.rank * self.chunk:(self.rank + 1) * self.chunk]
                self.gather_stream.wait_stream(cur)
                with torch.cuda.stream(self.gather_stream):
                    dist.all_gather_into_tensor(region, mine, group=self.group)
        self._step_small(harr, cur)
        if W > 1 and self.gather_mode == "nccl":
            cur.wait_stream(self.gather_stream)
        if self.symm is not None:
            # every rank's multimem stores are in every replica once all
            # ranks' update kernels have completed
            self.symm.barrier(channel=0)
        elif reduce_mc:
            # no rank's next backward overwrites gradients another rank is
            # still reading
            self.gsymm.barrier(channel=0)

    def _step_small(self, harr, cur) -> None:
        """The FP32-state update of the small tensors, identical on every rank
        (adamw.py:807-817); with master weights the BF16 model copy follows."""
        if not self.small:
            return
        dev = self.device
        pdt = N.DTYPE_CODES[torch.float32 if self.master_weights else self.dtype]
        reduce_mc = self.grad_reduce == "multicast"
        if reduce_mc:
            # the small tensors' summed gradients, read through NVSwitch into FP32
            esz = self.gbuf.element_size()
            N.check(N.lib().aw4_reduce_multicast(self.gmc + self.padded * esz,
                                                 N.DTYPE_CODES[self.gbuf.dtype],
                                                 self.small_gtotal, self.grad_scale,
                                                 N.ptr(self.small_g), dev.index, cur.cuda_stream),
                    "aw4_reduce_multicast")
            gdt = N.DTYPE_CODES[torch.float32]
        else:
            gdt = N.DTYPE_CODES[self.all_params[self.sindex[0]].grad.dtype]
        descs, keep = [], []
        for k, (i, st) in enumerate(zip(self.sindex, self.small)):
            p = self.all_params[i]
            target = st["master"] if self.master_weights else p
            if reduce_mc:
                o = self.small_goff[k] - self.padded
                g = self.small_g[o:o + p.numel()]
            else:
                g = p.grad.contiguous()
            keep.append(g)
            descs.append(N.FTensor(target.data_ptr(), g.data_ptr(),
                                   st["m1"].data_ptr(), st["m2"].data_ptr(), p.numel(), 0, 0))
        arr = (N.FTensor * len(descs))(*descs)
        N.check(N.lib().aw4_step_fp32_state(pdt, gdt, arr, len(descs), harr, 1, dev.index,
                                            cur.cuda_stream), "aw4_step_fp32_state")
        if self.master_weights:
            for i, st in zip(self.sindex, self.small):
                self.all_params[i].data.copy_(st["master"].view(self.all_params[i].shape))

    def owned_numel(self) -> int:
        return self.plan.owned_numel()

    # ------------------------------------------------------------ checkpoints
    _SHARD_KIND = "zero1-shard"

    def _shard_buffers(self) -> dict:
        bufs = {"m1_codes": self.m1_codes, "m1_scales": self.m1_scales,
                "m2_codes": self.m2_codes, "m2_scales": self.m2_scales}
        if self.master is not None:
            bufs["master"] = self.master
        return bufs

    def _config(self) -> dict:
        return {"world": self.world, "rounds": self.plan.rounds,
                "sizes": list(self.plan.sizes), "small": [self.all_params[i].numel()
                                                          for i in self.sindex],
                "recipe": (self.m1, self.m2, self.eden), "master_weights": self.master_weights}

    def state_dict(self, consolidated: bool = False) -> dict:
        """Optimizer state for a checkpoint.

        Default: this rank's shard (its packed codes, block scales and FP32
        masters, as device tensors) plus the sharding it depends on; every rank
        saves its own and loads it back into the same layout.

        ``consolidated=True`` (a collective: every rank must call it): the
        whole state in the per-parameter layout of the single-GPU
        optimizer's ``state_dict`` (``m1_code`` / ``m1_quant_state`` / ...,
        adamw.py:330-336), on the CPU, so a ZeRO run can resume on one GPU and
        the other way round; FP32 masters, if any, under ``"master_weights"``.
        """
        group = {"lr": self.lr, "betas": self.betas, "eps": self.eps,
                 "weight_decay": self.wd}
        if not consolidated:
            return {"kind": self._SHARD_KIND, "rank": self.rank, "step": self.step_count,
                    "config": self._config(), "param_group": group,
                    "buffers": {k: v.detach().clone() for k, v in self._shard_buffers().items()},
                    "small": [{k: v.detach().clone() for k, v in st.items()}
                              for st in self.small]}
        glob = self._gather_state()
        from .optimizer import ZEEDENAdamW4Bit, ZIPSRAdamW4Bit
        cls = ZEEDENAdamW4Bit if self.eden else ZIPSRAdamW4Bit
        template = cls([torch.nn.Parameter(torch.zeros(4096))],
                       quant_rng_seed=None if self.eden else self.quant_rng_seed)
        defaults = {k: v for k, v in template.param_groups[0].items() if k != "params"}
        defaults.update(group)
        state, masters = {}, {}
        for ti, (p, s0) in enumerate(zip(self.params, self.plan.starts)):
            i = self.qindex[ti]
            n = p.numel()
            entry = {"step": self.step_count}
            for m in ("m1", "m2"):
                entry[f"{m}_code"] = glob[f"{m}_codes"][s0 // 2:(s0 + n) // 2].clone()
                entry[f"{m}_quant_state"] = {
                    "absmax": glob[f"{m}_scales"][s0 // 128:(s0 + n) // 128].clone(),
                    "shape": p.shape, "dtype": torch.float32, "blocksize": 128, "packed": True}
            state[i] = entry
            if "master" in glob:
                masters[i] = glob["master"][s0:s0 + n].clone().view(p.shape)
        for i, st in zip(self.sindex, self.small):
            shape = self.all_params[i].shape
            state[i] = {"step": self.step_count, "m1": st["m1"].view(shape).cpu().clone(),
                        "m2": st["m2"].view(shape).cpu().clone()}
            if "master" in st:
                masters[i] = st["master"].view(shape).cpu().clone()
        result = {"state": state,
                  "param_groups": [{**defaults, "params": list(range(len(self.all_params)))}]}
        if not self.eden:
            result["_quant_rng_state"] = {"version": 2, "seed": self.quant_rng_seed,
                                          "stream": "philox4x32-10"}
        if masters:
            result["master_weights"] = masters
        return result

    def _gather_state(self) -> dict:
        """All ranks' state buffers in the global flat element order, on the CPU."""
        W, R, c = self.world, self.plan.rounds, self.chunk
        units = {"m1_codes": c // 2, "m2_codes": c // 2, "m1_scales": c // 128,
                 "m2_scales": c // 128, "master": c}
        totals = {"m1_codes": self.total // 2, "m2_codes": self.total // 2,
                  "m1_scales": self.total // 128, "m2_scales": self.total // 128,
                  "master": self.total}
        out = {}
        for name, buf in self._shard_buffers().items():
            if W > 1:
                g = torch.empty((W,) + tuple(buf.shape), dtype=buf.dtype, device=buf.device)
                dist.all_gather_into_tensor(g.view(-1), buf.contiguous(), group=self.group)
            else:
                g = buf.unsqueeze(0)
            # rank k's round-r chunk is global chunk r*W + k
            g = g.view(W, R, units[name]).transpose(0, 1).reshape(-1)
            out[name] = g[:totals[name]].cpu()
        return out

    def load_state_dict(self, state_dict: dict) -> None:
        """Restore a shard dict saved by this rank (same sharding) or a
        consolidated / single-GPU optimizer state dict (re-sharded here)."""
        if state_dict.get("kind") == self._SHARD_KIND:
            if state_dict["config"] != self._config() or state_dict["rank"] != self.rank:
                raise ValueError("shard checkpoint was saved with a different sharding "
                                 "(world, rounds, sizes, recipe) or rank")
            for k, v in self._shard_buffers().items():
                v.copy_(state_dict["buffers"][k])
            for st, saved in zip(self.small, state_dict["small"]):
                for k, v in st.items():
                    v.copy_(saved[k])
            self.step_count = int(state_dict["step"])
            g = state_dict["param_group"]
            self.lr, self.betas, self.eps, self.wd = g["lr"], tuple(g["betas"]), g["eps"], g["weight_decay"]
            return
        states = state_dict["state"]
        groups = state_dict["param_groups"]
        order = [i for grp in groups for i in grp["params"]]
        if len(order) != len(self.all_params):
            raise ValueError("state dict holds a different number of parameters")
        masters = state_dict.get("master_weights", {})
        if self.master_weights and not masters:
            raise ValueError("master_weights=True needs FP32 masters in the state dict")
        steps = set()
        for i, st_local in zip(self.sindex, self.small):
            index = order[i]
            st = states.get(index)
            if not st or "m1" not in st:
                raise ValueError(f"parameter {i}: no FP32 moments in the state dict")
            steps.add(int(st["step"]))
            st_local["m1"].copy_(st["m1"].reshape(-1))
            st_local["m2"].copy_(st["m2"].reshape(-1))
            if "master" in st_local:
                st_local["master"].copy_(masters[index].reshape(-1).to(torch.float32))
        for ti, i in enumerate(self.qindex):
            index = order[i]
            st = states.get(index)
            if not st or "m1_code" not in st:
                raise ValueError(f"parameter {i}: no packed 4-bit state in the state dict")
            steps.add(int(st["step"]))
            for segs in self.segments:
                for sti, s0, n, so in segs:
                    if sti != ti:
                        continue
                    for m in ("m1", "m2"):
                        codes = getattr(self, f"{m}_codes")
                        scales = getattr(self, f"{m}_scales")
                        qs = st[f"{m}_quant_state"]
                        absmax = qs["absmax"] if isinstance(qs, dict) else qs.absmax
                        codes[so // 2:(so + n) // 2].copy_(
                            st[f"{m}_code"].reshape(-1)[s0 // 2:(s0 + n) // 2])
                        scales[so // 128:(so + n) // 128].copy_(
                            absmax.reshape(-1)[s0 // 128:(s0 + n) // 128])
                    if self.master is not None:
                        self.master[so:so + n].copy_(
                            masters[index].reshape(-1)[s0:s0 + n].to(torch.float32))
        if len(steps) != 1:
            raise ValueError("parameters are at different steps")
        self.step_count = steps.pop()
        g = groups[0]
        self.lr, self.betas, self.eps, self.wd = g["lr"], tuple(g["betas"]), g["eps"], g["weight_decay"]
