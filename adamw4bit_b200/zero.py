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
    """Sharded fused step over quantized parameters (every tensor eligible:
    numel a multiple of 128 and at least 4096).

    Args:
        params: CUDA parameters of one dtype, all on this rank's device.
        recipe: ``"ze-eden"`` or ``"zip-sr"``.
        process_group: NCCL group (default: the world).
        rounds: number of pipelined gather rounds.
        quant_rng_seed: Philox seed for SR recipes.
        reserve_sms: SMs the update grid leaves to the concurrent all-gather.
        master_weights: the parameters are a BF16 model; keep FP32 master
            weights for the owned elements and gather the BF16 model.
    """

    def __init__(self, params, *, recipe: str = "ze-eden", lr: float = 1e-3,
                 betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.1,
                 process_group=None, rounds: int = 4, quant_rng_seed: int = 0,
                 reserve_sms: int = 16, master_weights: bool = False):
        self.params = [p for p in params]
        if not self.params:
            raise ValueError("ZeRO1AdamW4Bit needs parameters")
        self.m1, self.m2, self.eden = _RECIPES[recipe]
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        dev = self.params[0].device
        dtype = self.params[0].dtype
        for p in self.params:
            N.require_cuda(p, "ZeRO1AdamW4Bit")
            if p.device != dev or p.dtype != dtype:
                raise ValueError("all parameters must share one device and dtype")
            if p.numel() % 128 or p.numel() < 4096:
                raise NotImplementedError("ZeRO1AdamW4Bit shards quantized tensors only "
                                          "(numel >= 4096, multiple of 128)")
        if master_weights and dtype != torch.bfloat16:
            raise ValueError("master_weights=True needs BF16 parameters (the model copy)")
        self.master_weights = master_weights
        self.device, self.dtype = dev, dtype
        self.keys = ((quant_rng_seed + _M1_OFFSET) % _MAX_SEED,
                     (quant_rng_seed + _M2_OFFSET) % _MAX_SEED)
        W = self.world
        plan = ShardPlan([p.numel() for p in self.params], W, self.rank, rounds)
        self.plan = plan
        self.chunk, self.padded, self.total = plan.chunk, plan.padded, plan.total
        # re-home parameters into one flat buffer (zero padding at the end)
        flat = torch.zeros(plan.padded, dtype=dtype, device=dev)
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
        self.step_count = 0
        self.segments = plan.segments
        self.gather_stream = torch.cuda.Stream(dev) if W > 1 else None
        # With a concurrent all-gather, leave `reserve_sms` SMs free so NCCL's
        # kernels can run beside the persistent update grid (4 CTAs per SM).
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.max_ctas = max(1, (sms - reserve_sms) * 4) if W > 1 else 0
        self.launch_timings: list | None = None

    @torch.no_grad()
    def step(self) -> None:
        self.step_count += 1
        t = self.step_count
        hy = hyper_scalars(self.lr, self.betas[0], self.betas[1], self.eps, self.wd, t,
                           SCHEMES[self.m2].next_bias)
        harr = (N.Hyper * 1)(N.Hyper(hy["w1"], hy["w2"], hy["decay"], hy["neg_step"],
                                     hy["sqrt_bc2"], hy["eps"], hy["sr_bias"], t, self.keys[0],
                                     self.keys[1]))
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        pdt = N.DTYPE_CODES[torch.float32 if self.master_weights else self.dtype]
        esz_p = self.flat.element_size()
        grads = [p.grad for p in self.params]
        if any(g is None for g in grads):
            raise RuntimeError("ZeRO1AdamW4Bit.step needs a gradient for every parameter")
        gdt = N.DTYPE_CODES[grads[0].dtype]
        W = self.world
        for r, segs in enumerate(self.segments):
            descs = []
            for ti, s, n, so in segs:
                p, g = self.params[ti], grads[ti]
                model = p.data_ptr() + s * esz_p
                if self.master_weights:   # update the FP32 master, write the BF16 model
                    target, copy = self.master.data_ptr() + so * 4, model
                else:
                    target, copy = model, None
                descs.append(N.QTensor(
                    target, g.data_ptr() + s * g.element_size(),
                    self.m1_codes.data_ptr() + so // 2, self.m1_scales.data_ptr() + (so // 128) * 4,
                    self.m2_codes.data_ptr() + so // 2, self.m2_scales.data_ptr() + (so // 128) * 4,
                    None, None, n, s, ti, 0, copy))
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
            if W > 1:
                base = r * W * self.chunk
                region = self.flat[base:base + W * self.chunk]
                mine = region[self.rank * self.chunk:(self.rank + 1) * self.chunk]
                self.gather_stream.wait_stream(cur)
                with torch.cuda.stream(self.gather_stream):
                    dist.all_gather_into_tensor(region, mine, group=self.group)
        if W > 1:
            cur.wait_stream(self.gather_stream)

    def owned_numel(self) -> int:
        return self.plan.owned_numel()
