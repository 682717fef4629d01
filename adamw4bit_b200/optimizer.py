"""QuantizedAdamW and the paper recipes, stepping through the fused CUDA kernels.

Drop-in for nubank/adamw4bit's public optimizer API (src/adamw4bit/adamw.py):
the same constructor arguments and validation messages, the same per-parameter
state layout (packed 4-bit codes + ``QuantState`` block scales for eligible
tensors, FP32 ``m1``/``m2`` for the rest), the same ``state_dict`` format and
``set_m1_quant_scheme_for_parameters``.  ``step()`` gathers every parameter
with a gradient into one multi-tensor launch per (device, dtype, scheme)
combination of the CUDA library; there is no per-tensor Python arithmetic and
no CPU path.

Random streams.  With ``quant_rng="philox"`` (default) stochastic rounding
draws come from a counter-based Philox4x32-10 stream evaluated inside the
kernel, keyed by ``(quant_rng_seed + moment offset)`` and countered by
(element, step, parameter ordinal): stateless, independent of chunking or
sharding, and checkpointed by the step count alone.  With
``quant_rng="torch"`` the optimizer draws the uniforms with ``torch.rand`` from
per-moment generators in exactly the reference's order (adamw.py:281-324,
524-545, 675-683, 764-771) and feeds them to the kernel, reproducing the
reference's codes bit for bit on the same device.
"""

from __future__ import annotations

import math
from collections.abc import Iterable, Mapping

import numpy as np
import torch
from torch.optim.optimizer import Optimizer

from . import _native as N
from .quantization import (
    SCHEMES,
    QuantState,
    pack_4bit_codes,
    prepared,
    scheme_info,
)

_TORCHAO_MIN_QUANT_NUMEL = 4096  # adamw.py:19
_M1_OFFSET = 0x1A2B3C4D          # adamw.py:122-125
_M2_OFFSET = 0x5E6F7789
_MAX_SEED = (1 << 63) - 1


def _f32(x: float) -> float:
    """Round a Python float to float32 (how a scalar meets a float32 tensor)."""
    return float(np.float32(x))


def byte_range(t: torch.Tensor) -> tuple[str, int, int]:
    """(device, first byte, end byte) of a tensor's storage, without touching
    its values (the reference's tensor_byte_range, _moment_buffer.py:13-20)."""
    if t.is_contiguous():
        start = t.data_ptr()
        return str(t.device), start, start + t.numel() * t.element_size()
    storage = t.untyped_storage()
    start = storage.data_ptr()
    return str(t.device), start, start + storage.nbytes()


def _overlapping_pairs(regions: list[tuple]) -> list[tuple[tuple, tuple]]:
    """Pairs of overlapping (device, start, stop, owner, kind) regions, as
    ((owner, kind), (owner, kind)); empty regions never overlap."""
    out = []
    active: list[tuple] = []
    for r in sorted((r for r in regions if r[2] > r[1]), key=lambda r: (r[0], r[1])):
        active = [a for a in active if a[0] == r[0] and a[2] > r[1]]
        for a in active:
            out.append(((a[3], a[4]), (r[3], r[4])))
        active.append(r)
    return out


def _moment_buffers(st: dict) -> list[tuple[str, torch.Tensor]]:
    """The writable moment tensors of one parameter's state
    (the reference's moment_tensors, _moment_buffer.py:27-41)."""
    out = []
    for key in ("m1", "m2"):
        t = st.get(key)
        if torch.is_tensor(t) and t.numel():
            out.append((key, t))
        t = st.get(f"{key}_code")
        if torch.is_tensor(t) and t.numel():
            out.append((f"{key}_code", t))
        qs = st.get(f"{key}_quant_state")
        if isinstance(qs, QuantState) and torch.is_tensor(qs.absmax) and qs.absmax.numel():
            out.append((f"{key}_absmax", qs.absmax))
    return out


def _set_moment_buffer(st: dict, key: str, t: torch.Tensor) -> None:
    if key.endswith("_absmax"):
        st[f"{key[:2]}_quant_state"].absmax = t
    else:
        st[key] = t


class QuantizedAdamW(Optimizer):
    r"""AdamW with 4-bit (or FP32) moment storage, stepped on B200 by one fused kernel.

    Arguments follow ``adamw4bit.QuantizedAdamW`` (adamw.py:46-145).  The fused
    kernels implement the 4-bit schemes of :data:`adamw4bit_b200.quantization.SCHEMES`
    with 128-value blocks; ``"fp32"`` for both moments gives plain AdamW.
    Options whose only purpose is diagnostics or research ablations
    (``telemetry``, update clipping, update/preconditioner recording, 8-bit
    and lookahead-oracle schemes) raise ``NotImplementedError``.

    Extra argument:
        quant_rng: ``"philox"`` (default, in-kernel counter-based stream) or
            ``"torch"`` (reference-identical ``torch.Generator`` draws).
    """

    _VALID_SCHEMES = (
        "linear", "dynamic",
        "sdyn4", "sdyn4_sr", "nf4", "nf4_sr",
        "lin4", "lin4_sr", "lin4_upd_sr", "lin4_upd_sr_store_eden", "lin4_upd_sr_fp32read",
        "lin4_nz",
        "dyn4", "dyn4_sr", "dyn4_upd_sr", "dyn4_upd_sr_store_eden", "dyn4_upd_sr_fp32read",
        "dyn4_lookahead_sr", "dyn4_upd_sr_fp32read_nextbc", "dyn4_la_upd_sr",
        "dyn4_proxy_la_upd_sr", "dyn4_vproxy_la_upd_sr", "dyn4_nz",
        "fp32",
    )
    _UPDATE_SR_STORE_EDEN_SCHEMES = {"lin4_upd_sr_store_eden", "dyn4_upd_sr_store_eden"}
    _LOOKAHEAD_SCHEMES = {"dyn4_la_upd_sr", "dyn4_proxy_la_upd_sr", "dyn4_vproxy_la_upd_sr"}
    _QUANT_RNG_STATE_KEY = "_quant_rng_state"
    _QUANT_RNG_OFFSETS = {"m1": _M1_OFFSET, "m2": _M2_OFFSET}

    def __init__(self, params, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.95),
                 eps: float = 1e-8, weight_decay: float = 1e-1, block_size: int | None = None,
                 quant_scheme: str = "linear", use_eden_m2: bool = False,
                 m1_quant_scheme: str | None = None, m2_quant_scheme: str | None = None,
                 quant_rng_seed: int | None = None, telemetry=None,
                 update_sign_clip: float | None = None, update_norm_clip: float | None = None,
                 record_update_direction_every: int | None = None,
                 record_preconditioner_every: int | None = None,
                 record_preconditioner_steps=None, optimized: bool = False,
                 quant_rng: str = "philox"):
        # Validation mirrors adamw.py:148-208 (same conditions and messages).
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not 0.0 <= weight_decay:
            raise ValueError(f"Invalid weight_decay value: {weight_decay}")
        if quant_rng_seed is not None and (
            isinstance(quant_rng_seed, bool) or not isinstance(quant_rng_seed, int)
            or quant_rng_seed < 0
        ):
            raise ValueError("quant_rng_seed must be a non-negative integer or None, "
                             f"got {quant_rng_seed!r}")
        if update_sign_clip is not None and not update_sign_clip > 0.0:
            raise ValueError(f"update_sign_clip must be positive or None, got {update_sign_clip}")
        if update_norm_clip is not None and not update_norm_clip > 0.0:
            raise ValueError(f"update_norm_clip must be positive or None, got {update_norm_clip}")
        if update_sign_clip is not None and update_norm_clip is not None:
            raise ValueError("Set at most one of update_sign_clip / update_norm_clip "
                             "(they are alternative update-clip mechanisms).")
        if record_update_direction_every is not None and record_update_direction_every <= 0:
            raise ValueError("record_update_direction_every must be positive or None, "
                             f"got {record_update_direction_every}")
        if record_preconditioner_every is not None and record_preconditioner_every <= 0:
            raise ValueError("record_preconditioner_every must be positive or None, "
                             f"got {record_preconditioner_every}")
        if record_preconditioner_steps is not None:
            record_preconditioner_steps = tuple(sorted(set(int(s) for s in record_preconditioner_steps)))
            if any(s <= 0 for s in record_preconditioner_steps):
                raise ValueError("record_preconditioner_steps must contain positive optimizer steps")
        m1_scheme = m1_quant_scheme or quant_scheme
        m2_scheme = m2_quant_scheme or quant_scheme
        for name, s in (("quant_scheme", quant_scheme), ("m1_quant_scheme", m1_scheme),
                        ("m2_quant_scheme", m2_scheme)):
            if s not in self._VALID_SCHEMES:
                raise ValueError(f"{name} must be one of {self._VALID_SCHEMES}, got {s!r}")
        if use_eden_m2 and m2_scheme in {"lin4_sr", "dyn4_sr"}:
            raise ValueError("Vanilla stochastic-rounding m2 schemes should not be combined with use_eden_m2")
        if use_eden_m2 and m2_scheme in self._UPDATE_SR_STORE_EDEN_SCHEMES:
            raise ValueError("Do not set use_eden_m2 with *_upd_sr_store_eden; EDEN is built into the store path")
        if m2_scheme in self._LOOKAHEAD_SCHEMES:
            if m1_scheme not in {"fp32", "nf4"}:
                raise ValueError("lookahead update-SR currently supports m1_quant_scheme='fp32' or 'nf4'")
            if use_eden_m2:
                raise ValueError("lookahead update-SR should not be combined with use_eden_m2")
            if update_sign_clip is not None or update_norm_clip is not None:
                raise ValueError("lookahead update-SR should not be combined with update clipping")
        if quant_rng not in ("philox", "torch"):
            raise ValueError(f"quant_rng must be 'philox' or 'torch', got {quant_rng!r}")

        # Scope of the fused kernels.
        unsupported = [name for name, v in (
            ("telemetry", telemetry), ("update_sign_clip", update_sign_clip),
            ("update_norm_clip", update_norm_clip),
            ("record_update_direction_every", record_update_direction_every),
            ("record_preconditioner_every", record_preconditioner_every),
            ("record_preconditioner_steps", record_preconditioner_steps)) if v is not None]
        if unsupported:
            raise NotImplementedError(
                f"{', '.join(unsupported)}: diagnostics/clipping options are not implemented "
                "by the fused B200 step")
        if block_size is not None and block_size != 128:
            raise NotImplementedError("the fused B200 step uses 128-value quantization blocks")
        if m2_scheme == "fp32" and m1_scheme != "fp32":
            raise NotImplementedError("a 4-bit m1 next to an FP32 m2 is not implemented; use "
                                      "'fp32' for m1 too, or a 4-bit m2")
        for s, moment in ((m1_scheme, "m1"), (m2_scheme, "m2")):
            if s == "fp32":
                continue
            info = scheme_info(s)  # NotImplementedError for schemes outside the kernels
            if moment == "m1" and info.round_mode == N.SR_UPDATE:
                raise NotImplementedError("update-SR is an m2 scheme")

        self.telemetry = None
        self._m1_quant_scheme_overrides: dict[int, str] = {}
        self._quant_rng_seed = quant_rng_seed
        self._quant_rng = quant_rng
        self._quant_generators: dict[str, dict[str, torch.Generator]] = {"m1": {}, "m2": {}}
        self._pending_quant_rng_states: dict[str, dict[str, torch.Tensor]] = {"m1": {}, "m2": {}}
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                        block_size=block_size, quant_scheme=quant_scheme,
                        use_eden_m2=use_eden_m2, m1_quant_scheme=m1_scheme,
                        m2_quant_scheme=m2_scheme, update_sign_clip=update_sign_clip,
                        update_norm_clip=update_norm_clip,
                        record_update_direction_every=record_update_direction_every,
                        record_preconditioner_every=record_preconditioner_every,
                        record_preconditioner_steps=record_preconditioner_steps)
        super().__init__(params, defaults)
        self._optimized = optimized
        # Optional per-launch CUDA-event timing: when set to a list, every
        # fused launch appends (start_event, end_event, numel) recorded on the
        # launching stream right around the native call.
        self.launch_timings: list | None = None
        # Test hook: {id(param): (m1_uniforms, m2_uniforms)} device tensors fed
        # to the kernel instead of the configured stream (for parity with the
        # reference's own draws).
        self._draws_override: dict | None = None
        self._check_groups()

    def _check_groups(self) -> None:
        for group in self.param_groups:
            if group.get("block_size") not in (None, 128):
                raise NotImplementedError("the fused B200 step uses 128-value quantization blocks")

    def add_param_group(self, param_group) -> None:
        super().add_param_group(param_group)
        if hasattr(self, "_m1_quant_scheme_overrides"):
            self._check_groups()

    # ------------------------------------------------------------------ API
    def _m1_scheme_for(self, parameter: torch.Tensor, group_scheme: str) -> str:
        return self._m1_quant_scheme_overrides.get(id(parameter), group_scheme)

    def set_m1_quant_scheme_for_parameters(self, parameters: Iterable[torch.nn.Parameter],
                                           scheme: str) -> None:
        """Retarget future m1 writes for existing optimizer parameters (adamw.py:251-279)."""
        if scheme not in {"nf4", "nf4_sr"}:
            raise ValueError("runtime m1 retargeting supports only nf4 and nf4_sr")
        ids = {id(p) for group in self.param_groups for p in group["params"]}
        selected = list(parameters)
        if not selected:
            raise ValueError("runtime m1 retargeting requires parameters")
        if any(id(p) not in ids for p in selected):
            raise ValueError("runtime m1 retargeting received parameters outside optimizer")
        for p in selected:
            self._m1_quant_scheme_overrides[id(p)] = scheme

    @staticmethod
    def _eligible_for_quantized_state(p: torch.Tensor, block_size: int) -> bool:
        """TorchAO eligibility (adamw.py:807-811)."""
        n = p.numel()
        return n >= _TORCHAO_MIN_QUANT_NUMEL and n % block_size == 0

    @classmethod
    def _effective_scheme(cls, p: torch.Tensor, scheme: str, block_size: int) -> str:
        if scheme == "fp32" or cls._eligible_for_quantized_state(p, block_size):
            return scheme
        return "fp32"

    # ----------------------------------------------------------- RNG streams
    def _quant_generator(self, moment: str, device: torch.device) -> torch.Generator | None:
        """Reference-identical per-moment generators (adamw.py:281-324), used
        by quant_rng='torch'."""
        if self._quant_rng_seed is None:
            return None
        key = str(device)
        gens = self._quant_generators[moment]
        if key in gens:
            return gens[key]
        gen = torch.Generator(device=device)
        gen.manual_seed((self._quant_rng_seed + self._QUANT_RNG_OFFSETS[moment]) % _MAX_SEED)
        pending = self._pending_quant_rng_states[moment]
        state = pending.pop(key, None)
        if state is None:
            compatible = [k for k in pending if k.split(":", maxsplit=1)[0] == device.type]
            if len(compatible) == 1:
                state = pending.pop(compatible[0])
            elif pending:
                raise ValueError(f"Unable to restore quantization RNG state for {moment} on "
                                 f"{device}; saved devices={sorted(pending)}")
        if state is not None:
            gen.set_state(state.detach().cpu())
        gens[key] = gen
        return gen

    def _philox_keys(self) -> tuple[int, int]:
        """Keys of the m1 / m2 Philox streams for one step() call."""
        if self._quant_rng_seed is not None:
            return ((self._quant_rng_seed + _M1_OFFSET) % _MAX_SEED,
                    (self._quant_rng_seed + _M2_OFFSET) % _MAX_SEED)
        # No seed: one fresh key pair per step() call from the global torch
        # RNG (the reference's unseeded SR consumes the global generator).
        # The parameter ordinal is a Philox counter word, so the tensors of a
        # step share the keys and stay one launch.
        k1 = int(torch.randint(0, _MAX_SEED, (1,)).item())
        k2 = int(torch.randint(0, _MAX_SEED, (1,)).item())
        return k1, k2

    # ------------------------------------------------------------ checkpoint
    def state_dict(self):
        result = super().state_dict()
        result["state"] = {
            index: {k: vars(v).copy() if isinstance(v, QuantState) else v for k, v in st.items()}
            for index, st in result["state"].items()
        }
        if self._quant_rng_seed is None:
            return result
        if self._quant_rng == "philox":
            result[self._QUANT_RNG_STATE_KEY] = {
                "version": 2, "seed": self._quant_rng_seed, "stream": "philox4x32-10"}
            return result
        states = {m: {d: s.detach().cpu().clone() for d, s in self._pending_quant_rng_states[m].items()}
                  for m in self._QUANT_RNG_OFFSETS}
        for m, gens in self._quant_generators.items():
            states[m].update({d: g.get_state().detach().cpu().clone() for d, g in gens.items()})
        result[self._QUANT_RNG_STATE_KEY] = {"version": 1, "seed": self._quant_rng_seed,
                                             "states": states}
        return result

    def load_state_dict(self, state_dict):
        """Restore FP32 moments, uint8 codes and QuantStates on each parameter's
        device (adamw.py:364-470)."""
        rng_payload = state_dict.get(self._QUANT_RNG_STATE_KEY)
        optimizer_state = {k: v for k, v in state_dict.items() if k != self._QUANT_RNG_STATE_KEY}

        def capture_state(_optimizer, loaded_state):
            nonlocal optimizer_state
            optimizer_state = loaded_state

        def restore_moments(_optimizer):
            for group, saved_group in zip(self.param_groups, optimizer_state["param_groups"]):
                for parameter, saved_index in zip(group["params"], saved_group["params"]):
                    original = optimizer_state["state"].get(saved_index, {})
                    if not original:
                        continue
                    state = self.state[parameter]
                    for key in ("m1", "m2"):
                        if key in original:
                            state[key] = original[key].to(device=parameter.device, dtype=torch.float32)
                    for key in ("m1_quant_state", "m2_quant_state"):
                        if key in original:
                            value = original[key]
                            fields = dict(value) if isinstance(value, Mapping) else vars(value).copy()
                            fields["absmax"] = fields["absmax"].to(device=parameter.device,
                                                                   dtype=torch.float32)
                            state[key] = QuantState(**fields)
                    for key in ("m1_code", "m2_code"):
                        if key in original:
                            state[key] = original[key].to(device=parameter.device, dtype=torch.uint8)

        capture_hook = self.register_load_state_dict_pre_hook(capture_state)
        restore_hook = self.register_load_state_dict_post_hook(restore_moments, prepend=True)
        try:
            result = super().load_state_dict(optimizer_state)
        finally:
            capture_hook.remove()
            restore_hook.remove()
        self._quant_generators = {"m1": {}, "m2": {}}
        self._pending_quant_rng_states = {"m1": {}, "m2": {}}
        if rng_payload is not None:
            if not isinstance(rng_payload, Mapping):
                raise ValueError("Invalid quantization RNG checkpoint payload")
            version = rng_payload.get("version")
            if version not in (1, 2):
                raise ValueError(f"Unsupported quantization RNG checkpoint version: {version!r}")
            if self._quant_rng_seed is None:
                raise ValueError("Checkpoint contains separated quantization RNG "
                                 "state, but quant_rng_seed is disabled")
            saved_seed = rng_payload.get("seed")
            if saved_seed != self._quant_rng_seed:
                raise ValueError("Quantization RNG seed mismatch: "
                                 f"checkpoint={saved_seed!r}, configured={self._quant_rng_seed!r}")
            if version == 1 and self._quant_rng == "torch":
                saved_states = rng_payload.get("states")
                if not isinstance(saved_states, Mapping):
                    raise ValueError("Quantization RNG checkpoint states are missing")
                for moment in self._QUANT_RNG_OFFSETS:
                    moment_states = saved_states.get(moment, {})
                    if not isinstance(moment_states, Mapping):
                        raise ValueError(f"Invalid quantization RNG states for {moment}")
                    for device, st in moment_states.items():
                        if not isinstance(device, str) or not torch.is_tensor(st):
                            raise ValueError(f"Invalid quantization RNG state entry for {moment}")
                        self._pending_quant_rng_states[moment][device] = st.detach().cpu().clone()
            # version 2 (Philox) carries no generator state: the stream is a
            # function of (seed, step, element); a version-1 payload loaded in
            # philox mode continues with the Philox stream.
        return result

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure=None):  # type: ignore[override]
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        plan = _StepPlan(self)
        ordinal = 0
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is not None:
                    plan.add(group, p, ordinal)
                ordinal += 1
        plan.launch()
        return loss


class AdamW8bit(QuantizedAdamW):
    """The reference's compatibility name (adamw.py:865-866), kept so imports
    resolve.  8-bit schemes are not supported by this package: constructed
    with its 8-bit defaults it raises NotImplementedError, and it steps only
    when 4-bit schemes are given explicitly."""


class ZIPSRAdamW4Bit(QuantizedAdamW):
    """NF4 first moments and zero-inclusive Dyn4 preconditioner-space SR (adamw.py:869-879)."""

    def __init__(self, params, **kwargs):
        super().__init__(params, m1_quant_scheme="nf4", m2_quant_scheme="dyn4_upd_sr_fp32read",
                         use_eden_m2=False, **kwargs)


class ZEEDENAdamW4Bit(QuantizedAdamW):
    """NF4 first moments and zero-exclusive Dyn4 second moments with EDEN (adamw.py:882-892)."""

    def __init__(self, params, **kwargs):
        super().__init__(params, m1_quant_scheme="nf4", m2_quant_scheme="dyn4_nz",
                         use_eden_m2=True, **kwargs)


# ---------------------------------------------------------------------------
# one step: gather tensors, then one launch per (device, dtypes, schemes)
# ---------------------------------------------------------------------------

_FP32_MOMENT = None


def _kernel_scheme(mode: str):
    """The prepared scheme of a quantized moment, or the FP32-moment mode
    (an m1 kept as float32 values next to a 4-bit m2)."""
    global _FP32_MOMENT
    if mode != "fp32":
        return prepared(mode)
    if _FP32_MOMENT is None:
        s = N.Scheme()
        s.round_mode = N.FP32_MOMENT
        _FP32_MOMENT = s
    return _FP32_MOMENT


def hyper_scalars(lr: float, beta1: float, beta2: float, eps: float, weight_decay: float,
                  step: int, next_bias: bool) -> dict:
    """Per-step float32 scalars, derived in float64 as adamw.py:557-564, 684-691
    and 743 do before torch rounds them to float32 against float32 tensors."""
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    storage_bc = 1 - beta2 ** (step + 1) if next_bias else bc2
    return dict(w1=_f32(1 - beta1), w2=_f32(1 - beta2), decay=_f32(1 - lr * weight_decay),
                neg_step=_f32(-(lr / bc1)), sqrt_bc2=_f32(math.sqrt(bc2)), eps=_f32(eps),
                sr_bias=_f32(max(storage_bc, 1e-12)), step=step)


class _StepPlan:
    def __init__(self, opt: QuantizedAdamW):
        self.opt = opt
        self.qgroups: dict[tuple, list] = {}
        self.fgroups: dict[tuple, list] = {}
        self.keepalive: list = []
        self.keys: tuple[int, int] | None = None   # Philox keys of this step() call

    def _init_state(self, st: dict, p: torch.Tensor, m1: str, m2: str, eden: bool,
                    quantized: bool) -> None:
        """State initialisation (adamw.py:524-545): zero moments."""
        st["step"] = 0
        n = p.numel()
        if not quantized:
            st["m1"] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
            st["m2"] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
            return
        stream = N.stream_handle(p.device)
        for key, scheme, e in (("m1", m1, False), ("m2", m2, eden)):
            if scheme == "fp32":   # an FP32 m1 next to a 4-bit m2 (adamw.py:830-833)
                st[key] = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
                continue
            codes = torch.empty(n // 2, dtype=torch.uint8, device=p.device)
            scales = torch.empty(n // 128, dtype=torch.float32, device=p.device)
            N.check(N.lib().aw4_init_zero_state(prepared(scheme), int(e), N.ptr(codes), N.ptr(scales),
                                                n, p.device.index, stream), "aw4_init_zero_state")
            st[f"{key}_code"] = codes
            st[f"{key}_quant_state"] = QuantState(absmax=scales, shape=p.shape,
                                                  dtype=torch.float32, blocksize=128, packed=True)

    def add(self, group: dict, p: torch.Tensor, ordinal: int) -> None:
        opt = self.opt
        N.require_cuda(p, "QuantizedAdamW.step")
        g = p.grad
        if g.is_sparse:
            raise RuntimeError("QuantizedAdamW does not support sparse gradients")
        if p.dtype not in N.DTYPE_CODES or g.dtype not in N.DTYPE_CODES:
            raise NotImplementedError(f"parameter/gradient dtype {p.dtype}/{g.dtype} not supported")
        if not p.is_contiguous():
            raise NotImplementedError("the fused B200 step needs contiguous parameters")
        if g.device != p.device:
            raise RuntimeError("gradient and parameter are on different devices")
        g = g.contiguous()
        self.keepalive.append(g)
        beta1, beta2 = group["betas"]
        m1_req = opt._m1_scheme_for(p, group["m1_quant_scheme"])
        m2_req = group["m2_quant_scheme"]
        m1 = opt._effective_scheme(p, m1_req, 128)
        m2 = opt._effective_scheme(p, m2_req, 128)
        eden = bool(group["use_eden_m2"])
        quantized = m2 != "fp32"
        st = opt.state[p]
        first = "step" not in st
        if first:
            self._init_state(st, p, m1, m2, eden, quantized)
        st["step"] += 1
        t = st["step"]
        next_bias = quantized and SCHEMES[m2].next_bias
        hy = hyper_scalars(group["lr"], beta1, beta2, group["eps"], group["weight_decay"], t,
                           next_bias)
        pdt, gdt = N.DTYPE_CODES[p.dtype], N.DTYPE_CODES[g.dtype]
        if not quantized:
            self.fgroups.setdefault((p.device, pdt, gdt), []).append((p, g, st, hy))
            return
        m1_sr = m1 != "fp32" and SCHEMES[m1].round_mode != N.RTN
        m2_sr = SCHEMES[m2].round_mode != N.RTN
        d1 = d2 = None
        override = opt._draws_override
        if override is not None and id(p) in override:
            # test hook: explicit uniforms (e.g. the reference's CPU draws)
            d1, d2 = override[id(p)]
            keys = (0, 0)
        elif opt._quant_rng == "torch":
            d1, d2 = self._torch_draws(p, first, m1, m2, m1_sr, m2_sr)
            keys = (0, 0)
        elif m1_sr or m2_sr:
            if self.keys is None:
                self.keys = opt._philox_keys()
            keys = self.keys
        else:
            keys = (0, 0)
        # legacy one-code-per-byte state is repacked before the kernel reads it
        for key in ("m1", "m2") if m1 != "fp32" else ("m2",):
            qs = st[f"{key}_quant_state"]
            if not getattr(qs, "packed", False):
                codes = st[f"{key}_code"]
                if codes.numel() == p.numel():
                    st[f"{key}_code"] = pack_4bit_codes(codes.reshape(-1).contiguous())
                qs.packed = True
            self._check_state(st, key, p)
        if m1 == "fp32":
            t1 = st.get("m1")
            if (not torch.is_tensor(t1) or t1.dtype != torch.float32 or t1.numel() != p.numel()
                    or t1.device != p.device or not t1.is_contiguous()):
                raise RuntimeError("optimizer state m1 of an FP32 first moment must be a "
                                   f"contiguous float32 tensor of {p.numel()} values")
        self.qgroups.setdefault((p.device, pdt, gdt, m1, m2, eden), []).append(
            (p, g, st, hy, keys, ordinal, d1, d2))

    @staticmethod
    def _check_state(st: dict, key: str, p: torch.Tensor) -> None:
        codes, qs = st[f"{key}_code"], st[f"{key}_quant_state"]
        n = p.numel()
        if (codes.dtype != torch.uint8 or codes.numel() != n // 2 or codes.device != p.device
                or not codes.is_contiguous() or qs.absmax.numel() != n // 128
                or qs.absmax.dtype != torch.float32 or qs.absmax.device != p.device
                or not qs.absmax.is_contiguous() or qs.blocksize != 128):
            raise RuntimeError(f"optimizer state {key} of a parameter with {n} values does not have "
                               "the packed 4-bit layout (uint8[n/2] codes, float32[n/128] scales)")

    def _torch_draws(self, p, first, m1, m2, m1_sr, m2_sr):
        """Reference-order uniforms for quant_rng='torch' (adamw.py:524-545 init,
        675-683 m2 before the update, 764-771 m1 after it)."""
        opt = self.opt
        n = p.numel()
        g1 = opt._quant_generator("m1", p.device)
        g2 = opt._quant_generator("m2", p.device)

        def draw(gen):
            return torch.rand((n // 128, 128), device=p.device, dtype=torch.float32,
                              generator=gen).reshape(-1)

        if first:
            if m1_sr:
                draw(g1)
            if m2_sr:
                draw(g2)
        d2 = draw(g2) if m2_sr else None
        d1 = draw(g1) if m1_sr else None
        self.keepalive.extend([d1, d2])
        return d1, d2

    def resolve_aliases(self) -> None:
        """Byte-range overlap checks before the launches (the reference's GPU
        backend refuses overlapping param/grad/moment storage,
        _optimized.py:110-118 with _moment_buffer.py:13-41).  The fused launch
        updates every tensor of a step at once, so the reference eager path's
        results are kept where they can be:
          * a gradient overlapping its own parameter is copied first (eager
            reads the whole gradient before writing the parameter);
          * moment buffers overlapping any other buffer are copied first
            (eager decodes them, then stores the new moments in fresh storage,
            which also detaches aliases across parameters after a load);
        and a parameter overlapping another parameter or another parameter's
        gradient is refused: eager updates them one after the other, which
        one concurrent launch cannot reproduce."""
        items = [(p, g, st) for its in self.qgroups.values() for p, g, st, *_ in its]
        items += [(p, g, st) for its in self.fgroups.values() for p, g, st, *_ in its]
        regions = []   # (device, start, stop, owner, kind)
        moments = []
        for k, (p, g, st) in enumerate(items):
            regions.append((*byte_range(p), k, "param"))
            regions.append((*byte_range(g), k, "grad"))
            for key, t in _moment_buffers(st):
                moments.append((k, key, t))
                regions.append((*byte_range(t), k, key))
        conflicts = _overlapping_pairs(regions)
        if not conflicts:
            return
        copy_grad, copy_moment = set(), set()
        for (ka, kind_a), (kb, kind_b) in conflicts:
            kinds = {kind_a, kind_b}
            if kinds == {"grad"}:
                continue   # gradients are only read
            if ka == kb and kinds == {"param", "grad"}:
                copy_grad.add(ka)
            elif kinds <= {"param", "grad"}:
                raise RuntimeError(
                    "QuantizedAdamW.step: a parameter's storage overlaps another parameter or "
                    "its gradient; the fused step updates all tensors of a step concurrently "
                    "and cannot reproduce one-after-the-other updates of aliased parameters")
            else:
                for k, kind in ((ka, kind_a), (kb, kind_b)):
                    if kind not in ("param", "grad"):
                        copy_moment.add((k, kind))
        for k in copy_grad:
            self._replace_grad(items[k][0], items[k][1])
        for k, key, t in moments:
            if (k, key) in copy_moment:
                _set_moment_buffer(items[k][2], key, t.clone())

    def _replace_grad(self, p, g) -> None:
        snap = g.clone()
        self.keepalive.append(snap)
        for groups in (self.qgroups, self.fgroups):
            for its in groups.values():
                for i, it in enumerate(its):
                    if it[0] is p:
                        its[i] = (it[0], snap, *it[2:])

    def launch(self) -> None:
        self.resolve_aliases()
        for (dev, pdt, gdt, m1, m2, eden), items in self.qgroups.items():
            hypers, hindex, tensors = [], {}, []
            for p, g, st, hy, keys, ordinal, d1, d2 in items:
                hk = (tuple(hy.values()), keys)
                if hk not in hindex:
                    hindex[hk] = len(hypers)
                    hypers.append(N.Hyper(hy["w1"], hy["w2"], hy["decay"], hy["neg_step"],
                                          hy["sqrt_bc2"], hy["eps"], hy["sr_bias"], hy["step"],
                                          keys[0], keys[1]))
                tensors.append(N.QTensor(
                    N.ptr(p), N.ptr(g),
                    N.ptr(st["m1"]) if m1 == "fp32" else N.ptr(st["m1_code"]),
                    None if m1 == "fp32" else N.ptr(st["m1_quant_state"].absmax),
                    N.ptr(st["m2_code"]), N.ptr(st["m2_quant_state"].absmax), N.ptr(d1), N.ptr(d2),
                    p.numel(), 0, ordinal, hindex[hk]))
            tarr = (N.QTensor * len(tensors))(*tensors)
            harr = (N.Hyper * len(hypers))(*hypers)
            timing = self.opt.launch_timings
            if timing is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record(torch.cuda.current_stream(dev))
            N.check(N.lib().aw4_step_quantized(_kernel_scheme(m1), prepared(m2), int(eden), pdt,
                                               gdt, tarr,
                                               len(tensors), harr, len(hypers), 0, dev.index,
                                               N.stream_handle(dev)), "aw4_step_quantized")
            if timing is not None:
                ev1.record(torch.cuda.current_stream(dev))
                timing.append((ev0, ev1, sum(t.numel for t in tensors), pdt, gdt))
        for (dev, pdt, gdt), items in self.fgroups.items():
            hypers, hindex, tensors = [], {}, []
            for p, g, st, hy in items:
                hk = tuple(hy.values())
                if hk not in hindex:
                    hindex[hk] = len(hypers)
                    hypers.append(N.Hyper(hy["w1"], hy["w2"], hy["decay"], hy["neg_step"],
                                          hy["sqrt_bc2"], hy["eps"], hy["sr_bias"], hy["step"], 0, 0))
                tensors.append(N.FTensor(N.ptr(p), N.ptr(g), N.ptr(st["m1"]), N.ptr(st["m2"]),
                                         p.numel(),
                                         hindex[hk], 0))
            tarr = (N.FTensor * len(tensors))(*tensors)
            harr = (N.Hyper * len(hypers))(*hypers)
            N.check(N.lib().aw4_step_fp32_state(pdt, gdt, tarr, len(tensors), harr, len(hypers),
                                                dev.index, N.stream_handle(dev)),
                    "aw4_step_fp32_state")
        # The kernels run asynchronously on the current stream; temporaries
        # (contiguous grads, draws) are owned by the caching allocator, whose
        # stream-ordered reuse keeps them valid for the queued kernels.
        self.keepalive.clear()
