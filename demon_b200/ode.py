"""Fused per-slot ODE step: host side of ``demon_ode_step`` / ``demon_ode_prepare``.

One :class:`OdeTick` collects the slots that advance this tick, resolves each
slot's integration branch exactly as the reference's ``StreamPipeline._tick_pt``
does (acestep/engine/stream.py:1125-1194: fast Euler path vs x0-blend path,
SDE curve / bare SDE, final step, x0-target gates), stages every per-frame
curve and the slot descriptors in one pinned buffer, copies it to the device
with a single async H2D copy and launches one kernel for all slots.

Curves follow ``ode_steps.normalize_curve`` (acestep/engine/ode_steps.py:36-64):
a Python scalar, a 0-d tensor or a [T] / [1, T] / [1, T, 1] tensor; they are
converted to the pipeline dtype (bf16) like the reference's ``.to(dtype=...)``
at each use site (stream.py:590-602, 1106-1116).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import torch

from . import _native as nat

Curve = "float | torch.Tensor | None"


def _bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def _as_curve(v, T: int):
    """None | (scalar float) | fp32 CPU tensor [T] (bf16-rounded)."""
    if v is None:
        return None
    if isinstance(v, (int, float, bool)):
        return float(_bf16_round(torch.tensor([float(v)]))[0])
    t = torch.as_tensor(v).detach().to("cpu", torch.float32).reshape(-1)
    if t.numel() == 1:
        return float(_bf16_round(t)[0])
    if t.numel() != T:
        raise ValueError(f"curve has {t.numel()} values, expected 1 or T={T}")
    return _bf16_round(t)


def _norm_curve(v) -> torch.Tensor:
    """normalize_curve (acestep/engine/ode_steps.py:36-64) on the host: a Python scalar -> fp32
    [1, 1, 1]; a tensor keeps its dtype, reshaped to [1, 1, 1] / [1, T, 1] / [B, T, 1]."""
    if isinstance(v, (int, float, bool)):
        return torch.tensor([[[float(v)]]], dtype=torch.float32)
    t = torch.as_tensor(v).detach().to("cpu")
    if t.ndim == 0:
        return t.reshape(1, 1, 1).to(torch.float32)
    if t.ndim == 1:
        return t.unsqueeze(0).unsqueeze(-1)
    if t.ndim == 2:
        return t.unsqueeze(-1)
    if t.ndim == 3:
        return t
    raise ValueError(f"normalize_curve: expected scalar / 0-d / 1-d / 2-d / 3-d, got {t.ndim}-d")


@dataclass
class LatentMask:
    """Latent-noise mask of a slot (acestep/engine/masking.py:9-71): mask [T]
    (1 = generate), original latents and fixed noise [T, 64] on the device,
    and the step strengths (step_strength_fn evaluated on the host)."""
    mask: torch.Tensor            # fp32 [T] on device
    original: torch.Tensor        # bf16 [T, 64]
    noise: torch.Tensor           # bf16 [T, 64]
    strength: float = 1.0
    strength_next: float = 1.0


@dataclass
class SlotStep:
    """Everything the fused kernel needs to advance one slot by one step.

    Field names follow the reference's SlotRequest / _Slot (stream.py:31-198).
    Latents are bf16 [T, 64] CUDA tensors; ``xt`` is updated in place.
    """
    xt: torch.Tensor
    t_curr: float
    t_next: float
    step_idx: int
    total_steps: int
    pos: Sequence                                  # [(v [T,64], weight curve | None)]
    has_cfg: bool = False
    rcfg_mode: Optional[str] = None
    neg: Optional[Sequence] = None                 # negative forward outputs this tick
    neg_cached: Optional[torch.Tensor] = None
    initial_noise: Optional[torch.Tensor] = None
    momentum: Optional[torch.Tensor] = None        # running average buffer [T, 64]
    momentum_fresh: bool = True                    # running average still 0
    neg_cache_out: Optional[torch.Tensor] = None   # where RCFG-initialize caches v_neg
    guidance: object = None
    apg_momentum: object = -0.75
    cfg_rescale: object = None
    velocity_scale: object = None
    sde_denoise_curve: object = None
    ode_noise_curve: object = None
    source: Optional[torch.Tensor] = None
    x0_target: Optional[torch.Tensor] = None
    x0_target_curve: object = None
    x0_target_gate: float = 0.0
    x0_target_strength: object = 0.0
    mask: Optional[LatentMask] = None
    complex_extra: bool = False                    # extra conds / temporal weight / step range
    infer_method: str = "ode"
    noise: Optional[torch.Tensor] = None           # explicit step noise (else in-kernel counter-based noise)
    dec_out: Optional[torch.Tensor] = None         # next tick's decoder input row
    dcw: Optional[tuple] = None                    # active DCW corrector: (mode, scaler, high_scaler)
    seed: int = 0
    keep: list = field(default_factory=list)


def resolve_flags(s: SlotStep) -> tuple[int, dict]:
    """Branch selection of stream.py:1131-1194 plus the APG source of
    stream.py:1086-1104.  Returns (DEMON_ODE_* flags, resolved curves)."""
    T = s.xt.shape[0]
    f = 0
    vs = _as_curve(s.velocity_scale, T)
    sdc = _as_curve(s.sde_denoise_curve, T)
    onc = _as_curve(s.ode_noise_curve, T)
    strength = _as_curve(s.x0_target_strength, T)
    sde_curve_active = sdc is not None and s.source is not None
    use_sde = sde_curve_active or s.infer_method == "sde"
    if strength is None:
        strength_active = False
    elif isinstance(strength, float):
        strength_active = strength != 0.0
    else:
        strength_active = bool(strength.abs().gt(0).any())
    scalar_x0 = (s.x0_target is not None and strength_active and s.x0_target_curve is None
                 and s.step_idx >= s.total_steps // 2 and s.t_curr > 0)
    has_x0_curve = s.x0_target is not None and s.x0_target_curve is not None
    has_complex = s.mask is not None or s.complex_extra or has_x0_curve or s.has_cfg
    needs_x0 = has_complex or scalar_x0 or use_sde or s.t_next <= 0
    cur = {"vs": vs, "sdc": sdc, "onc": onc, "x0c": None, "x0mul": 1.0}

    neg_src = None
    if s.has_cfg:
        if s.rcfg_mode == "self":
            neg_src = "self"
        elif s.neg:
            neg_src = "forward"
        elif s.neg_cached is not None:
            neg_src = "cache"
    cur["neg_src"] = neg_src
    if neg_src is not None:
        f |= nat.ODE_CFG
        if s.momentum_fresh:
            f |= nat.ODE_MOM_INIT
        if s.cfg_rescale is not None:
            f |= nat.ODE_RESCALE
        if neg_src == "forward" and s.rcfg_mode == "initialize":
            f |= nat.ODE_CACHE_NEG
    if vs is not None:
        f |= nat.ODE_VS
    if onc is not None:
        f |= nat.ODE_ONC
    if s.mask is not None:
        f |= nat.ODE_MASK
    if needs_x0:
        f |= nat.ODE_X0PATH
        if has_x0_curve:
            progress = s.step_idx / max(s.total_steps - 1, 1)
            gate = float(s.x0_target_gate)
            bg = max(0.0, progress - gate) / max(1.0 - gate, 1e-6)
            if bg > 0:
                f |= nat.ODE_X0_TARGET
                cur["x0c"] = _as_curve(s.x0_target_curve, T)
                cur["x0mul"] = bg
        elif scalar_x0:
            f |= nat.ODE_X0_TARGET
            cur["x0c"] = strength
        if s.t_next <= 0:
            f |= nat.ODE_FINAL
        if sde_curve_active:
            f |= nat.ODE_SDE_CURVE
        elif use_sde:
            f |= nat.ODE_SDE_BARE
    if s.dec_out is not None:
        f |= nat.ODE_DEC_OUT
        if s.mask is not None:
            f |= nat.ODE_DEC_MASK
    return f, cur


class OdeTick:
    """Stages one tick's slots and launches the fused kernel.

    Two pinned staging buffers alternate between ticks; before a buffer is
    rewritten, the event recorded after its last H2D copy is synchronised, so
    the host never overwrites bytes an in-flight copy still reads.
    """

    SLOT_BYTES = ctypes.sizeof(nat.DemonOdeSlot)

    def __init__(self, device, T: int, max_slots: int = 64, D: int = 64):
        if D != 64:
            raise ValueError("latent width must be 64")
        self.device = torch.device(device)
        self.T, self.D, self.max_slots = T, D, max_slots
        # per slot: descriptor + up to 18 curves of T floats (weights, step curves, DCW bands)
        self.capacity = max_slots * (self.SLOT_BYTES + 18 * (4 * T + 16) + 256)
        self._host = [torch.empty(self.capacity, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self._dev = [torch.empty(self.capacity, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self._events = [None, None]
        self._buf = 0
        self.reset()

    def reset(self) -> None:
        self.slots: list[SlotStep] = []

    def add(self, s: SlotStep) -> None:
        if len(self.slots) >= self.max_slots:
            raise ValueError("too many slots for this OdeTick")
        if s.xt.shape != (self.T, self.D) or s.xt.dtype != torch.bfloat16 or not s.xt.is_contiguous():
            raise ValueError(f"xt must be a contiguous bf16 [{self.T}, {self.D}] tensor")
        # the kernel moves latents in 16-byte vectors: every latent must start 16-byte aligned
        lat = [s.xt, s.neg_cached, s.initial_noise, s.momentum, s.neg_cache_out, s.source, s.x0_target, s.noise,
               s.dec_out] + [v for v, _ in s.pos] + [v for v, _ in (s.neg or [])]
        if s.mask is not None:
            lat += [s.mask.original, s.mask.noise]
        for t in lat:
            if t is not None and (t.data_ptr() % 16 or not t.is_contiguous()):
                raise ValueError("slot latents must be contiguous and 16-byte aligned")
        self.slots.append(s)

    # ------------------------------------------------------------------
    def _stage(self):
        b = self._buf
        if self._events[b] is not None:
            self._events[b].synchronize()
        host, dev = self._host[b], self._dev[b]
        base_dev = dev.data_ptr()
        T = self.T
        n = len(self.slots)
        table = (nat.DemonOdeSlot * n).from_buffer(host.numpy())
        off = [(self.SLOT_BYTES * n + 255) // 256 * 256]
        fview = host.numpy()

        def put_curve(c, expand=False):
            if c is None:
                return 0
            if isinstance(c, float):
                if not expand:
                    return 0
                c = torch.full((T,), c, dtype=torch.float32)
            o = off[0]
            arr = c.numpy().view("u1")
            fview[o:o + arr.size] = arr
            off[0] = o + (arr.size + 15) // 16 * 16
            return base_dev + o

        for i, s in enumerate(self.slots):
            flags, cur = resolve_flags(s)
            d = table[i]
            ctypes.memset(ctypes.addressof(d), 0, self.SLOT_BYTES)
            d.xt = nat.ptr(s.xt)
            d.n_pos = len(s.pos)
            for j, (v, w) in enumerate(s.pos):
                d.v_pos[j] = nat.ptr(v)
                d.w_pos[j] = put_curve(_as_curve(w, T), expand=True) if (w is not None and len(s.pos) > 1) else 0
            src = cur["neg_src"]
            if src == "self":
                d.n_neg, d.v_neg[0] = 1, nat.ptr(s.initial_noise)
            elif src == "cache":
                d.n_neg, d.v_neg[0] = 1, nat.ptr(s.neg_cached)
            elif src == "forward":
                d.n_neg = len(s.neg)
                for j, (v, w) in enumerate(s.neg):
                    d.v_neg[j] = nat.ptr(v)
                    d.w_neg[j] = put_curve(_as_curve(w, T), expand=True) if (w is not None and len(s.neg) > 1) else 0
            if flags & nat.ODE_CACHE_NEG:
                d.neg_cache = nat.ptr(s.neg_cache_out)
            if flags & nat.ODE_CFG:
                d.momentum = nat.ptr(s.momentum)
                g = _as_curve(s.guidance, T)
                d.guidance, d.guidance_s = put_curve(g), (g if isinstance(g, float) else 0.0)
                m = _as_curve(s.apg_momentum if s.apg_momentum is not None else -0.75, T)
                d.apg_mom, d.apg_mom_s = put_curve(m), (m if isinstance(m, float) else 0.0)
                if flags & nat.ODE_RESCALE:
                    r = _as_curve(s.cfg_rescale, T)
                    d.rescale, d.rescale_s = put_curve(r), (r if isinstance(r, float) else 0.0)
            for name, fld in (("vs", "vscale"), ("sdc", "sdc"), ("onc", "onc")):
                c = cur[name]
                if c is not None:
                    setattr(d, fld, put_curve(c))
                    setattr(d, fld + "_s", c if isinstance(c, float) else 0.0)
            if flags & nat.ODE_X0_TARGET:
                c = cur["x0c"]
                d.x0_coef, d.x0_coef_s, d.x0_coef_mul = put_curve(c), (c if isinstance(c, float) else 0.0), cur["x0mul"]
                d.x0_target = nat.ptr(s.x0_target)
            if s.mask is not None:
                d.mask = nat.ptr(s.mask.mask)
                d.mask_orig, d.mask_noise = nat.ptr(s.mask.original), nat.ptr(s.mask.noise)
                d.mask_s, d.mask_s_next = float(s.mask.strength), float(s.mask.strength_next)
            if flags & nat.ODE_SDE_CURVE:
                d.source = nat.ptr(s.source)
            d.noise = nat.ptr(s.noise)
            d.dec_out = nat.ptr(s.dec_out)
            d.t_curr, d.t_next = float(s.t_curr), float(s.t_next)
            if s.dcw is not None:
                flags |= self._stage_dcw(d, s, put_curve)
            d.flags = flags
            d.seed = int(s.seed) & ((1 << 64) - 1)
            d.step = int(s.step_idx)
        del table
        return b, off[0]

    def _stage_dcw(self, d, s: SlotStep, put_curve) -> int:
        """DCW coefficients of one slot: DCWCorrector.apply (acestep/engine/dcw.py:428-490) scales
        the low band by t * scaler and the high band by (1 - t) * scaler (double: high_scaler),
        resampled to the band length by _shape_for_wavelet (dcw.py:408-426); pix mode uses the
        raw scaler per frame in the pipeline dtype.  Evaluated with the reference's own tensor
        ops on the host."""
        mode, sc, hsc = s.dcw
        T, t = self.T, float(s.t_curr)
        if mode == "pix":
            c = _as_curve(sc, T)
            d.dcw_lo, d.dcw_lo_s = put_curve(c), (c if isinstance(c, float) else 0.0)
            return nat.ODE_DCW_PIX
        if mode not in ("low", "high", "double"):
            raise ValueError(f"invalid dcw mode {mode!r}")
        Td = (T + 1) // 2

        def band(coef, tm):
            c = _norm_curve(coef)                              # [1, T, 1] or [1, 1, 1]
            c = (tm * c).permute(0, 2, 1).contiguous().to(torch.float32)
            if c.shape[-1] not in (1, T):
                raise ValueError(f"DCW scaler curve has {c.shape[-1]} frames, expected 1 or T={T}")
            if c.shape[-1] == 1:
                return float(c.reshape(-1)[0])
            if c.shape[-1] != Td:
                c = torch.nn.functional.interpolate(c, size=Td, mode="linear", align_corners=False)
            return c.reshape(-1).contiguous()

        f = 0
        if mode in ("low", "double"):
            b = band(sc, t)
            d.dcw_lo, d.dcw_lo_s = put_curve(b), (b if isinstance(b, float) else 0.0)
            f |= nat.ODE_DCW_LO
        if mode in ("high", "double"):
            b = band(hsc if mode == "double" else sc, 1.0 - t)
            d.dcw_hi, d.dcw_hi_s = put_curve(b), (b if isinstance(b, float) else 0.0)
            f |= nat.ODE_DCW_HI
        return f

    def _launch(self, fn, gain: Optional[torch.Tensor], stream) -> None:
        if not self.slots:
            return
        if gain is not None and (gain.dtype != torch.bfloat16 or gain.shape != (self.T, self.D)):
            raise ValueError(f"gain must be bf16 [{self.T}, {self.D}]")
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        b, nbytes = self._stage()
        with torch.cuda.stream(st):
            self._dev[b][:nbytes].copy_(self._host[b][:nbytes], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(st)
        self._events[b] = ev
        self._buf ^= 1
        nat.check(fn(self._dev[b].data_ptr(), len(self.slots), self.T, self.D, nat.ptr(gain), int(st.cuda_stream)))

    def step(self, gain: Optional[torch.Tensor] = None, stream=None) -> None:
        """Advance every added slot by one step (demon_ode_step)."""
        self._launch(nat.load().demon_ode_step, gain, stream)

    def prepare(self, gain: Optional[torch.Tensor] = None, stream=None) -> None:
        """Write the decoder input of every added slot at its current step (demon_ode_prepare)."""
        self._launch(nat.load().demon_ode_prepare, gain, stream)
