"""Ring-buffer streaming pipeline on B200: the reference's ``StreamPipeline`` tick
with the fused ODE-step kernel.

Mirrors ``acestep/engine/stream.py`` (``StreamPipeline`` 200-1490, ``SlotRequest``
57-180, ``SlotCondition`` 31-55): same public methods (``submit``, ``tick``,
``set_depth``, ``set_shared_curve``, ``set_channel_gain_tensor``, ``flush``,
``stats``, ``close``), same slot lifecycle (queue capped at depth, finished
slot popped before new slots are initialised, T-coherence purge), same
timestep schedule and CPU noise initialisation.  The per-slot post-forward
math of ``_tick_pt`` (stream.py:1060-1276) runs as ONE ``demon_ode_step``
launch for all slots, which also writes the next tick's decoder input rows
(mask pre-blend at t_next times the channel gain, stream.py:983-998), so a
tick is: gather decoder rows -> decoder forward (pos, then neg) -> one ODE
launch.  The decoder is any module with the ``AceStepDiTModel.forward``
signature (``demon_b200.dit.DemonDiT`` on B200).

Noise: slot initial noise is drawn on the CPU exactly as the reference does
(stream.py:403-451); per-step noise (SDE / ode_noise_curve) is drawn in the
kernel from a counter-based generator keyed by (slot seed, step), so a slot's trajectory does
not depend on which other slots share its ticks.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Tuple

import torch

from . import nvfp4 as Q
from . import ode as O


# ---------------------------------------------------------------------------
# request types (field names and semantics of the reference's dataclasses)
# ---------------------------------------------------------------------------

@dataclass
class SlotCondition:
    """stream.py:31-55."""
    encoder_hidden_states: torch.Tensor
    encoder_attention_mask: torch.Tensor
    temporal_weight: Optional[torch.Tensor] = None
    step_range: Optional[Tuple[float, float]] = None

    def is_active_at_step(self, step_idx: int, total_steps: int) -> bool:
        if self.step_range is None or total_steps <= 0:
            return True
        progress = step_idx / total_steps
        return self.step_range[0] <= progress < self.step_range[1]


@dataclass
class LatentNoiseMask:
    """acestep/engine/masking.py:9-71."""
    mask: torch.Tensor
    original_latents: torch.Tensor
    step_strength_fn: Optional[Callable[[int, int], float]] = None
    noise: Optional[torch.Tensor] = None

    def strength(self, step_idx: int, total_steps: int) -> float:
        return 1.0 if self.step_strength_fn is None else float(self.step_strength_fn(step_idx, total_steps))


@dataclass
class SlotRequest:
    """stream.py:57-180 (same fields, same defaults)."""
    encoder_hidden_states: torch.Tensor
    encoder_attention_mask: torch.Tensor
    context_latents: torch.Tensor
    seed: Optional["int | List[int]"] = None
    source_latents: Optional[torch.Tensor] = None
    denoise: float = 1.0
    sde_denoise_curve: Optional[torch.Tensor] = None
    velocity_scale: Optional[torch.Tensor] = None
    ode_noise_curve: Optional[torch.Tensor] = None
    x0_target: Optional[torch.Tensor] = None
    x0_target_strength: "float | torch.Tensor" = 0.0
    x0_target_curve: Optional[torch.Tensor] = None
    x0_target_gate: float = 0.0
    initial_noise_curve: Optional[torch.Tensor] = None
    latent_mask: Optional[LatentNoiseMask] = None
    extra_conditions: List[SlotCondition] = field(default_factory=list)
    primary_temporal_weight: Optional[torch.Tensor] = None
    primary_step_range: Optional[Tuple[float, float]] = None
    neg_conditions: List[SlotCondition] = field(default_factory=list)
    guidance_curve: Optional[torch.Tensor] = None
    apg_momentum: "float | torch.Tensor" = -0.75
    rcfg_mode: Optional[str] = None
    cfg_rescale_curve: "Optional[float | torch.Tensor]" = None

    def all_conditions(self) -> List[SlotCondition]:
        primary = SlotCondition(self.encoder_hidden_states, self.encoder_attention_mask,
                                self.primary_temporal_weight, self.primary_step_range)
        return [primary] + list(self.extra_conditions)

    @property
    def has_cfg(self) -> bool:
        if self.guidance_curve is None:
            return False
        if self.rcfg_mode == "self":
            return True
        return bool(self.neg_conditions)

    def needs_neg_forward(self, step_idx: int) -> bool:
        if not self.has_cfg or self.rcfg_mode == "self":
            return False
        if self.rcfg_mode == "initialize":
            return step_idx == 0
        return True


class GraphedDecoder:
    """Replays the decoder forward as one CUDA graph per input shape.

    A DiT forward is ~400 kernel launches; replaying a captured graph removes the host
    launch cost between them.  Inputs are copied into the graph's static buffers before
    each replay; graphs are dropped when any packed weight or hot-LoRA bank changed
    (``nvfp4.weights_generation``), since they bake in those device pointers.
    """

    def __init__(self, decoder):
        self.decoder = decoder
        self._graphs: dict = {}
        self._gen = None
        self._pool = None

    def _capture(self, x, t, enc, ctx):
        static = [x.clone(), t.clone(), enc.clone(), ctx.clone()]

        def run():
            return self.decoder(hidden_states=static[0], timestep=static[1], timestep_r=static[1],
                                attention_mask=None, encoder_hidden_states=static[2],
                                encoder_attention_mask=None, context_latents=static[3], use_cache=False,
                                past_key_values=None)[0]
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            run()  # warm-up: packs weights, sets kernel attributes, fills caches
        torch.cuda.current_stream(x.device).wait_stream(side)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._pool):
            out = run()
        return g, static, out

    def __call__(self, hidden_states, timestep, timestep_r=None, attention_mask=None, encoder_hidden_states=None,
                 encoder_attention_mask=None, context_latents=None, use_cache=False, past_key_values=None, **kw):
        gen = Q.weights_generation()
        if gen != self._gen:
            self._graphs.clear()
        key = (tuple(hidden_states.shape), tuple(encoder_hidden_states.shape), tuple(context_latents.shape))
        ent = self._graphs.get(key)
        if ent is None:
            ent = self._capture(hidden_states, timestep, encoder_hidden_states, context_latents)
            self._graphs[key] = ent
            self._gen = Q.weights_generation()
        g, static, out = ent
        for dst, src in zip(static, (hidden_states, timestep, encoder_hidden_states, context_latents)):
            dst.copy_(src)
        g.replay()
        # a copy: the next replay of the same shape (e.g. the negative pass) reuses `out`
        return out.clone(), past_key_values


@dataclass
class StreamConfig:
    """The DiffusionConfig fields the tick reads (acestep/engine/diffusion.py:13-59).

    DCW (Differential Correction in Wavelet domain, acestep/engine/dcw.py) is on by default
    with the reference's defaults (diffusion.py:48-59) and runs inside the fused ODE kernel;
    the haar wavelet is implemented (the reference's default), other wavelets and the
    advanced faders (DCWAdvanced) raise NotImplementedError."""
    infer_steps: int = 8
    infer_method: str = "ode"
    shift: float = 3.0
    noise_on_cpu: bool = True
    dcw_enabled: bool = True
    dcw_mode: str = "double"
    dcw_scaler: object = 0.05
    dcw_high_scaler: object = 0.02
    dcw_wavelet: str = "haar"
    dcw_advanced: object = None


DCW_MODES = ("low", "high", "double", "pix")


def _dcw_spec(enabled: bool, mode: str, scaler, high_scaler, wavelet: str, advanced) -> Optional[tuple]:
    """DCWCorrector construction (dcw.py:348-391): validates the mode and returns the
    (mode, scaler, high_scaler) the kernel applies, or None when the corrector is inactive
    (disabled, or every scaler it uses is zero)."""
    if mode not in DCW_MODES:
        raise ValueError(f"Invalid dcw_mode='{mode}'. Expected one of {DCW_MODES}.")
    if not enabled:
        return None
    if wavelet != "haar":
        raise NotImplementedError(f"DCW wavelet {wavelet!r}: only 'haar' is implemented")
    if advanced is not None and any(float(getattr(advanced, f, 0.0)) > 0.0
                                    for f in ("mult_blend", "mag_phase", "soft_thresh")):
        raise NotImplementedError("DCW advanced faders (mult_blend / mag_phase / soft_thresh) are not implemented")

    def nz(v):
        return bool(torch.as_tensor(v, dtype=torch.float32).abs().gt(0).any())
    active = nz(scaler) or (mode == "double" and nz(high_scaler))
    return (mode, scaler, high_scaler) if active else None


def build_schedule(steps: int, shift: float, denoise: float, dtype=torch.bfloat16) -> torch.Tensor:
    """DiffusionEngine._build_timestep_schedule (diffusion.py:656-699), evaluated on the CPU
    in the pipeline dtype like the reference (stream.py:385-396)."""
    if denoise <= 1e-6:
        return torch.zeros(2, dtype=dtype)
    t_start = 1.0 if denoise >= 1.0 else steps / int(steps / denoise)
    t = torch.linspace(t_start, 0.0, steps + 1, dtype=dtype)
    if shift != 1.0:
        t = shift * t / (1 + (shift - 1) * t)
    return t


@dataclass
class _Slot:
    request: SlotRequest
    xt: torch.Tensor                 # [T, 64] bf16 (state)
    t_schedule: torch.Tensor         # CPU
    seed: int
    step_idx: int = 0
    momentum: Optional[torch.Tensor] = None
    momentum_fresh: bool = True
    initial_noise: Optional[torch.Tensor] = None
    neg_cache: Optional[torch.Tensor] = None
    neg_cached_valid: bool = False
    mask: Optional[O.LatentMask] = None
    conds: list = field(default_factory=list)   # request.all_conditions(), built once
    ctx: Optional[torch.Tensor] = None          # context latents on the device
    enc: dict = field(default_factory=dict)     # id(condition) -> encoder states on the device


class StreamPipeline:
    """B200 ring-buffer pipeline; one batched decoder forward (two with CFG) and one
    fused ODE launch per tick."""

    def __init__(self, decoder, config: Optional[StreamConfig] = None, pipeline_depth: Optional[int] = None,
                 device=None, dtype=torch.bfloat16, use_graphs: bool = False):
        self.decoder = GraphedDecoder(decoder) if use_graphs else decoder
        self.config = config or StreamConfig()
        self._depth = pipeline_depth if pipeline_depth is not None else self.config.infer_steps
        self._slots: List[Optional[_Slot]] = [None] * self._depth
        self._queue: List[SlotRequest] = []
        self._device = torch.device(device) if device is not None else None
        self._dtype = dtype
        self._schedule_cache: dict = {}
        self._shared_curves: dict = {}
        self._channel_gain: Optional[torch.Tensor] = None
        self._dec: Optional[torch.Tensor] = None   # [depth, T, 64] next decoder inputs
        self._ode: Optional[O.OdeTick] = None
        self._T: Optional[int] = None
        self.ticks = 0
        self._last_tick_ms = 0.0
        self._gain_dirty = False
        self._stage = [(None, None)] * 16   # pinned noise staging ring
        cfg = self.config
        self._dcw_cfg = dict(mode=cfg.dcw_mode, scaler=cfg.dcw_scaler, high_scaler=cfg.dcw_high_scaler,
                             wavelet=cfg.dcw_wavelet, advanced=cfg.dcw_advanced)
        self._dcw = _dcw_spec(cfg.dcw_enabled, **self._dcw_cfg)
        self._stage_i = 0

    # ------------------------------------------------------------------ properties
    @property
    def depth(self) -> int:
        return self._depth

    @property
    def active_slots(self) -> int:
        return sum(1 for s in self._slots if s is not None)

    @property
    def is_warmed_up(self) -> bool:
        return all(s is not None for s in self._slots)

    # ------------------------------------------------------------------ public API
    def submit(self, request: SlotRequest) -> None:
        """Queue capped at depth, oldest dropped (stream.py:372-383)."""
        if len(self._queue) >= self._depth:
            self._queue.pop(0)
        self._queue.append(request)

    def set_dcw(self, *, enabled: bool, mode: Optional[str] = None, scaler=None, high_scaler=None,
                wavelet: Optional[str] = None, advanced=None) -> None:
        """stream.py:1357-1385: replace the DCW corrector; takes effect on the next tick."""
        c = self._dcw_cfg
        self._dcw_cfg = dict(mode=mode if mode is not None else c["mode"],
                             scaler=scaler if scaler is not None else c["scaler"],
                             high_scaler=high_scaler if high_scaler is not None else c["high_scaler"],
                             wavelet=wavelet if wavelet is not None else c["wavelet"],
                             advanced=advanced if advanced is not None else c["advanced"])
        self._dcw = _dcw_spec(enabled, **self._dcw_cfg)

    def set_shared_curve(self, name: str, value) -> None:
        """stream.py:1319-1340: override a per-slot curve for every in-flight slot."""
        if value is None:
            self._shared_curves.pop(name, None)
        else:
            self._shared_curves[name] = value

    def set_channel_gain_tensor(self, gain: Optional[torch.Tensor]) -> None:
        """stream.py:1426-1437; takes effect on the next tick's decoder input."""
        if gain is None:
            self._channel_gain = None
            self._gain_dirty = True
            return
        dev = self._device or torch.device("cuda")
        self._channel_gain = gain.to(device=dev, dtype=self._dtype).reshape(gain.shape[-2], gain.shape[-1]).contiguous()
        self._gain_dirty = True

    def set_depth(self, depth: int) -> None:
        """stream.py:1278-1301 (clamped to [1, 8] like the reference)."""
        depth = max(1, min(depth, 8))
        if depth == self._depth:
            return
        self._slots = self._slots[:depth] if depth < self._depth else self._slots + [None] * (depth - self._depth)
        self._depth = depth
        if self._dec is not None:  # keep the decoder inputs of the slots that stay
            old, T = self._dec, self._T
            self._T = None
            self._ensure_buffers(T)
            n = min(old.shape[0], depth)
            self._dec[:n].copy_(old[:n])

    def flush(self) -> List[torch.Tensor]:
        results = []
        for _ in range(self._depth * 2):
            r = self.tick()
            if r is not None:
                results.append(r)
            if self.active_slots == 0 and not self._queue:
                break
        return results

    def stats(self) -> dict:
        return {"ticks": self.ticks, "active_slots": self.active_slots, "queue_depth": len(self._queue),
                "last_tick_ms": round(self._last_tick_ms, 2), "is_warmed_up": self.is_warmed_up,
                "backend": "demon_b200"}

    def close(self) -> None:
        self._slots, self._queue = [], []
        self._dec, self._ode, self._channel_gain = None, None, None
        self._schedule_cache.clear()
        self._shared_curves.clear()
        self.decoder = None

    # ------------------------------------------------------------------ internals
    def _eff(self, slot: _Slot, name: str):
        v = self._shared_curves.get(name)
        return v if v is not None else getattr(slot.request, name, None)

    def _schedule(self, denoise: float) -> torch.Tensor:
        if denoise not in self._schedule_cache:
            self._schedule_cache[denoise] = build_schedule(self.config.infer_steps, self.config.shift, denoise,
                                                           self._dtype)
        return self._schedule_cache[denoise]

    @staticmethod
    def noise_host(seed, T: int, D: int, dtype=torch.bfloat16) -> torch.Tensor:
        """A slot's initial noise [T, D] on the host, as the reference draws it
        (StreamPipeline._make_noise, stream.py:403-451, with noise_on_cpu, its default): torch's
        CPU generator, randn [1, D, T] per seed (an int seeds once, a list seeds row by row and a
        negative or None entry keeps the generator's state), transposed to [T, D] and rounded to
        the pipeline dtype.  A slot holds one sample: with a list of seeds its first row."""
        if isinstance(seed, list):
            rows = []
            for s in seed:
                if s is not None and s >= 0:
                    torch.manual_seed(int(s))
                rows.append(torch.randn(1, D, T, dtype=torch.float32))
            n = torch.cat(rows, 0)[:1]
        else:
            if seed is not None:
                torch.manual_seed(int(seed))
            n = torch.randn(1, D, T, dtype=torch.float32)
        return n.movedim(-1, -2)[0].to(dtype).contiguous()   # bf16 rounding as .to(dtype) does

    def _make_noise(self, req: SlotRequest, T: int, D: int) -> torch.Tensor:
        """The initial noise (noise_host) uploaded to the device."""
        host = self.noise_host(req.seed, T, D, self._dtype)
        # upload through a ring of pinned buffers (a pageable copy would stall the host on the GPU)
        k = self._stage_i = (self._stage_i + 1) % len(self._stage)
        buf, ev = self._stage[k]
        if buf is None or buf.shape != host.shape:
            buf = torch.empty(host.shape, dtype=host.dtype).pin_memory()
        elif ev is not None:
            ev.synchronize()        # the copy that last read this buffer has finished
        buf.copy_(host)
        out = buf.to(self._device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self._device))
        self._stage[k] = (buf, ev)
        return out

    def _ensure_buffers(self, T: int) -> None:
        if self._T != T or self._dec is None or self._dec.shape[0] != self._depth:
            self._T = T
            self._dec = torch.zeros(self._depth, T, 64, dtype=self._dtype, device=self._device)
            self._ode = O.OdeTick(self._device, T, max_slots=self._depth)
            self._prep = O.OdeTick(self._device, T, max_slots=self._depth)

    def _init_slot(self, req: SlotRequest, index: int) -> _Slot:
        """stream.py:453-502."""
        if self._device is None:
            self._device = req.encoder_hidden_states.device
        T = req.context_latents.shape[1]
        D = req.context_latents.shape[-1] // 2
        self._ensure_buffers(T)
        sched = self._schedule(req.denoise)
        noise = self._make_noise(req, T, D)
        t_start = float(sched[0])
        src = req.source_latents if req.source_latents is not None else (
            req.latent_mask.original_latents if req.latent_mask is not None else None)
        if req.initial_noise_curve is not None and src is not None:
            curve = torch.as_tensor(req.initial_noise_curve).reshape(-1, 1).to(self._device, self._dtype)
            xt = curve * noise + (1.0 - curve) * src.reshape(T, -1).to(self._dtype)
        elif src is not None and req.denoise < 1.0:
            xt = t_start * noise + (1.0 - t_start) * src.reshape(T, -1).to(self._dtype)
        else:
            xt = noise.clone()
        # per-step noise (SDE / ode_noise_curve) is drawn in the kernel from (seed, step): the
        # slot's trajectory then never depends on which other slots share its ticks
        seed = req.seed[0] if isinstance(req.seed, list) else req.seed
        sl = _Slot(request=req, xt=xt.contiguous(), t_schedule=sched,
                   seed=int(seed) if seed is not None else int(torch.randint(0, 2 ** 62, (1,))))
        if req.has_cfg:
            sl.momentum = torch.zeros(T, D, dtype=self._dtype, device=self._device)
        if req.rcfg_mode == "self":
            sl.initial_noise = noise.clone()
        if req.rcfg_mode == "initialize":
            sl.neg_cache = torch.zeros(T, D, dtype=self._dtype, device=self._device)
        # the request's conditioning moves to the device once (host requests: one H2D per slot)
        sl.ctx = req.context_latents.to(self._device, self._dtype, non_blocking=True)
        sl.conds = req.all_conditions()
        for c in sl.conds + list(req.neg_conditions):
            sl.enc[id(c)] = c.encoder_hidden_states.to(self._device, self._dtype, non_blocking=True)
        if req.latent_mask is not None:
            lm = req.latent_mask
            if lm.noise is None:
                lm.noise = torch.randn_like(lm.original_latents)
            sl.mask = O.LatentMask(lm.mask.reshape(-1).to(self._device, torch.float32),
                                   lm.original_latents.reshape(T, -1).to(self._device, self._dtype).contiguous(),
                                   lm.noise.reshape(T, -1).to(self._device, self._dtype).contiguous())
        return sl

    def _active_conds(self, sl: _Slot):
        total = len(sl.t_schedule) - 1
        conds = sl.conds
        act = [c for c in conds if c.is_active_at_step(sl.step_idx, total)]
        return act if act else [conds[0]]

    def _active_negs(self, sl: _Slot):
        if not sl.request.has_cfg:
            return []
        total = len(sl.t_schedule) - 1
        negs = sl.request.neg_conditions
        act = [c for c in negs if c.is_active_at_step(sl.step_idx, total)]
        return act if act else [negs[0]]

    def _forward(self, rows, slots):
        """One batched decoder call over (slot index, condition) rows (stream.py:605-663)."""
        # small host -> device inputs go through pinned memory: a pageable copy would make the
        # host wait for the device (cudaMemcpyAsync from pageable memory synchronises the stream)
        idx = torch.tensor([si for si, _ in rows], pin_memory=True).to(self._device, non_blocking=True)
        xb = self._dec.index_select(0, idx)
        mL = max(c.encoder_hidden_states.shape[1] for _, c in rows)
        enc = []
        for si, c in rows:
            e = slots[si].enc[id(c)]
            if e.shape[1] < mL:  # zero padding to the longest condition, as the reference does
                e = torch.nn.functional.pad(e, (0, 0, 0, mL - e.shape[1]))
            enc.append(e)
        enc = torch.cat(enc, 0)
        ctx = torch.cat([slots[si].ctx for si, _ in rows], 0)
        t = torch.tensor([float(slots[si].t_schedule[slots[si].step_idx]) for si, _ in rows],
                         dtype=self._dtype, pin_memory=True).to(self._device, non_blocking=True)
        out = self.decoder(hidden_states=xb, timestep=t, timestep_r=t, attention_mask=None,
                           encoder_hidden_states=enc, encoder_attention_mask=None, context_latents=ctx,
                           use_cache=False, past_key_values=None)
        return out[0]

    def _step_for(self, sl: _Slot, si: int, pos, neg, dec_next: bool) -> O.SlotStep:
        req = sl.request
        total = len(sl.t_schedule) - 1
        tc = float(sl.t_schedule[sl.step_idx])
        tn = float(sl.t_schedule[sl.step_idx + 1])
        mask = sl.mask
        if mask is not None:
            lm = req.latent_mask
            mask.strength = lm.strength(sl.step_idx, total)
            mask.strength_next = lm.strength(sl.step_idx + 1, total)
        st = O.SlotStep(
            xt=sl.xt, t_curr=tc, t_next=tn, step_idx=sl.step_idx, total_steps=total, pos=pos,
            has_cfg=req.has_cfg, rcfg_mode=req.rcfg_mode, neg=neg,
            neg_cached=sl.neg_cache if (req.rcfg_mode == "initialize" and sl.neg_cached_valid) else None,
            initial_noise=sl.initial_noise, momentum=sl.momentum, momentum_fresh=sl.momentum_fresh,
            neg_cache_out=sl.neg_cache, guidance=self._eff(sl, "guidance_curve"),
            apg_momentum=self._eff(sl, "apg_momentum"), cfg_rescale=self._eff(sl, "cfg_rescale_curve"),
            velocity_scale=self._eff(sl, "velocity_scale"), sde_denoise_curve=self._eff(sl, "sde_denoise_curve"),
            ode_noise_curve=self._eff(sl, "ode_noise_curve"),
            source=None if req.source_latents is None else req.source_latents.reshape(sl.xt.shape).to(
                self._device, self._dtype).contiguous(),
            x0_target=None if req.x0_target is None else req.x0_target.reshape(sl.xt.shape).to(
                self._device, self._dtype).contiguous(),
            x0_target_curve=req.x0_target_curve, x0_target_gate=req.x0_target_gate,
            x0_target_strength=self._eff(sl, "x0_target_strength"), mask=mask,
            complex_extra=bool(req.extra_conditions or req.primary_temporal_weight is not None
                               or req.primary_step_range is not None),
            infer_method=self.config.infer_method,
            dec_out=self._dec[si] if dec_next else None, dcw=self._dcw, seed=sl.seed)
        return st

    @torch.no_grad()
    def tick(self) -> Optional[torch.Tensor]:
        """stream.py:849-917 with the post-forward section as one fused launch: returns the
        finished latent [1, T, 64] of at most one slot, like the reference."""
        out = self._tick(pop_all=False)
        return out[0] if out else None

    @torch.no_grad()
    def tick_many(self) -> List[torch.Tensor]:
        """One tick that pops every finished slot (the reference pops one per tick, which
        stalls rings deeper than the step count): a ring of depth > infer_steps then keeps
        every slot active.  Returns the finished latents [1, T, 64] in slot order."""
        return self._tick(pop_all=True)

    def _tick(self, pop_all: bool) -> List[torch.Tensor]:
        t_start = time.time()
        if self._queue:
            target_T = self._queue[-1].context_latents.shape[1]
            self._queue = [r for r in self._queue if r.context_latents.shape[1] == target_T]
            for i, s in enumerate(self._slots):
                if s is not None and s.xt.shape[0] != target_T:
                    self._slots[i] = None
        finished = []
        for i, s in enumerate(self._slots):
            if s is not None and s.step_idx >= len(s.t_schedule) - 1:
                finished.append(s.xt.unsqueeze(0))
                self._slots[i] = None
                if not pop_all:
                    break
        new = []
        for i, s in enumerate(self._slots):
            if s is None and self._queue:
                self._slots[i] = self._init_slot(self._queue.pop(0), i)
                new.append(i)
        active = [(i, s) for i, s in enumerate(self._slots) if s is not None and s.step_idx < len(s.t_schedule) - 1]
        if not active:
            self._last_tick_ms = (time.time() - t_start) * 1000
            self.ticks += 1
            return finished
        gain = self._channel_gain
        if new or self._gain_dirty:
            # decoder input (mask pre-blend at t_curr, times the channel gain; stream.py:983-998) of
            # new slots, and of every slot after a gain change; afterwards each ODE step writes
            # its slot's next input
            self._prep.reset()
            for i, s in active:
                if i in new or self._gain_dirty:
                    self._prep.add(self._step_for(s, i, [(s.xt, None)], None, True))
            self._prep.prepare(gain=gain)
            self._gain_dirty = False
        slots = dict(active)
        pos_rows, neg_rows = [], []
        for i, s in active:
            for c in self._active_conds(s):
                pos_rows.append((i, c))
            if s.request.needs_neg_forward(s.step_idx):
                for c in self._active_negs(s):
                    neg_rows.append((i, c))
        # The reference runs the positive and the negative pass as two forwards (stream.py:1038-1054);
        # every decoder row here is computed from its own inputs alone, so one forward over both
        # row sets gives the same bits with twice the rows per GEMM and half the launches.
        v_all = self._forward(pos_rows + neg_rows, slots)
        v_pos = v_all[:len(pos_rows)]
        v_neg = v_all[len(pos_rows):] if neg_rows else None
        self._ode.reset()
        pp = pn = 0
        for i, s in active:
            np_ = sum(1 for si, _ in pos_rows if si == i)
            pos = [(v_pos[pp + k], pos_rows[pp + k][1].temporal_weight) for k in range(np_)]
            pp += np_
            neg = None
            nn_ = sum(1 for si, _ in neg_rows if si == i)
            if nn_:
                neg = [(v_neg[pn + k], neg_rows[pn + k][1].temporal_weight) for k in range(nn_)]
                pn += nn_
            dec_next = s.step_idx + 1 < len(s.t_schedule) - 1
            self._ode.add(self._step_for(s, i, pos, neg, dec_next))
        self._ode.step(gain=gain)
        for i, s in active:
            if s.request.has_cfg and (s.request.rcfg_mode == "self" or s.request.neg_conditions):
                s.momentum_fresh = False
            if s.request.rcfg_mode == "initialize" and s.request.needs_neg_forward(s.step_idx):
                s.neg_cached_valid = True
            s.step_idx += 1
        self._last_tick_ms = (time.time() - t_start) * 1000
        self.ticks += 1
        return finished


def generate(decoder, request: SlotRequest, config: Optional[StreamConfig] = None, device=None) -> torch.Tensor:
    """The single-request (batch) path: the request alone through a depth-1 ring.

    Every decoder row and every ODE slot is computed independently of the others, so the
    result is bit-identical to the same request's output from a shared streaming ring.
    """
    pipe = StreamPipeline(decoder, config, pipeline_depth=1, device=device)
    pipe.submit(request)
    while True:
        out = pipe.tick()
        if out is not None:
            return out
