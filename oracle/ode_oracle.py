"""ODE-step oracle: numpy restatement of the reference's per-slot post-forward step.

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package (demon_b200/).

Restates, for one slot of one tick, acestep/engine/stream.py:
  - the integration base: mask_pre_blend on x_t              (stream.py:983-998)
  - velocity assembly: blend_velocities, the vt_neg source   (stream.py:1060-1104)
  - APG + cfg_rescale                                          (stream.py:1106-1123)
  - branch selection and integration                          (stream.py:1125-1276)
composed from acestep/engine/ode_steps.py (line numbers on each helper below),
plus the next tick's decoder input (mask_pre_blend at t_next times the channel
gain, stream.py:983-998 of the following tick).

Arithmetic is float64.  ``rnd`` is applied where the reference materialises a
tensor that the step reuses; pass ``rnd=ident`` to compare with the reference
run in float32 and ``rnd=bf16`` to mirror a bfloat16 pipeline (the CUDA kernel
rounds at exactly these points).

A slot is described by a plain dict (see :func:`step_slot`), shared by the
fixture generator (which turns it into the reference's SlotRequest) and the
product-side tests (which turn it into DemonOdeSlot descriptors).
"""
from __future__ import annotations

import numpy as np


def ident(x):
    return np.asarray(x, np.float64)


def bf16(x):
    """Round-to-nearest-even to bfloat16, returned as float64."""
    f = np.asarray(x, np.float64).astype(np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    out = np.where(np.isfinite(f), out, f)
    return out.astype(np.float64)


def _curve(v, T):
    """normalize_curve (ode_steps.py:36-64) for one slot: scalar or [T] -> [T, 1]."""
    if v is None:
        return None
    a = np.asarray(v, np.float64)
    if a.ndim == 0 or a.size == 1:
        return np.full((T, 1), float(a.reshape(-1)[0]))
    return a.reshape(T, 1)


def pre_blend(x, t, m, noise, orig, rnd):
    """mask_pre_blend (ode_steps.py:89-106), rounded op by op like the reference's
    eager bf16 tensors: noised = t*noise + (1-t)*orig; m*x + (1-m)*noised."""
    noised = rnd(rnd(t * noise) + rnd((1.0 - t) * orig))
    return rnd(rnd(m * x) + rnd(rnd(1.0 - m) * noised))


def lerp_eager(x, c, y, rnd):
    """(1 - c) * x + c * y evaluated op by op (mask_post_blend_x0 writes it as
    m*x + (1-m)*y, ode_steps.py:109-142) -- the same rounding sequence."""
    return rnd(rnd(rnd(1.0 - c) * x) + rnd(c * y))


def blend(pairs, T, rnd):
    """blend_velocities (ode_steps.py:150-183); a single condition is used as is
    (stream.py:1068-1069)."""
    if len(pairs) == 1:
        return np.asarray(pairs[0][0], np.float64)
    num = 0.0
    den = 0.0
    for v, w in pairs:
        wc = np.ones((T, 1)) if w is None else _curve(w, T)
        num = num + np.asarray(v, np.float64) * wc
        den = den + wc
    return rnd(num / np.maximum(den, 1e-8))


def apg(vp, vn, r_old, g, m, rho, rnd):
    """MomentumBuffer.update + apg_forward + cfg_rescale (ode_steps.py:276-392),
    dims=(1,) i.e. norms over T per channel, eta=0, norm_threshold=2.5."""
    m = rnd(m)
    diff = rnd(vp - vn)
    r = diff if r_old is None else rnd(diff + rnd(m * r_old))
    nr = np.sqrt((r * r).sum(0, keepdims=True))
    with np.errstate(divide="ignore"):
        k = np.minimum(1.0, np.where(nr > 0, 2.5 / nr, np.inf))
    d = r * k
    nvp = np.sqrt((vp * vp).sum(0, keepdims=True))
    v1 = vp / np.maximum(nvp, 1e-12)
    par = (d * v1).sum(0, keepdims=True) * v1
    orth = d - par
    vg = vp + (rnd(g) - 1.0) * orth
    if rho is not None:
        ng = np.sqrt((vg * vg).sum(0, keepdims=True))
        sigma = nvp / np.maximum(ng, 1e-12)
        rb = rnd(rho)
        vg = rb * (vg * sigma) + (1.0 - rb) * vg
    return rnd(vg), r


def step_slot(s: dict, rnd=bf16) -> dict:
    """One slot, one tick.  Keys of ``s`` (latents are [T, 64] arrays, curves [T] or scalars):

    xt, t_curr, t_next, step_idx, total_steps, infer_method ('ode' | 'sde'),
    pos: [(v, weight|None), ...]  decoder outputs of the active positive conditions,
    has_cfg, rcfg_mode (None | 'full' | 'initialize' | 'self'),
    neg: [(v, weight|None), ...] or None (a negative forward ran this tick),
    neg_cached, initial_noise, momentum (None = fresh MomentumBuffer),
    guidance, apg_momentum, cfg_rescale (None = off),
    velocity_scale, sde_denoise_curve, ode_noise_curve (None = absent),
    source, x0_target, x0_target_curve, x0_target_gate, x0_target_strength,
    mask: None or {mask [T], strength, strength_next, original, noise},
    complex_extra (extra_conditions / primary_temporal_weight / primary_step_range set),
    noise: the step's randn draw [T, 64], gain: [T, 64] or None, dec_next (bool),
    dcw: None or (mode, scaler, high_scaler) of an active DCW corrector (see :func:`dcw`).
    """
    T = s["xt"].shape[0]
    x_state = np.asarray(s["xt"], np.float64)
    tc, tn = float(s["t_curr"]), float(s["t_next"])
    mask = s.get("mask")
    if mask is not None:
        m = rnd(_curve(mask["mask"], T) * float(mask.get("strength", 1.0)))
        x = pre_blend(x_state, tc, m, mask["noise"], mask["original"], rnd)
    else:
        x = x_state

    out = {}
    vp = blend(s["pos"], T, rnd)
    vn = None
    mode = s.get("rcfg_mode")
    if s.get("has_cfg"):
        if mode == "self":
            vn = np.asarray(s["initial_noise"], np.float64)
        elif s.get("neg") is not None:
            vn = blend(s["neg"], T, rnd)
            if mode == "initialize":
                out["neg_cache"] = vn
        elif s.get("neg_cached") is not None:
            vn = np.asarray(s["neg_cached"], np.float64)
    if vn is not None:
        vt, r = apg(vp, vn, s.get("momentum"), _curve(s["guidance"], T), _curve(s.get("apg_momentum", -0.75), T),
                    _curve(s.get("cfg_rescale"), T), rnd)
        out["momentum"] = r
    else:
        vt = vp

    # ---- branch selection (stream.py:1131-1194) ----
    vs = _curve(s.get("velocity_scale"), T)
    vs = rnd(vs) if vs is not None else 1.0
    sdc = _curve(s.get("sde_denoise_curve"), T)
    onc = _curve(s.get("ode_noise_curve"), T)
    onc = rnd(onc) if onc is not None else 0.0
    src = s.get("source")
    sde_curve_active = sdc is not None and src is not None
    use_sde = sde_curve_active or s.get("infer_method", "ode") == "sde"
    strength = _curve(s.get("x0_target_strength"), T)
    strength_active = strength is not None and bool(np.any(np.abs(strength) > 0))
    x0_target = s.get("x0_target")
    x0_curve = s.get("x0_target_curve")
    scalar_x0 = (x0_target is not None and strength_active and x0_curve is None
                 and s["step_idx"] >= s["total_steps"] // 2 and tc > 0)
    has_x0_curve = x0_target is not None and x0_curve is not None
    has_complex = (mask is not None or bool(s.get("complex_extra")) or has_x0_curve or bool(s.get("has_cfg")))
    needs_x0 = has_complex or scalar_x0 or use_sde or tn <= 0
    eps = np.asarray(s["noise"], np.float64) if s.get("noise") is not None else np.zeros_like(x)

    if not needs_x0:
        xn = x + (tn - tc) * (vt * vs) + eps * onc * tn                 # step_ode_euler (:191-216)
    else:
        x0 = rnd(x - rnd(rnd(vt * vs) * tc))                             # x0_from_vel (:72-81)
        if mask is not None:                                             # mask_post_blend_x0 (:109-121)
            x0 = rnd(rnd(m * x0) + rnd(rnd(1.0 - m) * mask["original"]))
        if has_x0_curve:
            total = s["total_steps"]
            progress = s["step_idx"] / max(total - 1, 1)
            gate = float(s.get("x0_target_gate", 0.0))
            bg = max(0.0, progress - gate) / max(1.0 - gate, 1e-6)
            if bg > 0:
                c = rnd(rnd(_curve(x0_curve, T)) * bg)
                x0 = lerp_eager(x0, c, x0_target, rnd)                   # blend_x0_target (:129-142)
        elif scalar_x0:
            x0 = lerp_eager(x0, rnd(strength), x0_target, rnd)           # stream.py:1231-1233
        if sde_curve_active:                                             # step_sde_curve (:219-242)
            sb = rnd(sdc)
            e = eps if tn > 0 else np.zeros_like(eps)
            xn = sb * (tn * e + (1.0 - tn) * x0) + (1.0 - sb) * (tn * e + (1.0 - tn) * src)
        elif tn <= 0:
            xn = x0
        elif use_sde:                                                    # step_sde_renoise (:245-266)
            nz = mask["noise"] if mask is not None else eps
            xn = tn * nz + (1.0 - tn) * x0
        else:
            vb = rnd(rnd(x - x0) / tc)                                   # stream.py:1269-1273
            xn = x + (tn - tc) * vb + eps * onc * tn
    xn = rnd(xn)
    if s.get("dcw") is not None:                                         # _maybe_dcw (stream.py:1387-1405)
        xn = dcw(xn, x, vt, tc, s["dcw"], rnd)
    out["xt"] = xn
    if s.get("dec_next"):
        out["dec"] = next_dec(xn, s, rnd)
    return out


def next_dec(xn, s: dict, rnd=bf16):
    """The next tick's decoder input from the new state: mask_pre_blend at t_next with the
    next step's strength, times the channel gain (stream.py:983-998 of the following tick)."""
    T = xn.shape[0]
    d = np.asarray(xn, np.float64)
    mask = s.get("mask")
    if mask is not None:
        mn = rnd(_curve(mask["mask"], T) * float(mask.get("strength_next", 1.0)))
        d = pre_blend(d, float(s["t_next"]), mn, mask["noise"], mask["original"], rnd)
    if s.get("gain") is not None:
        d = rnd(d * np.asarray(s["gain"], np.float64))
    return d


SQRT_HALF = 0.7071067811865476


def _band_scale(coef, t_mult: float, T: int, Td: int) -> np.ndarray:
    """DCWCorrector._shape_for_wavelet of ``t_mult * coef`` (acestep/engine/dcw.py:408-426):
    a scalar or [T] curve resampled to the band length Td by linear interpolation with
    align_corners=False (torch.nn.functional.interpolate)."""
    f32 = np.float32
    c = (f32(t_mult) * np.asarray(coef, np.float64).reshape(-1).astype(f32)).astype(f32)  # fp32 tensor ops
    if c.size == 1:
        return np.full(Td, float(c[0]))
    n = c.size
    # the source index in fp32 as the interpolation kernel computes it
    scale = f32(n) / f32(Td)
    src = np.maximum(scale * (np.arange(Td, dtype=f32) + f32(0.5)) - f32(0.5), f32(0.0)).astype(f32)
    i0 = src.astype(np.int64)
    i1 = np.minimum(i0 + 1, n - 1)
    lam = (src - i0.astype(f32)).astype(f32)
    return ((f32(1.0) - lam) * c[i0] + lam * c[i1]).astype(np.float64)


def dcw(x_next, x_pre, vt, t_curr: float, cfg, rnd=bf16):
    """DCW post-step correction (Yu et al., CVPR 2026), the reference's fast path:
    StreamPipeline._maybe_dcw (stream.py:1387-1405) -> DCWCorrector.apply (dcw.py:428-490)
    -> dcw_low / dcw_high / dcw_double / dcw_pix (dcw.py:164-234).

    denoised = x_pre - vt * t_curr (bf16 ops); then, for the wavelet modes, a single-level
    haar DWT along T of both latents (zero padding of an odd T, pytorch_wavelets
    DWT1DForward(J=1, mode='zero', wave='haar')), xL += t s (xL - yL) and / or
    xH += (1 - t) s_h (xH - yH), inverse DWT, trim to T, round.  ``cfg`` = (mode, scaler,
    high_scaler) with scalers scalar or [T].  Restated from the haar transform's definition
    (cA = (a + b)/sqrt 2, cD = (a - b)/sqrt 2 and its inverse): the sign convention of the
    detail band cancels between analysis and synthesis.  pytorch_wavelets is not installed
    here, so this restatement is not pinned to it."""
    mode, sc, hsc = cfg
    x_next = np.asarray(x_next, np.float64)
    T = x_next.shape[0]
    den = rnd(np.asarray(x_pre, np.float64) - rnd(np.asarray(vt, np.float64) * t_curr))
    if mode == "pix":                                                     # dcw_pix (:164-174)
        s = rnd(_curve(sc, T))
        return rnd(x_next + rnd(s * rnd(x_next - den)))
    Td = (T + 1) // 2
    xp = np.zeros((2 * Td, x_next.shape[1]))
    yp = np.zeros_like(xp)
    xp[:T], yp[:T] = x_next, den
    xl, xh = (xp[0::2] + xp[1::2]) * SQRT_HALF, (xp[0::2] - xp[1::2]) * SQRT_HALF
    yl, yh = (yp[0::2] + yp[1::2]) * SQRT_HALF, (yp[0::2] - yp[1::2]) * SQRT_HALF
    if mode in ("low", "double"):
        xl = xl + _band_scale(sc, t_curr, T, Td)[:, None] * (xl - yl)
    if mode in ("high", "double"):
        xh = xh + _band_scale(hsc if mode == "double" else sc, 1.0 - t_curr, T, Td)[:, None] * (xh - yh)
    out = np.empty_like(xp)
    out[0::2], out[1::2] = (xl + xh) * SQRT_HALF, (xl - xh) * SQRT_HALF
    return rnd(out[:T])


def prepare_dec(s: dict, rnd=bf16):
    """Decoder input of a slot at its current step: mask_pre_blend(x_t) * gain."""
    T = s["xt"].shape[0]
    x = np.asarray(s["xt"], np.float64)
    mask = s.get("mask")
    if mask is not None:
        m = rnd(_curve(mask["mask"], T) * float(mask.get("strength", 1.0)))
        x = pre_blend(x, float(s["t_curr"]), m, mask["noise"], mask["original"], rnd)
    if s.get("gain") is not None:
        x = rnd(x * np.asarray(s["gain"], np.float64))
    return x


def schedule(steps: int, shift: float, denoise: float) -> np.ndarray:
    """DiffusionEngine._build_timestep_schedule (acestep/engine/diffusion.py:656-699), evaluated
    in bfloat16 like the reference (stream.py:385-396): torch's linspace in the pipeline dtype
    (a numpy linspace rounded afterwards differs in the last bit for truncated schedules), then
    the shift as bf16 tensor ops.  Pinned by tests/golden/schedule_golden.json."""
    import torch
    if denoise <= 1e-6:
        return np.zeros(2)
    t_start = 1.0 if denoise >= 1.0 else steps / int(steps / denoise)
    t = torch.linspace(t_start, 0.0, steps + 1, dtype=torch.bfloat16)
    if shift != 1.0:
        t = shift * t / (1 + (shift - 1) * t)
    return t.float().numpy().astype(np.float64)
