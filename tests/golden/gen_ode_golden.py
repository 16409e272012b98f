"""Generate golden vectors for the ODE step from the reference's own StreamPipeline.

Run in the build container only (needs the reference checkout):

    PYTHONPATH=/path/to/DEMON PYTHONDONTWRITEBYTECODE=1 python tests/golden/gen_ode_golden.py /path/to/DEMON

It drives acestep.engine.stream.StreamPipeline (dcw off, eager step helpers)
with a deterministic fake decoder, intercepts ``torch.randn_like`` with a seeded
generator so every noise draw is recorded, and stores, for each active slot of
each tick: the state before the step, the decoder velocities that belong to the
slot, the noise it drew, and the state after.  Writes ode_golden.npz next to
this script.  Scenarios cover the fast path, per-frame curves, SDE (curve and
bare), CFG / RCFG-initialize / RCFG-self with APG momentum and cfg_rescale
curves, latent masks, x0-target blends (curve + gate, scalar strength),
multi-condition blends, shared-curve overrides and channel gain.
"""
from __future__ import annotations

import json
import sys
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
T, D, STEPS, DEPTH, TICKS = 12, 64, 4, 3, 6


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from acestep.engine import stream as S
    from acestep.engine.diffusion import DiffusionConfig, DiffusionEngine
    from acestep.engine.masking import LatentNoiseMask

    out_arrays: dict[str, np.ndarray] = {}
    records = []

    def fake_engine():
        eng = object.__new__(DiffusionEngine)
        eng.model = None
        eng._trt_ctx = eng._trt_stream = eng._trt_engine = None
        eng._compile_loops = False
        eng._engine_swap_listeners = []

        class Dec:
            def __call__(self, hidden_states, timestep, encoder_hidden_states, **kw):
                # v = a(t) x + 0.3 c, c = first encoder row (per condition)
                a = torch.cos(3.0 * timestep.float()).to(hidden_states.dtype).view(-1, 1, 1) * 0.8
                c = encoder_hidden_states[:, :1, :D]
                return (hidden_states * a + c * 0.3,)
        eng.decoder = Dec()
        return eng

    def curve(g, lo=0.0, hi=1.5):
        knots = torch.rand(5, generator=g) * (hi - lo) + lo
        xs = torch.linspace(0, 4, T)
        i = xs.floor().clamp(max=3).long()
        f = xs - i
        return knots[i] * (1 - f) + knots[i + 1] * f

    def cond(g, dtype, L=5, weight=None, step_range=None):
        enc = torch.randn(1, L, 2048, generator=g).to(dtype)
        return S.SlotCondition(encoder_hidden_states=enc, encoder_attention_mask=torch.ones(1, L, dtype=dtype),
                               temporal_weight=weight, step_range=step_range)

    def request(g, dtype, **kw):
        c = cond(g, dtype)
        ctx = torch.randn(1, T, 2 * D, generator=g).to(dtype)
        return S.SlotRequest(encoder_hidden_states=c.encoder_hidden_states,
                             encoder_attention_mask=c.encoder_attention_mask, context_latents=ctx,
                             seed=int(torch.randint(0, 10000, (1,), generator=g)), **kw)

    def scenario(name, dtype, build, infer_method="ode", shared=None, gain=False):
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()) % 10000)
        cfg = DiffusionConfig(infer_steps=STEPS, shift=3.0, dcw_enabled=False, infer_method=infer_method)
        pipe = S.StreamPipeline(fake_engine(), cfg, pipeline_depth=DEPTH)
        reqs = build(g, dtype)
        noise_gen = torch.Generator().manual_seed(1234)
        state = {"slot": None, "draws": {}}
        orig_randn_like = torch.randn_like

        def randn_like(t, *a, **k):
            z = torch.randn(t.shape, generator=noise_gen).to(t.dtype)
            if state["slot"] is not None:
                state["draws"][state["slot"]] = z.clone()
            return z

        orig_resolve = pipe._resolve_slot_curves

        def resolve(slot, vt):
            state["slot"] = id(slot)
            return orig_resolve(slot, vt)
        pipe._resolve_slot_curves = resolve
        fw_out = []
        fw_in = []
        orig_fw = pipe._decoder_forward

        def fw(*a, **k):
            fw_in.append(k["xt_batch"].clone())
            o = orig_fw(*a, **k)
            fw_out.append(o.clone())
            return o
        pipe._decoder_forward = fw
        if gain:
            pipe._device, pipe._dtype = torch.device("cpu"), dtype
            pipe.set_channel_gain_tensor((torch.rand(1, T, D, generator=g) * 0.4 + 0.8).to(dtype))
        if shared:
            for k_, v_ in shared(g).items():
                pipe.set_shared_curve(k_, v_)

        orig_tick_pt = pipe._tick_pt

        def tick_pt(slots, indices):
            pre = []
            for sl in slots:
                pos = pipe._active_conditions(sl)
                negs = pipe._active_neg_conditions(sl) if sl.request.needs_neg_forward(sl.step_idx) else []
                mb = sl.momentum_buffer
                ra = mb.running_average if mb is not None and torch.is_tensor(mb.running_average) else None
                pre.append(dict(slot=sl, idx=sl.step_idx, xt=sl.xt.clone(), n_pos=len(pos), n_neg=len(negs),
                                pos_w=[c.temporal_weight for c in pos], neg_w=[c.temporal_weight for c in negs],
                                mom=None if ra is None else ra.clone(),
                                cached=None if sl.vt_neg_cached is None else sl.vt_neg_cached.clone()))
            fw_out.clear()
            fw_in.clear()
            state["draws"] = {}
            torch.randn_like = randn_like
            try:
                orig_tick_pt(slots, indices)
            finally:
                torch.randn_like = orig_randn_like
                state["slot"] = None
            vpos_all = fw_out[0]
            vneg_all = fw_out[1] if len(fw_out) > 1 else None
            pp = pn = 0
            for p in pre:
                sl = p["slot"]
                key = f"{name}/{dtype_name}/t{pipe.ticks}/s{len(records)}"
                req = sl.request
                rec = dict(key=key, scenario=name, dtype=dtype_name, step_idx=p["idx"],
                           t_curr=float(sl.t_schedule[p["idx"]]), t_next=float(sl.t_schedule[p["idx"] + 1]),
                           total_steps=len(sl.t_schedule) - 1, infer_method=infer_method,
                           n_pos=p["n_pos"], n_neg=p["n_neg"], rcfg_mode=req.rcfg_mode, has_cfg=req.has_cfg,
                           complex_extra=bool(req.extra_conditions or req.primary_temporal_weight is not None
                                              or req.primary_step_range is not None))
                arrays = {"xt": p["xt"][0], "xt_new": sl.xt[0]}
                arrays["dec_in"] = fw_in[0][pp]
                for i in range(p["n_pos"]):
                    arrays[f"vpos{i}"] = vpos_all[pp + i]
                    if p["pos_w"][i] is not None:
                        arrays[f"wpos{i}"] = p["pos_w"][i].reshape(-1)
                pp += p["n_pos"]
                for i in range(p["n_neg"]):
                    arrays[f"vneg{i}"] = vneg_all[pn + i]
                    if p["neg_w"][i] is not None:
                        arrays[f"wneg{i}"] = p["neg_w"][i].reshape(-1)
                pn += p["n_neg"]
                if p["mom"] is not None:
                    arrays["mom"] = p["mom"][0]
                if sl.momentum_buffer is not None and torch.is_tensor(sl.momentum_buffer.running_average):
                    arrays["mom_new"] = sl.momentum_buffer.running_average[0]
                if p["cached"] is not None:
                    arrays["neg_cached"] = p["cached"][0]
                if sl.vt_neg_cached is not None:
                    arrays["neg_cached_new"] = sl.vt_neg_cached[0]
                if sl.initial_noise is not None:
                    arrays["initial_noise"] = sl.initial_noise[0]
                if id(sl) in state["draws"]:
                    arrays["noise"] = state["draws"][id(sl)][0]
                for fld in ("source_latents", "x0_target"):
                    v = getattr(req, fld)
                    if v is not None:
                        arrays[fld] = v[0]
                eff = {}
                for nm in ("guidance_curve", "apg_momentum", "cfg_rescale_curve", "velocity_scale",
                           "sde_denoise_curve", "ode_noise_curve", "x0_target_strength"):
                    v = pipe._eff_shared(sl, nm)
                    if v is not None:
                        eff[nm] = v.reshape(-1)
                for nm, v in eff.items():
                    arrays["c_" + nm] = v
                if req.x0_target_curve is not None:
                    arrays["x0_target_curve"] = req.x0_target_curve.reshape(-1)
                    rec["x0_target_gate"] = req.x0_target_gate
                if req.latent_mask is not None:
                    lm = req.latent_mask
                    arrays["mask"] = lm.mask.reshape(-1)
                    arrays["mask_original"] = lm.original_latents[0]
                    arrays["mask_noise"] = lm.noise[0]
                if pipe._channel_gain is not None:
                    arrays["gain"] = pipe._channel_gain[0]
                rec["arrays"] = sorted(arrays)
                for k_, v_ in arrays.items():
                    t_ = v_.detach()
                    out_arrays[f"{key}/{k_}"] = (t_.view(torch.int16).numpy() if t_.dtype == torch.bfloat16
                                                 else t_.float().numpy())
                records.append(rec)

        pipe._tick_pt = tick_pt
        dtype_name = "bf16" if dtype == torch.bfloat16 else "fp32"
        for r in reqs:
            pipe.submit(r)
        for _ in range(TICKS):
            if len(pipe._queue) < 1:
                for r in build(g, dtype)[:1]:
                    pipe.submit(r)
            pipe.tick()

    def b_fast(g, dt):
        return [request(g, dt, denoise=d) for d in (1.0, 1.0, 1.0)]

    def b_curves(g, dt):
        src = lambda: torch.randn(1, T, D, generator=g).to(dt)  # noqa: E731
        return [
            request(g, dt, denoise=0.75, source_latents=src(), velocity_scale=curve(g).view(1, T, 1).to(dt),
                    ode_noise_curve=(curve(g) * 0.2).view(1, T, 1).to(dt)),
            request(g, dt, denoise=0.5, source_latents=src(), sde_denoise_curve=curve(g, 0, 1).view(1, T, 1).to(dt)),
            request(g, dt, denoise=1.0, velocity_scale=curve(g).view(1, T, 1).to(dt)),
        ]

    def b_cfg(g, dt):
        gc = lambda: (curve(g) * 2.5 + 3.0).to(dt)  # noqa: E731  guidance 3..6.75
        return [
            request(g, dt, neg_conditions=[cond(g, dt)], guidance_curve=gc(), rcfg_mode=None,
                    apg_momentum=(curve(g, -0.9, 0.0)).to(dt), cfg_rescale_curve=curve(g, 0, 1).to(dt)),
            request(g, dt, neg_conditions=[cond(g, dt)], guidance_curve=gc(), rcfg_mode="initialize"),
            request(g, dt, guidance_curve=gc(), rcfg_mode="self", cfg_rescale_curve=0.7),
        ]

    def b_mask(g, dt):
        m = torch.zeros(T)
        m[2:7] = 1.0
        orig = torch.randn(1, T, D, generator=g).to(dt)
        lm = LatentNoiseMask(mask=m.to(dt), original_latents=orig, noise=torch.randn(1, T, D, generator=g).to(dt))
        tgt = torch.randn(1, T, D, generator=g).to(dt)
        return [
            request(g, dt, latent_mask=lm, denoise=1.0),
            request(g, dt, x0_target=tgt, x0_target_curve=curve(g, 0, 1).to(dt), x0_target_gate=0.25),
            request(g, dt, x0_target=tgt, x0_target_strength=0.4),
        ]

    def b_multi(g, dt):
        w1, w2 = curve(g, 0.1, 1.0).to(dt), curve(g, 0.1, 1.0).to(dt)
        return [
            request(g, dt, extra_conditions=[cond(g, dt, weight=w2)], primary_temporal_weight=w1),
            request(g, dt, neg_conditions=[cond(g, dt, weight=w1), cond(g, dt, weight=w2)],
                    guidance_curve=torch.full((T,), 4.0).to(dt)),
            request(g, dt, denoise=1.0),
        ]

    def b_sde_mask(g, dt):
        m = torch.zeros(T)
        m[5:] = 1.0
        lm = LatentNoiseMask(mask=m.to(dt), original_latents=torch.randn(1, T, D, generator=g).to(dt),
                             noise=torch.randn(1, T, D, generator=g).to(dt))
        return [request(g, dt, latent_mask=lm), request(g, dt), request(g, dt, denoise=0.75,
                                                                        source_latents=torch.randn(1, T, D, generator=g).to(dt))]

    shared_vs = lambda g: {"velocity_scale": curve(g, 0.5, 1.5), "ode_noise_curve": 0.1}  # noqa: E731

    with torch.no_grad():
        for dt in (torch.float32, torch.bfloat16):
            scenario("fast", dt, b_fast)
            scenario("curves", dt, b_curves)
            scenario("cfg", dt, b_cfg, gain=True)
            scenario("mask_x0", dt, b_mask)
            scenario("multicond", dt, b_multi)
            scenario("sde_mask", dt, b_sde_mask, infer_method="sde")
            scenario("shared", dt, b_fast, shared=shared_vs, gain=True)

    np.savez_compressed(HERE / "ode_golden.npz", **out_arrays)
    (HERE / "ode_golden.json").write_text(json.dumps({"T": T, "D": D, "records": records}, indent=0))
    print(f"{len(records)} slot-steps, {len(out_arrays)} arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_ode_golden.py <reference checkout>")
    main(sys.argv[1])
