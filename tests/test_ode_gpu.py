"""GPU parity of the fused ODE-step kernel against the ODE oracle (pinned to the
reference's StreamPipeline by tests/test_oracle_ode.py).

The kernel rounds to bf16 at the same tensor boundaries as the oracle; the only
differences left are fp32-vs-fp64 arithmetic inside the fused formulas, so the
bar is: >= 99% of elements bit-identical and every element within 1 bf16 ulp
of the operands' magnitude.
"""
import numpy as np
import pytest
import torch

from oracle import ode_oracle as OO

pytestmark = pytest.mark.gpu
D = 64


def bf(a):
    return OO.bf16(a)


def rand_curve(rng, T, lo, hi):
    knots = rng.uniform(lo, hi, 16)
    xs = np.linspace(0, 15, T)
    return np.interp(xs, np.arange(16), knots)


def make_spec(rng, T, kind):
    tcs = [(1.0, 0.8984375), (0.75, 0.5), (0.5, 0.25), (0.25, 0.0), (0.3984375, 0.0)]
    tc, tn = tcs[rng.integers(0, len(tcs))]
    s = dict(xt=bf(rng.standard_normal((T, D))), t_curr=tc, t_next=tn, step_idx=int(rng.integers(0, 8)),
             total_steps=8, infer_method="ode", has_cfg=False, rcfg_mode=None, complex_extra=False,
             pos=[(bf(rng.standard_normal((T, D))), None)], noise=bf(rng.standard_normal((T, D))),
             dec_next=tn > 0)
    if "cfg" in kind:
        s["has_cfg"] = True
        s["guidance"] = bf(rand_curve(rng, T, 3, 7)) if "curve" in kind else 4.5
        s["apg_momentum"] = bf(rand_curve(rng, T, -0.9, 0.0)) if "curve" in kind else -0.75
        s["momentum"] = None if "fresh" in kind else bf(rng.standard_normal((T, D)) * 0.5)
        if "rescale" in kind:
            s["cfg_rescale"] = bf(rand_curve(rng, T, 0, 1))
        if "self" in kind:
            s["rcfg_mode"] = "self"
            s["initial_noise"] = bf(rng.standard_normal((T, D)))
        elif "init0" in kind:
            s["rcfg_mode"] = "initialize"
            s["neg"] = [(bf(rng.standard_normal((T, D))), None)]
        elif "cached" in kind:
            s["rcfg_mode"] = "initialize"
            s["neg_cached"] = bf(rng.standard_normal((T, D)))
        else:
            s["neg"] = [(bf(rng.standard_normal((T, D))), None)]
    if "multi" in kind:
        s["pos"].append((bf(rng.standard_normal((T, D))), bf(rand_curve(rng, T, 0.1, 1.0))))
        s["pos"][0] = (s["pos"][0][0], bf(rand_curve(rng, T, 0.1, 1.0)))
        s["complex_extra"] = True
    if "vs" in kind:
        s["velocity_scale"] = bf(rand_curve(rng, T, 0, 1.5))
    if "onc" in kind:
        s["ode_noise_curve"] = bf(rand_curve(rng, T, 0, 0.3))
    if "sdecurve" in kind:
        s["sde_denoise_curve"] = bf(rand_curve(rng, T, 0, 1))
        s["source"] = bf(rng.standard_normal((T, D)))
    if "sdebare" in kind:
        s["infer_method"] = "sde"
    if "mask" in kind:
        m = np.zeros(T)
        a = int(rng.integers(0, T // 2))
        m[a:a + int(0.4 * T)] = 1.0
        s["mask"] = dict(mask=m, strength=1.0, strength_next=1.0, original=bf(rng.standard_normal((T, D))),
                         noise=bf(rng.standard_normal((T, D))))
    if "x0curve" in kind:
        s["x0_target"] = bf(rng.standard_normal((T, D)))
        s["x0_target_curve"] = bf(rand_curve(rng, T, 0, 1))
        s["x0_target_gate"] = 0.25
        s["step_idx"] = 6
    if "x0scalar" in kind:
        s["x0_target"] = bf(rng.standard_normal((T, D)))
        s["x0_target_strength"] = 0.375
        s["step_idx"] = 5
    for mode in ("double", "low", "high", "pix"):
        if "dcw" + mode in kind:
            sc = rand_curve(rng, T, 0.0, 0.1).astype(np.float32) if "dcwcurve" in kind else 0.05
            s["dcw"] = (mode, sc, 0.02)
    return s


KINDS = ["plain", "vs", "vs+onc", "cfg", "cfg+curve+rescale", "cfg+fresh", "cfg+self+rescale", "cfg+init0+fresh",
         "cfg+cached+curve", "multi", "multi+cfg", "mask", "mask+cfg+curve", "x0curve", "x0scalar",
         "sdecurve", "sdecurve+vs", "sdebare", "sdebare+mask", "mask+onc+vs",
         # DCW post-step correction (haar bands, scalar or per-frame scalers; pix mode)
         "dcwdouble", "cfg+vs+dcwdouble", "mask+cfg+dcwlow+dcwcurve", "sdecurve+dcwhigh", "x0scalar+dcwdouble+dcwcurve",
         "cfg+dcwpix+dcwcurve", "mask+onc+vs+dcwdouble"]


def to_slot(spec, dev, ode):
    t = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).to(dev).contiguous()  # noqa: E731
    T = spec["xt"].shape[0]
    mom = None
    fresh = True
    if spec.get("has_cfg"):
        if spec.get("momentum") is None:
            mom = torch.zeros(T, D, dtype=torch.bfloat16, device=dev)
        else:
            mom, fresh = t(spec["momentum"]), False
    mask = None
    if spec.get("mask"):
        mk = spec["mask"]
        mask = ode.LatentMask(torch.from_numpy(mk["mask"].astype(np.float32)).to(dev), t(mk["original"]),
                              t(mk["noise"]), mk["strength"], mk["strength_next"])
    st = ode.SlotStep(
        xt=t(spec["xt"]), t_curr=spec["t_curr"], t_next=spec["t_next"], step_idx=spec["step_idx"],
        total_steps=spec["total_steps"], pos=[(t(v), None if w is None else torch.from_numpy(w)) for v, w in spec["pos"]],
        has_cfg=spec.get("has_cfg", False), rcfg_mode=spec.get("rcfg_mode"),
        neg=[(t(v), None if w is None else torch.from_numpy(w)) for v, w in spec["neg"]] if spec.get("neg") else None,
        neg_cached=t(spec["neg_cached"]) if spec.get("neg_cached") is not None else None,
        initial_noise=t(spec["initial_noise"]) if spec.get("initial_noise") is not None else None,
        momentum=mom, momentum_fresh=fresh,
        neg_cache_out=torch.zeros(T, D, dtype=torch.bfloat16, device=dev) if spec.get("rcfg_mode") == "initialize" else None,
        guidance=_c(spec.get("guidance")), apg_momentum=_c(spec.get("apg_momentum", -0.75)),
        cfg_rescale=_c(spec.get("cfg_rescale")), velocity_scale=_c(spec.get("velocity_scale")),
        sde_denoise_curve=_c(spec.get("sde_denoise_curve")), ode_noise_curve=_c(spec.get("ode_noise_curve")),
        source=t(spec["source"]) if spec.get("source") is not None else None,
        x0_target=t(spec["x0_target"]) if spec.get("x0_target") is not None else None,
        x0_target_curve=_c(spec.get("x0_target_curve")), x0_target_gate=spec.get("x0_target_gate", 0.0),
        x0_target_strength=_c(spec.get("x0_target_strength", 0.0)), mask=mask,
        complex_extra=spec.get("complex_extra", False), infer_method=spec.get("infer_method", "ode"),
        noise=t(spec["noise"]), dec_out=torch.zeros(T, D, dtype=torch.bfloat16, device=dev) if spec.get("dec_next") else None,
        dcw=(lambda d: None if d is None else (d[0], _c(d[1]), _c(d[2])))(spec.get("dcw")), seed=1234)
    return st


def _c(v):
    if v is None or isinstance(v, (int, float)):
        return v
    return torch.from_numpy(np.asarray(v, np.float32))


def ulp_at(x):
    a = np.maximum(np.abs(x), 2.0 ** -8)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def check(name, got, ref, scale):
    got = got.float().cpu().numpy().astype(np.float64)
    diff = np.abs(got - ref)
    err = diff / ulp_at(scale)
    exact = np.mean(diff == 0)
    assert err.max() <= 1.0 + 1e-9, (name, err.max(), exact)
    assert exact >= 0.99, (name, exact)


def _slots_for_cluster(T, cl):
    """The fewest slots for which the ODE launch takes `cl`-CTA clusters on this device."""
    from demon_b200 import _native
    for n in range(1, 4096):
        if _native.ode_cluster_size(n, T) == cl:
            return n
    pytest.skip(f"no slot count takes {cl}-CTA clusters here")


@pytest.mark.parametrize("T,n", [(750, None), (123, None), (1500, None), (301, 64), (301, "cl4"), (301, "cl8"),
                                 (301, "cl16")])
def test_ode_step_matches_oracle(cuda, T, n):
    """Every kind of slot once (n None), or n slots cycling through the kinds.  The launch's
    cluster size (CTAs per slot: 4, 8 or 16) follows the slot count; "clX" takes the fewest
    slots for which the launch uses X (skipped when no slot count does on this GPU)."""
    from demon_b200 import ode
    if isinstance(n, str):
        n = _slots_for_cluster(T, int(n[2:]))
    rng = np.random.default_rng(T)
    kinds = KINDS if n is None else [KINDS[i % len(KINDS)] for i in range(n)]
    specs = [make_spec(rng, T, k) for k in kinds]
    gain = bf(rng.uniform(0.8, 1.2, (T, D)))
    for s in specs:
        s["gain"] = gain
    slots = [to_slot(s, cuda, ode) for s in specs]
    tick = ode.OdeTick(cuda, T, max_slots=len(slots))
    for st in slots:
        tick.add(st)
    gain_t = torch.from_numpy(gain.astype(np.float32)).to(torch.bfloat16).to(cuda)
    tick.step(gain=gain_t)
    torch.cuda.synchronize()
    from demon_b200 import _native
    assert _native.device_status() == (0, 0)
    for k, s, st in zip(kinds, specs, slots):
        ref = OO.step_slot(s, rnd=OO.bf16)
        scale = np.maximum(np.abs(ref["xt"]), np.abs(s["xt"]))
        check(f"{k}:xt", st.xt, ref["xt"], scale)
        if "momentum" in ref:
            # v_pos - v_neg can cancel: measure in ulps of the velocities' magnitude
            vmag = np.maximum(np.abs(s["pos"][0][0]), np.abs(ref["momentum"]))
            check(f"{k}:momentum", st.momentum, ref["momentum"], vmag)
        if "neg_cache" in ref:
            assert np.array_equal(st.neg_cache_out.float().cpu().numpy(), ref["neg_cache"]), k
        if "dec" in ref:
            # the decoder input from the kernel's own new state (the state is checked above; a
            # one-ulp difference there would otherwise be amplified by the mask blend and gain)
            xk = st.xt.float().cpu().numpy().astype(np.float64)
            dref = OO.next_dec(xk, s, rnd=OO.bf16)
            check(f"{k}:dec", st.dec_out, dref, np.maximum(np.abs(dref), scale))


@pytest.mark.parametrize("n", [2, 64])
def test_ode_prepare_matches_oracle(cuda, n):
    from demon_b200 import ode
    T = 300
    rng = np.random.default_rng(7)
    gain = bf(rng.uniform(0.8, 1.2, (T, D)))
    specs = [make_spec(rng, T, ("plain", "mask")[i % 2]) for i in range(n)]
    tick = ode.OdeTick(cuda, T, max_slots=n)
    slots = []
    for s in specs:
        s["gain"] = gain
        s["dec_next"] = True
        st = to_slot(s, cuda, ode)
        slots.append(st)
        tick.add(st)
    tick.prepare(gain=torch.from_numpy(gain.astype(np.float32)).to(torch.bfloat16).to(cuda))
    torch.cuda.synchronize()
    for s, st in zip(specs, slots):
        ref = OO.prepare_dec(s, rnd=OO.bf16)
        assert np.array_equal(st.dec_out.float().cpu().numpy(), ref)
        assert np.array_equal(st.xt.float().cpu().numpy(), s["xt"])  # prepare never writes the state


def test_ode_in_kernel_noise_is_deterministic_and_gaussian(cuda):
    """In-kernel noise: same seed/step -> identical bits; statistics of N(0,1)."""
    from demon_b200 import ode
    T = 1500
    outs = []
    for step in (3, 3, 4):
        xt = torch.zeros(T, D, dtype=torch.bfloat16, device=cuda)
        v = torch.zeros(T, D, dtype=torch.bfloat16, device=cuda)
        st = ode.SlotStep(xt=xt, t_curr=1.0, t_next=0.5, step_idx=step, total_steps=8, pos=[(v, None)],
                          infer_method="sde", seed=99)
        tick = ode.OdeTick(cuda, T, max_slots=1)
        tick.add(st)
        tick.step()
        outs.append(xt.float().cpu())
    assert torch.equal(outs[0], outs[1])
    z = outs[0] / 0.5  # bare SDE: xt = t_next * noise + (1 - t_next) * 0
    assert abs(float(z.mean())) < 0.02 and abs(float(z.std()) - 1.0) < 0.02
    # the two normals of one draw, neighbouring draws and the next step are uncorrelated
    def corr(a, b):
        a, b = a.flatten() - a.mean(), b.flatten() - b.mean()
        return float((a * b).sum() / (a.norm() * b.norm()))
    assert abs(corr(z[:, 0::2], z[:, 1::2])) < 0.02
    assert abs(corr(z[:, 0:D - 2], z[:, 2:D])) < 0.02
    assert abs(corr(z, outs[2] / 0.5)) < 0.02
    assert abs(float((z ** 4).mean()) - 3.0) < 0.15   # Gaussian kurtosis


def test_ode_rejects_bad_launches(cuda):
    """Shape and alignment checks run on the host before any launch: each bad argument raises
    DemonError through the C ABI, and the device status stays clean."""
    from demon_b200 import _native
    L = _native.load()
    table = torch.zeros(4096, dtype=torch.uint8, device=cuda)  # never read: every call is rejected
    gain = torch.zeros(2 * 64 + 8, dtype=torch.bfloat16, device=cuda)
    sp = _native.stream_ptr()
    bad = [
        (table.data_ptr(), 0, 100, 64, 0),                       # no slots
        (table.data_ptr(), 1, 0, 64, 0),                         # T = 0
        (table.data_ptr(), 1, 6401, 64, 0),                      # T above the maximum
        (table.data_ptr(), 1, 100, 32, 0),                       # latent width other than 64
        (table.data_ptr(), 4096, 100, 64, 0),                    # more slots than the grid allows
        (table.data_ptr() + 4, 1, 100, 64, 0),                   # slot table not 8-byte aligned
        (table.data_ptr(), 1, 100, 64, gain.data_ptr() + 2),     # gain not 16-byte aligned
    ]
    for args in bad:
        for fn in (L.demon_ode_step, L.demon_ode_prepare):
            with pytest.raises(_native.DemonError):
                _native.check(fn(*args, sp))
    with pytest.raises(_native.DemonError):
        _native.ode_cluster_size(1, 0)
    assert _native.device_status() == (0, 0)


def test_ode_cluster_size_choices(cuda):
    """One slot spreads over 16 CTAs (one per SM); a full B200 ring of 64 slots at T=1500 takes
    8-CTA clusters; far more slots than fit at once fall back to 4."""
    from demon_b200 import _native
    sizes = {n: _native.ode_cluster_size(n, 1500) for n in (1, 9, 10, 64, 400, 4095)}
    assert set(sizes.values()) <= {4, 8, 16}
    assert sizes[1] == 16 and sizes[4095] == 4
    n_sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    if n_sm >= 148:
        assert sizes[9] in (8, 16) and sizes[10] == 8 and sizes[64] == 8
