"""Host-side branch selection of the fused ODE step (CPU, no GPU).

`ode.resolve_flags` turns a slot's fields into the kernel's DEMON_ODE_* flags the way
StreamPipeline._tick_pt picks its branch (acestep/engine/stream.py:1131-1194) and its APG
negative source (stream.py:1086-1104).  Each case below states the reference's rule it checks.
"""
import pytest
import torch

from demon_b200 import _native as nat
from demon_b200 import ode

T, D = 40, 64


def lat():
    return torch.zeros(T, D, dtype=torch.bfloat16)


def step(**kw):
    base = dict(xt=lat(), t_curr=0.75, t_next=0.5, step_idx=1, total_steps=8, pos=[(lat(), None)])
    base.update(kw)
    return ode.SlotStep(**base)


def flags(**kw):
    return ode.resolve_flags(step(**kw))


def test_plain_ode_step_takes_the_fast_euler_branch():
    """No CFG, mask, SDE or x0 target: x + dt * v, no x0 path (stream.py:1188-1194)."""
    f, cur = flags()
    assert f == 0
    assert cur["neg_src"] is None


def test_cfg_sources_and_momentum():
    """APG's negative: the forward's v_neg, the RCFG cache, or the initial noise for
    rcfg_mode="self"; the first step starts the running average at zero; RCFG "initialize"
    caches the forward's negative.  Any CFG slot takes the x0 path (has_complex)."""
    f, cur = flags(has_cfg=True, neg=[(lat(), None)], momentum_fresh=True, cfg_rescale=0.7)
    assert cur["neg_src"] == "forward"
    assert f & nat.ODE_CFG and f & nat.ODE_MOM_INIT and f & nat.ODE_RESCALE and f & nat.ODE_X0PATH
    assert not f & nat.ODE_CACHE_NEG
    f, cur = flags(has_cfg=True, rcfg_mode="initialize", neg=[(lat(), None)], momentum_fresh=False)
    assert f & nat.ODE_CACHE_NEG and not f & nat.ODE_MOM_INIT and not f & nat.ODE_RESCALE
    f, cur = flags(has_cfg=True, rcfg_mode="initialize", neg_cached=lat())
    assert cur["neg_src"] == "cache" and not f & nat.ODE_CACHE_NEG
    f, cur = flags(has_cfg=True, rcfg_mode="self", initial_noise=lat(), neg=[(lat(), None)])
    assert cur["neg_src"] == "self" and f & nat.ODE_CFG
    f, cur = flags(has_cfg=True)  # no negative available: no guidance this step
    assert cur["neg_src"] is None and not f & nat.ODE_CFG


def test_sde_branches():
    """A sde_denoise_curve with source latents selects step_sde_curve; infer_method="sde"
    alone selects the bare re-noise; a curve without source does neither."""
    f, _ = flags(sde_denoise_curve=0.5, source=lat())
    assert f & nat.ODE_SDE_CURVE and f & nat.ODE_X0PATH and not f & nat.ODE_SDE_BARE
    f, _ = flags(infer_method="sde")
    assert f & nat.ODE_SDE_BARE and f & nat.ODE_X0PATH and not f & nat.ODE_SDE_CURVE
    f, _ = flags(sde_denoise_curve=0.5)
    assert f == 0


def test_final_step_and_scalars():
    """t_next <= 0 ends on x0; velocity scale and ode noise curve set their flags."""
    f, _ = flags(t_next=0.0)
    assert f & nat.ODE_FINAL and f & nat.ODE_X0PATH
    f, cur = flags(velocity_scale=1.25, ode_noise_curve=torch.linspace(0, 1, T))
    assert f & nat.ODE_VS and f & nat.ODE_ONC and not f & nat.ODE_X0PATH
    assert cur["vs"] == 1.25 and cur["onc"].shape == (T,)


def test_mask_and_next_decoder_input():
    """A latent mask takes the x0 path with the pre / post blends; the next decoder input is
    written, mask-pre-blended when the slot has a mask."""
    m = ode.LatentMask(torch.ones(T), lat(), lat())
    f, _ = flags(mask=m, dec_out=lat())
    assert f & nat.ODE_MASK and f & nat.ODE_X0PATH and f & nat.ODE_DEC_OUT and f & nat.ODE_DEC_MASK
    f, _ = flags(dec_out=lat())
    assert f == nat.ODE_DEC_OUT


@pytest.mark.parametrize("step_idx,active", [(3, False), (4, True), (7, True)])
def test_scalar_x0_target_from_half_way(step_idx, active):
    """A scalar x0 strength applies from step total_steps // 2 on (stream.py:1153-1166)."""
    f, cur = flags(x0_target=lat(), x0_target_strength=0.3, step_idx=step_idx, total_steps=8)
    assert bool(f & nat.ODE_X0_TARGET) == active
    assert bool(f & nat.ODE_X0PATH) == active
    if active:
        assert cur["x0c"] == pytest.approx(0.3, abs=2e-3)


@pytest.mark.parametrize("step_idx,gate,active", [(2, 0.5, False), (6, 0.5, True), (0, 0.0, False), (1, 0.0, True)])
def test_x0_target_curve_gate(step_idx, gate, active):
    """An x0 target curve blends in once progress = step / (total - 1) passes the gate, scaled by
    (progress - gate) / (1 - gate) (stream.py:1214-1224)."""
    curve = torch.full((T,), 0.5)
    f, cur = flags(x0_target=lat(), x0_target_curve=curve, x0_target_gate=gate, step_idx=step_idx, total_steps=8)
    assert f & nat.ODE_X0PATH  # a curve makes the step complex either way
    assert bool(f & nat.ODE_X0_TARGET) == active
    if active:
        progress = step_idx / 7
        assert cur["x0mul"] == pytest.approx((progress - gate) / (1 - gate))


def test_curve_length_is_checked():
    with pytest.raises(ValueError):
        flags(velocity_scale=torch.ones(T + 1))
