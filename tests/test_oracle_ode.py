"""Pin the ODE oracle against vectors produced by the reference's own
StreamPipeline._tick_pt (tests/golden/gen_ode_golden.py).

fp32 pipelines: the oracle (float64, no intermediate rounding) must match the
reference to float32 accuracy -- this pins every branch and formula.
bf16 pipelines: the oracle with bf16 rounding at the tensor boundaries the
CUDA kernel uses is compared with the reference's op-by-op bf16 eager path;
the two differ only by where bf16 rounding happens, bounded here in ulps.
"""
import numpy as np
import pytest

from oracle import ode_oracle as OO
from tests import ode_fixtures as F

RECS = F.records()


def ulp_bf16(x):
    a = np.maximum(np.abs(x), 2.0 ** -8)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def test_fixture_coverage():
    scen = {(r["scenario"], r["dtype"]) for r, _ in RECS}
    assert len(scen) == 14
    modes = {r["rcfg_mode"] for r, _ in RECS if r["has_cfg"]}
    assert modes == {None, "initialize", "self"}
    assert any("mask" in A for _, A in RECS) and any("x0_target_curve" in A for _, A in RECS)
    assert any(r["t_next"] <= 0 for r, _ in RECS)


@pytest.mark.parametrize("idx", [i for i, (r, _) in enumerate(RECS) if r["dtype"] == "fp32"])
def test_oracle_matches_reference_fp32(idx):
    rec, A = RECS[idx]
    s = F.spec(rec, A)
    out = OO.step_slot(s, rnd=OO.ident)
    ref = A["xt_new"]
    np.testing.assert_allclose(out["xt"], ref, rtol=2e-5, atol=2e-5, err_msg=rec["key"])
    if "mom_new" in A and "momentum" in out:
        np.testing.assert_allclose(out["momentum"], A["mom_new"], rtol=1e-5, atol=1e-5)
    if "neg_cache" in out:
        np.testing.assert_array_equal(out["neg_cache"], A["neg_cached_new"])
    dec = OO.prepare_dec(s, rnd=OO.ident)
    np.testing.assert_allclose(dec, A["dec_in"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("idx", [i for i, (r, _) in enumerate(RECS) if r["dtype"] == "bf16"])
def test_oracle_matches_reference_bf16(idx):
    rec, A = RECS[idx]
    s = F.spec(rec, A)
    out = OO.step_slot(s, rnd=OO.bf16)
    ref = A["xt_new"]
    # op-by-op eager bf16 rounding vs rounding at tensor boundaries: at most a few
    # bf16 ulps of the operands' magnitude (state and result), never a branch difference
    scale = np.maximum(np.maximum(np.abs(ref), np.abs(A["xt"])), 0.5)
    err = np.abs(out["xt"] - ref) / ulp_bf16(scale)
    assert err.max() <= 4, (rec["key"], err.max())
    assert np.mean(out["xt"] == ref) > 0.5, rec["key"]
    dec = OO.prepare_dec(s, rnd=OO.bf16)
    np.testing.assert_array_equal(dec, A["dec_in"])


# ---------------------------------------------------------------------------------------
# DCW post-step correction
# ---------------------------------------------------------------------------------------

def _dcw_records():
    import json
    from pathlib import Path
    g = Path(__file__).resolve().parent / "golden"
    meta = json.loads((g / "dcw_golden.json").read_text())["records"]
    arrs = np.load(g / "dcw_golden.npz")

    def val(a):
        return (a.view(np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    out = []
    for r in meta:
        A = {n: val(arrs[f"{r['key']}/{n}"]) for n in ("x_next", "x_pre", "vt", "out")}
        if r["curve"]:
            A["scaler"] = arrs[f"{r['key']}/scaler"].astype(np.float64)
            A["high_scaler"] = arrs[f"{r['key']}/high_scaler"].astype(np.float64)
        out.append((r, A))
    return out


def test_dcw_oracle_matches_reference():
    """oracle.dcw against the reference's DCWCorrector.apply (tests/golden/gen_dcw_golden.py):
    bf16 outputs identical but for fp32-vs-fp64 ties, every element within one ulp."""
    recs = _dcw_records()
    assert {r["mode"] for r, _ in recs} == {"low", "high", "double", "pix"}
    for r, A in recs:
        sc = A["scaler"] if r["curve"] else r["scaler"]
        hsc = A["high_scaler"] if r["curve"] else r["high_scaler"]
        got = OO.dcw(A["x_next"], A["x_pre"], A["vt"], r["t_curr"], (r["mode"], sc, hsc), rnd=OO.bf16)
        ref = A["out"]
        scale = np.maximum(np.abs(ref), 2.0 ** -8)
        ulp = 2.0 ** (np.floor(np.log2(scale)) - 7)
        assert np.max(np.abs(got - ref) / ulp) <= 1.0, r
        assert np.mean(got == ref) >= 0.99, (r, np.mean(got == ref))


def test_dcw_zero_scalers_and_perfect_reconstruction():
    rng = np.random.default_rng(3)
    for T in (10, 11, 1):
        x = OO.bf16(rng.standard_normal((T, 64)))
        pre, vt = OO.bf16(rng.standard_normal((T, 64))), OO.bf16(rng.standard_normal((T, 64)))
        for mode in ("low", "high", "double", "pix"):
            assert np.array_equal(OO.dcw(x, pre, vt, 0.5, (mode, 0.0, 0.0)), x), (T, mode)


def test_dcw_band_scale_matches_torch_interpolate():
    import torch
    for T in (1500, 751, 123, 10):
        c = torch.rand(T, generator=torch.Generator().manual_seed(T))
        Td = (T + 1) // 2
        ref = torch.nn.functional.interpolate((0.375 * c).reshape(1, 1, T), size=Td, mode="linear",
                                              align_corners=False).reshape(-1).double().numpy()
        got = OO._band_scale(c.numpy(), 0.375, T, Td)
        assert np.max(np.abs(got - ref)) <= 6e-8 * max(1.0, np.abs(ref).max())
