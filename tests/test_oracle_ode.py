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
