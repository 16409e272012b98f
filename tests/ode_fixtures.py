"""Load the reference-generated ODE golden vectors (tests/golden/ode_golden.*) as
slot dicts in the format of oracle.ode_oracle.step_slot."""
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=1)
def load():
    meta = json.loads((GOLDEN / "ode_golden.json").read_text())
    arrs = np.load(GOLDEN / "ode_golden.npz")
    return meta, {k: arrs[k] for k in arrs.files}


def _val(a, dtype):
    """int16 arrays hold bf16 bit patterns; float32 arrays hold values."""
    if a.dtype == np.int16:
        return (a.view(np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return a.astype(np.float64)


def records():
    meta, arrs = load()
    out = []
    for rec in meta["records"]:
        A = {n: _val(arrs[f"{rec['key']}/{n}"], rec["dtype"]) for n in rec["arrays"]}
        out.append((rec, A))
    return out


def spec(rec, A):
    """Slot dict for oracle.ode_oracle.step_slot from one golden record."""
    s = dict(xt=A["xt"], t_curr=rec["t_curr"], t_next=rec["t_next"], step_idx=rec["step_idx"],
             total_steps=rec["total_steps"], infer_method=rec["infer_method"],
             has_cfg=rec["has_cfg"], rcfg_mode=rec["rcfg_mode"], complex_extra=rec["complex_extra"])
    s["pos"] = [(A[f"vpos{i}"], A.get(f"wpos{i}")) for i in range(rec["n_pos"])]
    s["neg"] = [(A[f"vneg{i}"], A.get(f"wneg{i}")) for i in range(rec["n_neg"])] if rec["n_neg"] else None
    s["neg_cached"] = A.get("neg_cached")
    s["initial_noise"] = A.get("initial_noise")
    s["momentum"] = A.get("mom")
    s["guidance"] = A.get("c_guidance_curve")
    s["apg_momentum"] = A.get("c_apg_momentum", -0.75)
    s["cfg_rescale"] = A.get("c_cfg_rescale_curve")
    s["velocity_scale"] = A.get("c_velocity_scale")
    s["sde_denoise_curve"] = A.get("c_sde_denoise_curve")
    s["ode_noise_curve"] = A.get("c_ode_noise_curve")
    s["x0_target_strength"] = A.get("c_x0_target_strength")
    s["source"] = A.get("source_latents")
    s["x0_target"] = A.get("x0_target")
    s["x0_target_curve"] = A.get("x0_target_curve")
    s["x0_target_gate"] = rec.get("x0_target_gate", 0.0)
    if "mask" in A:
        s["mask"] = dict(mask=A["mask"], strength=1.0, strength_next=1.0, original=A["mask_original"],
                         noise=A["mask_noise"])
    s["noise"] = A.get("noise")
    s["gain"] = A.get("gain")
    return s
