"""Generate tests/golden/dcw_golden.{json,npz}: DCW post-step corrections computed by the
reference's own acestep/engine/dcw.py (DCWCorrector.apply -> dcw_low / dcw_high /
dcw_double / dcw_pix) in this container.

The reference's wavelet dependency, pytorch_wavelets, is not installed here.  A minimal
stand-in module is registered under that name for the run: DWT1DForward / DWT1DInverse for
the haar wavelet with zero padding (J=1), written from the transform's definition
(cA = (a + b)/sqrt 2, cD = (a - b)/sqrt 2 over sample pairs, an odd length padded with one
zero; the inverse interleaves (cA + cD)/sqrt 2, (cA - cD)/sqrt 2).  The goldens therefore pin
everything the reference does around the transform -- the denoised estimate of
StreamPipeline._maybe_dcw (stream.py:1387-1405), the t-modulated scalers, curve resampling to
the band length (_shape_for_wavelet), the band updates, the odd-T trim and the dtype round
trips -- while the haar transform itself stays a restatement.

Usage (from the repository root, with a checkout of the reference):
    python tests/golden/gen_dcw_golden.py /path/to/reference
"""
import json
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


class _DWT1DForward(torch.nn.Module):
    def __init__(self, J=1, mode="zero", wave="haar"):
        super().__init__()
        assert J == 1 and mode == "zero" and wave == "haar"

    def forward(self, x):                       # [N, C, L] -> (cA [N, C, ceil(L/2)], [cD])
        if x.shape[-1] % 2:
            x = torch.nn.functional.pad(x, (0, 1))
        a, b = x[..., 0::2], x[..., 1::2]
        r = 1.0 / math.sqrt(2.0)
        return (a + b) * r, [(a - b) * r]


class _DWT1DInverse(torch.nn.Module):
    def __init__(self, mode="zero", wave="haar"):
        super().__init__()
        assert mode == "zero" and wave == "haar"

    def forward(self, coeffs):
        lo, (hi,) = coeffs[0], coeffs[1]
        r = 1.0 / math.sqrt(2.0)
        out = torch.empty(*lo.shape[:-1], 2 * lo.shape[-1], dtype=lo.dtype, device=lo.device)
        out[..., 0::2] = (lo + hi) * r
        out[..., 1::2] = (lo - hi) * r
        return out


def bits(t):
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy()


def main(ref_root: str):
    stub = types.ModuleType("pytorch_wavelets")
    stub.DWT1DForward, stub.DWT1DInverse = _DWT1DForward, _DWT1DInverse
    sys.modules["pytorch_wavelets"] = stub
    sys.path.insert(0, ref_root)
    from acestep.engine.dcw import DCWCorrector

    g = torch.Generator().manual_seed(2026)
    cases = []
    for T in (150, 123, 10):
        for mode in ("double", "low", "high", "pix"):
            for curve in (False, True):
                for tc in (0.8984375, 0.25):
                    cases.append((T, mode, curve, tc))
    meta, arrs = [], {}
    for i, (T, mode, curve, tc) in enumerate(cases):
        x_next = torch.randn(1, T, 64, generator=g).to(torch.bfloat16)
        x_pre = torch.randn(1, T, 64, generator=g).to(torch.bfloat16)
        vt = torch.randn(1, T, 64, generator=g).to(torch.bfloat16)
        sc = (torch.rand(T, generator=g) * 0.1) if curve else 0.05
        hsc = (torch.rand(T, generator=g) * 0.05) if curve else 0.02
        corr = DCWCorrector(enabled=True, mode=mode, scaler=sc, high_scaler=hsc, wavelet="haar")
        denoised = x_pre - vt * tc                     # StreamPipeline._maybe_dcw
        out = corr.apply(x_next, denoised, tc)
        key = f"c{i}"
        for n, t in (("x_next", x_next), ("x_pre", x_pre), ("vt", vt), ("out", out)):
            arrs[f"{key}/{n}"] = bits(t[0])
        if curve:
            arrs[f"{key}/scaler"] = sc.numpy().astype(np.float32)
            arrs[f"{key}/high_scaler"] = hsc.numpy().astype(np.float32)
        meta.append(dict(key=key, T=T, mode=mode, curve=curve, t_curr=tc,
                         scaler=None if curve else sc, high_scaler=None if curve else hsc))
    (OUT / "dcw_golden.json").write_text(json.dumps({"records": meta}, indent=0))
    np.savez_compressed(OUT / "dcw_golden.npz", **arrs)
    print(f"{len(meta)} records")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_dcw_golden.py <reference checkout>")
    main(sys.argv[1])
