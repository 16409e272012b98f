"""Generate golden timestep schedules from the reference's own DiffusionEngine.

Run in the build container only (needs the reference checkout):

    PYTHONPATH=/path/to/DEMON PYTHONDONTWRITEBYTECODE=1 python tests/golden/gen_schedule_golden.py /path/to/DEMON

Calls acestep.engine.diffusion.DiffusionEngine._build_timestep_schedule (diffusion.py:656-699)
on the CPU in bfloat16, the dtype StreamPipeline evaluates it in (stream.py:385-396; the CPU and
CUDA bf16 results agree bit for bit on B200), over a grid of step counts, shifts and denoise
strengths, and writes schedule_golden.json next to this script: one record per case with the
schedule as bf16 bit patterns.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
STEPS = (1, 2, 4, 8, 12, 20, 50)
SHIFTS = (1.0, 2.0, 3.0, 5.0)
DENOISE = (1.0, 0.75, 0.5, 0.3, 0.1, 1e-7)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from acestep.engine.diffusion import DiffusionConfig, DiffusionEngine

    class _Engine:  # the method reads only the class constant _DENOISE_MIN
        _DENOISE_MIN = DiffusionEngine._DENOISE_MIN

    cases = []
    for steps in STEPS:
        for shift in SHIFTS:
            for dn in DENOISE:
                cfg = DiffusionConfig(infer_steps=steps, shift=shift, denoise=dn)
                t = DiffusionEngine._build_timestep_schedule(_Engine(), cfg, torch.device("cpu"), torch.bfloat16)
                bits = t.view(torch.int16).to(torch.int32).bitwise_and(0xFFFF).tolist()
                cases.append({"steps": steps, "shift": shift, "denoise": dn, "bf16_bits": bits})
    (HERE / "schedule_golden.json").write_text(json.dumps({"cases": cases}) + "\n")
    print(f"{len(cases)} schedules")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_schedule_golden.py <reference checkout>")
    main(sys.argv[1])
