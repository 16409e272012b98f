"""Generate golden initial-noise draws from the reference's own StreamPipeline._make_noise.

Run in the build container only (needs the reference checkout):

    PYTHONPATH=/path/to/DEMON PYTHONDONTWRITEBYTECODE=1 python tests/golden/gen_noise_golden.py /path/to/DEMON

Calls acestep.engine.stream.StreamPipeline._make_noise (stream.py:403-451) with noise_on_cpu
(its default) on a minimal pipeline stand-in (CPU device, bfloat16) for int seeds and
per-row seed lists, and writes noise_golden.json next to this script (bf16 bit patterns).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

HERE = Path(__file__).resolve().parent
T, D = 24, 64
SEEDS = [0, 1, 1234, 2**31 - 1, [7], [5, 9], [-1, 3], [11, -1]]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from acestep.engine import stream as S

    pipe = SimpleNamespace(config=SimpleNamespace(noise_on_cpu=True), _device=torch.device("cpu"),
                           _dtype=torch.bfloat16)
    cases = []
    for seed in SEEDS:
        torch.manual_seed(99)  # the state a negative list entry keeps
        req = SimpleNamespace(context_latents=torch.zeros(1, T, 2 * D), seed=seed)
        n = S.StreamPipeline._make_noise(pipe, req)
        first = n[0].contiguous()
        bits = first.view(torch.int16).to(torch.int32).bitwise_and(0xFFFF).reshape(-1).tolist()
        cases.append({"seed": seed, "T": T, "D": D, "bf16_bits": bits})
    (HERE / "noise_golden.json").write_text(json.dumps({"cases": cases}) + "\n")
    print(f"{len(cases)} draws")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/gen_noise_golden.py <reference checkout>")
    main(sys.argv[1])
