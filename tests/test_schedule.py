"""Timestep schedule against golden schedules from the reference's own
DiffusionEngine._build_timestep_schedule (tests/golden/gen_schedule_golden.py): the host's
stream.build_schedule and the oracle's restatement, bit for bit in bfloat16."""
import json
from pathlib import Path

import numpy as np
import torch

from demon_b200.stream import build_schedule
from oracle import ode_oracle as OO

GOLD = json.loads((Path(__file__).parent / "golden" / "schedule_golden.json").read_text())["cases"]


def _bits_to_f64(bits):
    return torch.tensor(bits, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).double().numpy()


def test_host_schedule_matches_reference():
    assert len(GOLD) >= 100
    for c in GOLD:
        ref = _bits_to_f64(c["bf16_bits"])
        got = build_schedule(c["steps"], c["shift"], c["denoise"]).double().numpy()
        assert np.array_equal(got, ref), (c["steps"], c["shift"], c["denoise"])


def test_oracle_schedule_matches_reference():
    for c in GOLD:
        ref = _bits_to_f64(c["bf16_bits"])
        assert np.array_equal(OO.schedule(c["steps"], c["shift"], c["denoise"]), ref), (c["steps"], c["shift"])
