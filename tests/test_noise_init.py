"""A slot's initial noise against golden draws from the reference's own
StreamPipeline._make_noise (tests/golden/gen_noise_golden.py): int seeds and per-row seed
lists (a negative entry keeps the generator's state), bit for bit in bfloat16."""
import json
from pathlib import Path

import torch

from demon_b200.stream import StreamPipeline

GOLD = json.loads((Path(__file__).parent / "golden" / "noise_golden.json").read_text())["cases"]


def test_initial_noise_matches_reference():
    assert len(GOLD) >= 8
    for c in GOLD:
        torch.manual_seed(99)  # the generator state the golden run had before each draw
        got = StreamPipeline.noise_host(c["seed"], c["T"], c["D"])
        ref = torch.tensor(c["bf16_bits"], dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
        assert torch.equal(got.reshape(-1).view(torch.int16), ref.view(torch.int16)), c["seed"]
