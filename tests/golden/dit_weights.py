"""Deterministic random weights for the small DiT parity fixture.

Both the fixture generator (which loads them into the reference
``AceStepDiTModel``) and the GPU test (which loads them into
``demon_b200.dit.DemonDiT``) build the state dict from the key list and
shapes stored in the fixture, so the two models see identical bf16 weights
without shipping a checkpoint.  Test infrastructure only.
"""
from __future__ import annotations

import zlib

import torch

# A small AceStep-shaped DiT: every GEMM dimension a multiple of 256 (K) / 128 (N), the
# reference's head_dim 128 with grouped-query heads (2 q / 1 kv), two layers so both a
# sliding-window and a full-attention layer run.
SMALL = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
             num_key_value_heads=1, head_dim=128, rms_norm_eps=1e-6, rope_theta=1_000_000.0, sliding_window=8,
             in_channels=192, audio_acoustic_hidden_dim=64, patch_size=2)


def make_state(shapes: dict, seed: int = 1234) -> dict:
    """Seeded bf16 tensors for every (name -> shape) entry; the draw per tensor
    depends only on its name, so key order does not matter."""
    out = {}
    for name, shape in shapes.items():
        g = torch.Generator().manual_seed(seed * 1_000_003 + zlib.crc32(name.encode()))
        shape = tuple(shape)
        if name.endswith("norm.weight") or name.endswith("norm_out.weight"):
            t = 1.0 + 0.1 * torch.randn(shape, generator=g)
        elif name.endswith("scale_shift_table"):
            t = torch.randn(shape, generator=g) / shape[-1] ** 0.5
        elif name.endswith(".bias"):
            t = 0.02 * torch.randn(shape, generator=g)
        else:
            fan_in = shape[1] * (shape[2] if len(shape) > 2 else 1)
            if "proj_out" in name:  # ConvTranspose1d weight is [in, out, k]
                fan_in = shape[0]
            t = torch.randn(shape, generator=g) / fan_in ** 0.5
        out[name] = t.to(torch.bfloat16)
    return out


def make_inputs(cfg: dict, B: int = 2, T: int = 30, L: int = 12, seed: int = 99):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, cfg["audio_acoustic_hidden_dim"], generator=g).to(torch.bfloat16)
    ctx = torch.randn(B, T, cfg["in_channels"] - cfg["audio_acoustic_hidden_dim"], generator=g).to(torch.bfloat16)
    enc = torch.randn(B, L, cfg["hidden_size"], generator=g).to(torch.bfloat16)
    t = torch.rand(B, generator=g).to(torch.bfloat16)
    return x, ctx, enc, t
