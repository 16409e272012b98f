"""Streaming ring on the NVFP4 DiT: stream output is bit-identical to the batch path.

A depth-4 ring advances requests with different features side by side (CFG, RCFG
initialize / self with APG momentum and cfg_rescale, partial denoise from a source with
per-frame velocity scale and in-kernel ode-noise, latent mask with an x0-target curve,
multi-condition temporal blending); ``stream.generate`` runs each request alone.  Every
decoder row and every ODE slot is computed independently of its batch, so the finished
latents must match bit for bit.
"""
import sys
from pathlib import Path

import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from dit_weights import SMALL, make_state  # noqa: E402

pytestmark = pytest.mark.gpu

T, L = 30, 12


def _decoder(dev):
    from demon_b200.dit import DemonDiT
    m = DemonDiT(SMALL)
    m.load_state_dict(make_state({k: list(v.shape) for k, v in m.state_dict().items()}))
    return m.to(dev, torch.bfloat16).eval()


def _requests(dev):
    from demon_b200.stream import LatentNoiseMask, SlotCondition, SlotRequest
    g = torch.Generator().manual_seed(5)
    H = SMALL["hidden_size"]

    def enc():
        return torch.randn(1, L, H, generator=g).to(torch.bfloat16).to(dev)

    def cond(**kw):
        return SlotCondition(enc(), torch.ones(1, L, dtype=torch.bfloat16, device=dev), **kw)

    def base(seed, **kw):
        c = cond()
        ctx = torch.randn(1, T, 128, generator=g).to(torch.bfloat16).to(dev)
        return SlotRequest(encoder_hidden_states=c.encoder_hidden_states,
                           encoder_attention_mask=c.encoder_attention_mask, context_latents=ctx, seed=seed, **kw)

    def curve(lo, hi):
        return torch.rand(T, generator=g) * (hi - lo) + lo

    src = torch.randn(1, T, 64, generator=g).to(torch.bfloat16).to(dev)
    mask = (torch.arange(T) % 10 < 4).float()
    reqs = [
        base(11),
        base(12, neg_conditions=[cond()], guidance_curve=curve(3, 7), cfg_rescale_curve=0.7),
        base(13, neg_conditions=[cond()], guidance_curve=torch.tensor(4.0), rcfg_mode="initialize",
             apg_momentum=curve(-0.9, -0.5)),
        base(14, guidance_curve=torch.tensor(5.0), rcfg_mode="self"),
        base(15, source_latents=src, denoise=0.5, velocity_scale=curve(0.8, 1.2), ode_noise_curve=curve(0, 0.3)),
        base(16, latent_mask=LatentNoiseMask(mask=mask.to(dev), original_latents=src,
                                             noise=torch.randn(1, T, 64, generator=g).to(torch.bfloat16).to(dev)),
             x0_target=src, x0_target_curve=curve(0, 1), x0_target_gate=0.25),
        base(17, extra_conditions=[cond(temporal_weight=curve(0, 1).reshape(1, T, 1).to(dev))],
             primary_temporal_weight=curve(0, 1).reshape(1, T, 1).to(dev)),
    ]
    return reqs


def _run_stream(dec, cfg, reqs, dev, **kw):
    from demon_b200.stream import StreamPipeline
    pipe = StreamPipeline(dec, cfg, pipeline_depth=4, device=dev, **kw)
    outs = []
    pending = list(reqs)
    for _ in range(200):
        if pending:
            pipe.submit(pending.pop(0))
        r = pipe.tick()
        if r is not None:
            outs.append(r)
        if not pending and pipe.active_slots == 0:
            break
    assert len(outs) == len(reqs)
    assert pipe.stats()["ticks"] > 8
    return outs


def test_stream_equals_batch(cuda):
    from demon_b200.stream import StreamConfig, generate
    dec = _decoder(cuda)
    cfg = StreamConfig(infer_steps=8)
    reqs = _requests(cuda)
    outs = _run_stream(dec, cfg, reqs, cuda)
    for i, req in enumerate(reqs):
        alone = generate(dec, req, cfg, device=cuda)
        assert alone.shape == (1, T, 64)
        assert torch.isfinite(alone.float()).all(), i
        assert torch.equal(outs[i], alone), f"request {i}: stream and batch paths differ"
    # the requests really are different computations
    assert not torch.equal(outs[0], outs[1])


def test_stream_graph_replay_equals_eager(cuda):
    """The CUDA-graph decoder (one graph per batch shape) gives the eager path's bits."""
    from demon_b200.stream import StreamConfig
    dec = _decoder(cuda)
    cfg = StreamConfig(infer_steps=8)
    eager = _run_stream(dec, cfg, _requests(cuda), cuda)
    graphed = _run_stream(dec, cfg, _requests(cuda), cuda, use_graphs=True)
    for i, (a, b) in enumerate(zip(eager, graphed)):
        assert torch.equal(a, b), i
