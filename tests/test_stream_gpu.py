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


def _cfg_requests(dev, n, H, T, L):
    """n standard-CFG requests (a positive and a negative decoder row every step) with
    per-request features: partial denoise from a source, velocity-scale and ode-noise curves,
    a latent mask, cfg_rescale, a per-frame APG momentum."""
    from demon_b200.stream import LatentNoiseMask, SlotCondition, SlotRequest
    g = torch.Generator().manual_seed(6)
    ones = torch.ones(1, L, dtype=torch.bfloat16, device=dev)

    def rnd(*shape):
        return torch.randn(*shape, generator=g).to(torch.bfloat16).to(dev)

    def curve(lo, hi):
        return torch.rand(T, generator=g) * (hi - lo) + lo
    out = []
    for i in range(n):
        kw = dict(neg_conditions=[SlotCondition(rnd(1, L, H), ones)], guidance_curve=curve(3, 7))
        src = rnd(1, T, 64)
        k = i % 4
        if k == 1:
            kw.update(source_latents=src, denoise=0.5, velocity_scale=curve(0.8, 1.2), ode_noise_curve=curve(0, 0.3))
        elif k == 2:
            mask = (torch.arange(T) % 10 < 4).float().to(dev)
            kw.update(latent_mask=LatentNoiseMask(mask=mask, original_latents=src, noise=rnd(1, T, 64)))
        elif k == 3:
            kw.update(cfg_rescale_curve=0.7, apg_momentum=curve(-0.9, -0.5))
        out.append(SlotRequest(encoder_hidden_states=rnd(1, L, H), encoder_attention_mask=ones,
                               context_latents=rnd(1, T, 128), seed=100 + i, **kw))
    return out


def test_stream_equals_batch_banded_gemm_order(cuda):
    """The same bit-identity with every NVFP4 GEMM of the ring's forward in the banded tile
    order of the production tick (A operand > 24 MB): hidden 2048, T = 1500 frames (750
    tokens), 16 standard-CFG slots started on the same tick, so M = 2 x 16 x 750 = 24,000 rows
    per forward, against each request alone at M = 1,500 (plain m-fastest order)."""
    from demon_b200.dit import DemonDiT, DiTConfig
    from demon_b200.stream import StreamConfig, StreamPipeline, generate
    cfgd = DiTConfig(num_hidden_layers=2)
    dec = DemonDiT(cfgd).to(cuda, torch.bfloat16).init_random_(3).eval()
    cfg = StreamConfig(infer_steps=8)
    Tb, Lb, depth = 1500, 32, 16
    reqs = _cfg_requests(cuda, depth, cfgd.hidden_size, Tb, Lb)
    assert 2 * depth * (Tb // 2) * cfgd.hidden_size * 0.5625 > 24e6
    pipe = StreamPipeline(dec, cfg, pipeline_depth=depth, device=cuda, use_graphs=True)
    for r in reqs:
        pipe.submit(r)
    outs = []
    for _ in range(12):
        outs += pipe.tick_many()   # all slots start on tick 0 and finish together, in slot order
    assert len(outs) == depth and pipe.active_slots == 0
    for i, req in enumerate(reqs):
        alone = generate(dec, req, cfg, device=cuda)
        assert torch.isfinite(alone.float()).all(), i
        assert torch.equal(outs[i], alone), f"request {i}: banded stream and batch paths differ"
    assert not torch.equal(outs[0], outs[1])


def test_batched_modulation_equals_per_layer(cuda):
    """The model computes every layer's AdaLN modulation (table + temb, 1 + scale, the shifts)
    in batched ops and hands each layer its slices; a layer that computes its own modulation
    gives the same bits."""
    dec = _decoder(cuda)
    g = torch.Generator(device=cuda).manual_seed(7)
    B, S, H = 2, 15, SMALL["hidden_size"]
    h = torch.randn(B * S, H, generator=g, device=cuda).to(torch.bfloat16)
    tproj = (0.1 * torch.randn(B, 6, H, generator=g, device=cuda)).to(torch.bfloat16)
    enc = torch.randn(B, L, H, generator=g, device=cuda).to(torch.bfloat16)
    kv, Lk = dec.encoder_kv(enc)
    rope = dec._rope(S, cuda, torch.bfloat16)
    mods = torch.stack([l.scale_shift_table[0] for l in dec.layers]).unsqueeze(1) + tproj.unsqueeze(0)
    scales1 = mods[:, :, 1::3] + 1
    shifts = mods[:, :, 0::3].contiguous()
    with torch.no_grad():
        for i, (layer, kv_l) in enumerate(zip(dec.layers, kv)):
            ada = (mods[i, :, 2], mods[i, :, 5], scales1[i, :, 0], scales1[i, :, 1], shifts[i, :, 0], shifts[i, :, 1])
            a = layer(h.clone(), tproj, kv_l, B, S, Lk, rope, ada)
            b = layer(h.clone(), tproj, kv_l, B, S, Lk, rope)
            assert torch.equal(a, b), i
