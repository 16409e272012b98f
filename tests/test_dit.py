"""The DiT decoder on NVFP4 linears against the reference's AceStepDiTModel.

Fixture ``tests/golden/dit_small.pt`` comes from the reference module itself
(``tests/golden/make_dit_fixture.py``): a 2-layer AceStep-shaped DiT with seeded
weights, run once with bf16 linears and once with every quantised linear replaced by
the oracle's NVFP4 fake-quant.

Tolerances, from measurements on the reference module itself (CPU): NVFP4 is
discontinuous, so a 1-ulp change on 0.1 %-10 % of a layer's input elements moves that
layer's update (output - input) by 1-13 % and the whole 2-layer forward by 5-9 %
(activation codes and block scales flip and propagate).  GPU kernels that sum in another
order cause exactly such 1-ulp differences, so:
* each linear, fed the reference's own activation, is held to the GEMM bar 1e-2;
* each layer, fed the reference's own inputs, to 0.15 on its update and 0.08 overall;
* the whole forward to 0.15.
The row kernels and fused GEMMs are checked exactly in test_rowops_gpu.py.
"""
import sys
from pathlib import Path

import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

from dit_weights import make_state  # noqa: E402

FIX = HERE / "golden" / "dit_small.pt"


def _fixture():
    return torch.load(FIX, weights_only=False)


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


def test_state_dict_names_match_reference():
    from demon_b200.dit import DemonDiT
    d = _fixture()
    ours = {k: list(v.shape) for k, v in DemonDiT(d["cfg"]).state_dict().items()}
    assert ours == d["shapes"]
    assert d["n_quantised"] == 2 * 11 + 1  # 11 linears per layer + condition_embedder


def _model(d, dev):
    from demon_b200.dit import DemonDiT
    m = DemonDiT(d["cfg"])
    m.load_state_dict(make_state(d["shapes"]))
    return m.to(dev, torch.bfloat16).eval()


def _run(m, d, dev):
    with torch.no_grad():
        t = d["t"].to(dev)
        return m(hidden_states=d["x"].to(dev), timestep=t, timestep_r=t, attention_mask=None,
                 encoder_hidden_states=d["enc"].to(dev), encoder_attention_mask=None,
                 context_latents=d["ctx"].to(dev), use_cache=False, past_key_values=None)[0]


@pytest.mark.gpu
def test_dit_layers_teacher_forced(cuda):
    """Each DiT layer fed the reference's own layer input, timestep projection and embedded
    encoder states, against the reference layer's output (fake-quant NVFP4 linears)."""
    from demon_b200 import nvfp4 as Q
    d = _fixture()
    m = _model(d, cuda)
    for i, rec in enumerate(d["layers"]):
        B, S, D = rec["h_in"].shape
        L = rec["enc"].shape[1]
        layer = m.layers[i]
        enc = rec["enc"].to(cuda).reshape(B * L, D).contiguous()
        kv = layer.cross_attn.cross_kv(Q.quantize(enc), enc, B, L)
        with torch.no_grad():
            h = layer(rec["h_in"].to(cuda).reshape(B * S, D).contiguous(), rec["tproj"].to(cuda), kv, B, S, L,
                      m._rope(S, cuda, torch.bfloat16))
        out, ref, hin = h.view(B, S, D).float().cpu(), rec["h_out"].float(), rec["h_in"].float()
        # the layer's update (output - input) carries the error; a 1-ulp input change on 1 %
        # of the elements moves it by 8 % on the reference itself
        upd_err = float((out - ref).norm() / (ref - hin).norm())
        assert upd_err < 0.15, (i, upd_err)
        assert _rel(out, ref) < 0.08, i


@pytest.mark.gpu
def test_dit_nvfp4_linears_teacher_forced(cuda):
    """Each recorded NVFP4 linear, fed the reference's activation, against the oracle's
    fake-quant output of the same call."""
    d = _fixture()
    m = _model(d, cuda)
    for name, rec in d["linears"].items():
        lin = m.get_submodule(name)
        with torch.no_grad():
            y = lin(rec["x"].to(cuda))
        assert _rel(y, rec["y"]) < 1e-2, name


@pytest.mark.gpu
def test_dit_nvfp4_forward_matches_reference_fake_quant(cuda):
    d = _fixture()
    m = _model(d, cuda)
    out = _run(m, d, cuda)
    assert torch.isfinite(out.float()).all()
    assert _rel(out, d["out_nvfp4"]) < 0.15
    # batch invariance: a row's output does not depend on the other rows of the batch
    d1 = {k: (v[:1] if isinstance(v, torch.Tensor) and v.dim() > 0 else v) for k, v in d.items()}
    out1 = _run(m, d1, cuda)
    assert torch.equal(out1, out[:1])


@pytest.mark.gpu
def test_attention_batch_invariant_at_dit_shapes(cuda):
    """The DiT attention (the sm_100a kernel: global, cross and the diagonal band) computes a
    sequence from that sequence alone at the DiT's shapes (750 tokens, GQA 16/8, text 256)."""
    from demon_b200.dit import _attention
    g = torch.Generator(device=cuda).manual_seed(0)
    B, S, L = 6, 750, 256
    q = torch.randn(B, S, 16, 128, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, S, 8, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, S, 8, 128, generator=g, device=cuda).to(torch.bfloat16)
    ke = torch.randn(B, L, 8, 128, generator=g, device=cuda).to(torch.bfloat16)
    ve = torch.randn(B, L, 8, 128, generator=g, device=cuda).to(torch.bfloat16)
    for kk, vv, w in ((k, v, None), (k, v, 128), (ke, ve, None)):
        full = _attention(q, kk, vv, w)
        for b in (0, B - 1):
            one = _attention(q[b:b + 1], kk[b:b + 1], vv[b:b + 1], w)
            assert torch.equal(one[0], full[b]), (w, b)
        # against fp32 math
        i = torch.arange(S, device=cuda)
        Lk = kk.shape[1]
        mask = None if w is None else ((i[:, None] - torch.arange(Lk, device=cuda)[None, :]).abs() <= w)
        ref = torch.nn.functional.scaled_dot_product_attention(
            q[:2].transpose(1, 2).float(), kk[:2].transpose(1, 2).float(), vv[:2].transpose(1, 2).float(),
            attn_mask=mask, enable_gqa=True).transpose(1, 2)
        assert _rel(full[:2], ref) < 1e-2


# ---------------------------------------------------------------------------------------
# Hot LoRA in the decoder (rank 64 on every attention q/k/v/o and MLP
# linear, strength swept, one enable / remove cycle)
# ---------------------------------------------------------------------------------------

def _lora_targets(n_layers):
    out = []
    for i in range(n_layers):
        p = f"layers.{i}"
        out += [f"{p}.self_attn.{n}_proj" for n in "qkvo"]
        out += [f"{p}.cross_attn.{n}_proj" for n in "qkvo"]
        out += [f"{p}.mlp.{n}_proj" for n in ("gate", "up", "down")]
    return out


def _lora_weights(m, rank, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    lora = {}
    for name in _lora_targets(len(m.layers)):
        lin = m.get_submodule(name)
        A = (torch.randn(rank, lin.in_features, generator=g) * std).to(torch.bfloat16)
        B = (torch.randn(lin.out_features, rank, generator=g) * std).to(torch.bfloat16)
        lora[name] = (A, B)
    return lora


@pytest.mark.gpu
def test_dit_hot_lora_layers_match_merged_weights(cuda):
    """Each layer with rank-64 hot LoRAs on all its attention and MLP linears, fed the
    reference's layer inputs, against the oracle layer whose linears add the merged delta
    s * B @ A exactly (lora.py:316-319, 824-833) to the fake-quant NVFP4 base."""
    from demon_b200 import nvfp4 as Q
    from oracle.dit_ref import DiTRef
    d = _fixture()
    m = _model(d, cuda)
    lora = _lora_weights(m, 64, 41, std=0.04)   # a delta well above the layer tolerance
    s = 0.75
    for name, (A, B) in lora.items():
        m.get_submodule(name).lora.set("cfg4", A.to(cuda), B.to(cuda), strength=s)
    ref = DiTRef(make_state(d["shapes"]), d["cfg"], fake_quant=True,
                 lora={n: [(A, B, s)] for n, (A, B) in lora.items()})
    for i, rec in enumerate(d["layers"]):
        B_, S, D = rec["h_in"].shape
        L = rec["enc"].shape[1]
        layer = m.layers[i]
        enc = rec["enc"].to(cuda).reshape(B_ * L, D).contiguous()
        kv = layer.cross_attn.cross_kv(Q.quantize(enc), enc, B_, L)
        with torch.no_grad():
            h = layer(rec["h_in"].to(cuda).reshape(B_ * S, D).contiguous(), rec["tproj"].to(cuda), kv, B_, S, L,
                      m._rope(S, cuda, torch.bfloat16))
        dt = torch.bfloat16
        window = ref.window if (i + 1) % 2 else None
        with torch.no_grad():
            want = ref.layer(i, rec["h_in"], rec["tproj"], rec["enc"], ref.rope(S, dt), ref.mask4d(S, dt, window),
                             ref.mask4d(max(S, L), dt, None)[:, :, :S, :L])
        out, want, hin = h.view(B_, S, D).float().cpu(), want.float(), rec["h_in"].float()
        upd_err = float((out - want).norm() / (want - hin).norm())
        assert upd_err < 0.15, (i, upd_err)
        assert _rel(out, want) < 0.08, i
        # the LoRA moved the layer by more than twice that tolerance
        assert float((want - rec["h_out"].float()).norm() / (rec["h_out"].float() - hin).norm()) > 0.3, i


@pytest.mark.gpu
def test_dit_hot_lora_strength_sweep_and_remove(cuda):
    """Strength 0 is a no-op, every strength change takes effect on the next (graph-replayed)
    forward without a weight rewrite, and removing the LoRAs restores the base bits."""
    from demon_b200.stream import GraphedDecoder
    d = _fixture()
    m = _model(d, cuda)
    g = GraphedDecoder(m)
    base = _run(m, d, cuda)
    assert torch.equal(_run(g, d, cuda), base)
    lora = _lora_weights(m, 64, 43)
    for name, (A, B) in lora.items():
        m.get_submodule(name).lora.set("cfg4", A.to(cuda), B.to(cuda), strength=0.0)
    assert torch.equal(_run(g, d, cuda), base)           # strength 0 contributes nothing
    prev = base
    for s in (0.25, 0.5, 1.0):
        for name in lora:
            m.get_submodule(name).lora.set_strength("cfg4", s)
        eager, graphed = _run(m, d, cuda), _run(g, d, cuda)
        assert torch.equal(graphed, eager), s             # the replayed graph follows the change
        assert not torch.equal(eager, prev), s
        prev = eager
    for name in lora:
        m.get_submodule(name).lora.remove("cfg4")
    assert torch.equal(_run(g, d, cuda), base)
