"""Generate the small-DiT parity fixture from the reference's own AceStepDiTModel.

Run in the build container only (needs the reference checkout):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_dit_fixture.py /path/to/DEMON

Builds ``AceStepDiTModel`` (acestep/models/modeling_acestep_v15_turbo.py:1247-1514) at
the small config in ``dit_weights.SMALL``, loads the seeded weights of
``dit_weights.make_state``, and runs one bf16 forward on the CPU (SDPA attention, the
reference's non-flash mask path) twice:

* ``out_bf16``: the reference as shipped (bf16 ``nn.Linear``);
* ``linears``: input and output of a few of those NVFP4 linears in that run, and
  ``layers``: each DiT layer's input, output, timestep projection and embedded encoder
  states in that run, for teacher-forced checks of single linears and single layers;
* ``out_nvfp4``: every linear the reference's low-precision export quantises (all but
  ``time_embed*``, acestep/engine/trt/fp8_onnx.py:101-104) replaced by the NVFP4
  fake-quant of the oracle: activation per-row quantise -> dequantise, weight
  per-tensor quantise -> dequantise, fp32 matmul, + bias, rounded to bf16.

Writes dit_small.pt (inputs, outputs, key list with shapes) next to this script.
The vector_quantize_pytorch import of the reference's tokenizer module is stubbed;
nothing of it runs in the DiT.
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

from dit_weights import SMALL, make_inputs, make_state  # noqa: E402
from oracle import nvfp4_oracle as NO  # noqa: E402


def _stub_vq():
    m = types.ModuleType("vector_quantize_pytorch")

    class ResidualFSQ(torch.nn.Module):
        def __init__(self, *a, **k):
            super().__init__()
    m.ResidualFSQ = ResidualFSQ
    sys.modules.setdefault("vector_quantize_pytorch", m)


RECORD = ("layers.0.self_attn.q_proj", "layers.0.cross_attn.k_proj", "layers.1.mlp.down_proj",
          "condition_embedder")


def fake_quant_linear(lin: torch.nn.Linear, record: dict | None = None):
    w_bits = lin.weight.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)
    c, _, sl, g = NO.quantize(w_bits, NO.GS_DYNAMIC)
    w_deq = torch.from_numpy(NO.dequantize(c, sl, g))
    bias = None if lin.bias is None else lin.bias.detach().float()

    def forward(x):
        shp = x.shape
        xb = x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous()
        bits = xb.view(torch.int16).numpy().view(np.uint16)
        ac, _, asl, ag = NO.quantize(bits, NO.GS_PER_ROW)
        a = torch.from_numpy(NO.dequantize(ac, asl, ag))
        y = a @ w_deq.t()
        if bias is not None:
            y = y + bias
        y = y.to(torch.bfloat16).reshape(*shp[:-1], -1)
        if record is not None:
            record["x"], record["y"] = x.detach().clone(), y.clone()
        return y
    lin.forward = forward


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    _stub_vq()
    from acestep.models.configuration_acestep_v15 import AceStepConfig
    from acestep.models.modeling_acestep_v15_turbo import AceStepDiTModel

    cfg = AceStepConfig(**SMALL)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    model = AceStepDiTModel(cfg).eval()
    shapes = {k: list(v.shape) for k, v in model.state_dict().items()}
    state = make_state(shapes)
    model.load_state_dict(state)
    inv_freq = model.rotary_emb.inv_freq.clone()
    model = model.to(torch.bfloat16)
    # as from_pretrained(dtype=bf16) leaves it: the rotary angles stay fp32
    model.rotary_emb.inv_freq = inv_freq
    x, ctx, enc, t = make_inputs(SMALL)

    def run():
        with torch.no_grad():
            return model(hidden_states=x, timestep=t, timestep_r=t, attention_mask=None,
                         encoder_hidden_states=enc, encoder_attention_mask=None, context_latents=ctx,
                         use_cache=False, past_key_values=None)[0]
    out_bf16 = run()
    n_q = 0
    records = {}
    for name, mod in model.named_modules():
        if isinstance(mod, torch.nn.Linear) and "time_embed" not in name:
            rec = records.setdefault(name, {}) if name in RECORD else None
            fake_quant_linear(mod, rec)
            n_q += 1
    layers = []

    def pre_hook(mod, args):
        # AceStepDiTLayer is called positionally: (h, rope, temb, mask, pos_ids, cache, out_attn,
        # use_cache, cache_pos, encoder_hidden_states, encoder_mask)  (turbo.py:1462-1476)
        layers.append({"h_in": args[0].detach().clone(), "tproj": args[2].detach().clone(),
                       "enc": args[9].detach().clone()})

    def post_hook(mod, args, out):
        layers[-1]["h_out"] = out[0].detach().clone()
    hooks = [l.register_forward_pre_hook(pre_hook) for l in model.layers]
    hooks += [l.register_forward_hook(post_hook) for l in model.layers]
    out_nvfp4 = run()
    for hk in hooks:
        hk.remove()
    rel = ((out_nvfp4.float() - out_bf16.float()).norm() / out_bf16.float().norm()).item()
    torch.save({"cfg": SMALL, "shapes": shapes, "x": x, "ctx": ctx, "enc": enc, "t": t,
                "out_bf16": out_bf16, "out_nvfp4": out_nvfp4, "n_quantised": n_q, "linears": records,
                "layers": layers,
                "rel_nvfp4_vs_bf16": rel}, HERE / "dit_small.pt")
    print(f"wrote dit_small.pt: {n_q} linears quantised, out {tuple(out_bf16.shape)}, "
          f"rel(nvfp4 vs bf16) = {rel:.4f}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_dit_fixture.py <reference checkout>")
    main(sys.argv[1])
