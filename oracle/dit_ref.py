"""CPU restatement of the reference DiT decoder forward.

TEST INFRASTRUCTURE AND CPU BASELINE ONLY: imported by tests/ (as a checker) and by
bench.py's reference arm (as the timed CPU path).  The product (demon_b200) never calls it.

Follows ``AceStepDiTModel.forward`` and ``AceStepDiTLayer.forward``
(acestep/models/modeling_acestep_v15_turbo.py:1310-1514, 484-547), ``AceStepAttention``
(:263-378) on the non-flash path (4-D additive masks from ``create_4d_mask``, :63-137, and
transformers' SDPA attention, which repeats the KV heads whenever a mask is given),
``TimestepEmbedding`` (:207-261), Qwen3RMSNorm / Qwen3MLP and the Qwen3 rotary embedding,
op for op in the same dtype, so that on the CPU it reproduces the reference module's bf16
output bit for bit.  Parity is pinned by tests/test_oracle_dit.py against
tests/golden/dit_small.pt, generated from the reference module itself.

Weights are a plain state dict with the reference's parameter names.  ``fake_quant``
replaces every linear the reference's FP8 export quantises (all but ``time_embed*``,
acestep/engine/trt/fp8_onnx.py:101-104) by the NVFP4 fake-quant of the C oracle:
activation per-row quantise -> dequantise, weight per-tensor quantise -> dequantise,
fp32 matmul, + bias, rounded to bf16.

``lora`` ({linear name: [(A [r, K], B [N, r], strength), ...]}) adds hot LoRA deltas the way
the reference's writeback defines them, ``W + sum_i s_i B_i A_i`` with raw ``B @ A``
(acestep/engine/lora.py:316-319, 824-833): with ``fake_quant`` the base weight stays the
NVFP4 fake-quant of W and the delta ``x (s B A)^T`` is added in fp32 from the bf16 input
(the merged-weight comparison of a hot-LoRA epilogue); without it the bf16 weight is merged
in fp32 and rounded to bf16, as the eager writeback ``param.add_(delta, alpha=s)`` does.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def _fq_weight(W: torch.Tensor) -> torch.Tensor:
    from oracle import nvfp4_oracle as NO
    bits = W.detach().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)
    c, _, sl, g = NO.quantize(bits, NO.GS_DYNAMIC)
    return torch.from_numpy(NO.dequantize(c, sl, g))


class DiTRef:
    def __init__(self, state: dict, cfg: dict, fake_quant: bool = False, lora: dict | None = None):
        self.lora = dict(lora or {})
        if not fake_quant and self.lora:
            state = dict(state)
            for name, entries in self.lora.items():
                W = state[name + ".weight"].double()
                for A, B, s in entries:
                    W = W + s * (B.double() @ A.double())
                state[name + ".weight"] = W.to(state[name + ".weight"].dtype)
        self.sd = state
        self.cfg = dict(cfg)
        self.fake_quant = fake_quant
        self._wq: dict = {}
        c = self.cfg
        self.hd = c.get("head_dim", 128)
        self.eps = c.get("rms_norm_eps", 1e-6)
        self.p = c.get("patch_size", 2)
        self.window = c.get("sliding_window", 128)
        self.n_layers = c["num_hidden_layers"]
        self.inv_freq = 1.0 / (c.get("rope_theta", 1e6) ** (torch.arange(0, self.hd, 2, dtype=torch.int64).float()
                                                            / self.hd))

    # -- primitives --------------------------------------------------------------------
    def linear(self, x, name):
        W = self.sd[name + ".weight"]
        b = self.sd.get(name + ".bias")
        if not self.fake_quant or "time_embed" in name:
            return F.linear(x, W, b)
        from oracle import nvfp4_oracle as NO
        if name not in self._wq:
            self._wq[name] = _fq_weight(W)
        shp = x.shape
        xb = x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous()
        ac, _, asl, ag = NO.quantize(xb.view(torch.int16).numpy().view(np.uint16), NO.GS_PER_ROW)
        y = torch.from_numpy(NO.dequantize(ac, asl, ag)) @ self._wq[name].t()
        for A, B, s in self.lora.get(name, ()):
            y = y + s * ((xb.double() @ A.double().t()) @ B.double().t()).float()
        if b is not None:
            y = y + b.float()
        return y.to(torch.bfloat16).reshape(*shp[:-1], -1)

    def rms(self, x, name):
        w = self.sd[name + ".weight"]
        dt = x.dtype
        h = x.to(torch.float32)
        var = h.pow(2).mean(-1, keepdim=True)
        h = h * torch.rsqrt(var + self.eps)
        return w * h.to(dt)

    @staticmethod
    def mask4d(S, dtype, window):
        i = torch.arange(S)
        diff = i.unsqueeze(1) - i.unsqueeze(0)
        valid = torch.ones((S, S), dtype=torch.bool)
        if window is not None:
            valid = valid & (torch.abs(diff) <= window)
        valid = valid.unsqueeze(0).unsqueeze(0)
        m = torch.full(valid.shape, torch.finfo(dtype).min, dtype=dtype)
        m.masked_fill_(valid, 0.0)
        return m

    def rope(self, S, dtype):
        pos = torch.arange(S)[None]
        inv = self.inv_freq[None, :, None].float().expand(1, -1, 1)
        freqs = (inv.float() @ pos[:, None, :].float()).transpose(1, 2)
        emb = torch.cat((freqs, freqs), dim=-1)
        return (emb.cos() * 1.0).to(dtype), (emb.sin() * 1.0).to(dtype)

    @staticmethod
    def _rot(x):
        x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return torch.cat((-x2, x1), dim=-1)

    def attention(self, x, pre, mask, rope=None, enc=None):
        B, S, _ = x.shape
        hd = self.hd
        q = self.rms(self.linear(x, pre + ".q_proj").view(B, S, -1, hd), pre + ".q_norm").transpose(1, 2)
        src = x if enc is None else enc
        L = src.shape[1]
        k = self.rms(self.linear(src, pre + ".k_proj").view(B, L, -1, hd), pre + ".k_norm").transpose(1, 2)
        v = self.linear(src, pre + ".v_proj").view(B, L, -1, hd).transpose(1, 2)
        if rope is not None:
            cos, sin = rope[0].unsqueeze(1), rope[1].unsqueeze(1)
            q, k = (q * cos) + (self._rot(q) * sin), (k * cos) + (self._rot(k) * sin)
        rep = q.shape[1] // k.shape[1]
        if rep > 1:  # transformers' repeat_kv (a mask is always given on this path)
            k = k[:, :, None].expand(B, k.shape[1], rep, L, hd).reshape(B, -1, L, hd)
            v = v[:, :, None].expand(B, v.shape[1], rep, L, hd).reshape(B, -1, L, hd)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0, scale=hd ** -0.5,
                                           is_causal=False)
        o = o.transpose(1, 2).contiguous().reshape(B, S, -1).contiguous()
        return self.linear(o, pre + ".o_proj")

    def time_embed(self, t, pre):
        half = 128
        tt = t * 1000
        freqs = torch.exp(-math.log(10000) * torch.arange(start=0, end=half, dtype=torch.float32) / half)
        args = tt[:, None].float() * freqs[None]
        emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
        temb = self.linear(F.silu(self.linear(emb.to(t.dtype), pre + ".linear_1")), pre + ".linear_2")
        proj = self.linear(F.silu(temb), pre + ".time_proj").unflatten(1, (6, -1))
        return temb, proj

    # -- forward -----------------------------------------------------------------------
    def layer(self, i, h, tproj, enc, rope, mask_self, mask_enc):
        pre = f"layers.{i}"
        shift, scale, gate, c_shift, c_scale, c_gate = (self.sd[pre + ".scale_shift_table"] + tproj).chunk(6, dim=1)
        n = (self.rms(h, pre + ".self_attn_norm") * (1 + scale) + shift).type_as(h)
        h = (h + self.attention(n, pre + ".self_attn", mask_self, rope=rope) * gate).type_as(h)
        n = self.rms(h, pre + ".cross_attn_norm").type_as(h)
        h = h + self.attention(n, pre + ".cross_attn", mask_enc, enc=enc)
        n = (self.rms(h, pre + ".mlp_norm") * (1 + c_scale) + c_shift).type_as(h)
        ff = self.linear(F.silu(self.linear(n, pre + ".mlp.gate_proj")) * self.linear(n, pre + ".mlp.up_proj"),
                         pre + ".mlp.down_proj")
        return (h + ff * c_gate).type_as(h)

    @torch.no_grad()
    def forward(self, hidden_states, timestep, timestep_r, encoder_hidden_states, context_latents):
        temb_t, proj_t = self.time_embed(timestep, "time_embed")
        temb_r, proj_r = self.time_embed(timestep - timestep_r, "time_embed_r")
        temb, tproj = temb_t + temb_r, proj_t + proj_r
        h = torch.cat([context_latents, hidden_states], dim=-1)
        T = h.shape[1]
        p = self.p
        if T % p:
            h = F.pad(h, (0, 0, 0, p - T % p), mode="constant", value=0)
        h = F.conv1d(h.transpose(1, 2), self.sd["proj_in.1.weight"], self.sd["proj_in.1.bias"], stride=p).transpose(1, 2)
        enc = self.linear(encoder_hidden_states, "condition_embedder")
        S, L = h.shape[1], enc.shape[1]
        dt = h.dtype
        full = self.mask4d(S, dt, None)
        sliding = self.mask4d(S, dt, self.window)
        mask_enc = self.mask4d(max(S, L), dt, None)[:, :, :S, :L]
        rope = self.rope(S, dt)
        for i in range(self.n_layers):
            m = sliding if (i + 1) % 2 else full
            h = self.layer(i, h, tproj, enc, rope, m, mask_enc)
        shift, scale = (self.sd["scale_shift_table"] + temb.unsqueeze(1)).chunk(2, dim=1)
        h = (self.rms(h, "norm_out") * (1 + scale) + shift).type_as(h)
        h = F.conv_transpose1d(h.transpose(1, 2), self.sd["proj_out.1.weight"], self.sd["proj_out.1.bias"],
                               stride=p).transpose(1, 2)
        return h[:, :T, :]
