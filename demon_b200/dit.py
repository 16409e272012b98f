"""ACE-Step v1.5 turbo DiT decoder on NVFP4 linears (B200).

Mirrors ``AceStepDiTModel`` (acestep/models/modeling_acestep_v15_turbo.py:1247-1514)
and ``AceStepDiTLayer`` (:450-547): same module tree and state-dict names
(``layers.{i}.self_attn.q_proj.weight``, ``proj_in.1.weight``, ...), same
``forward`` signature and ``(hidden_states, past_key_values)`` return, so it
drops in as ``engine.decoder`` for ``StreamPipeline._decoder_forward``
(acestep/engine/stream.py:652-663).

Data path of one layer (M = B * S rows of the residual stream ``h``):

* ``demon_adanorm_quantize``: RMSNorm + AdaLN modulation written straight into the
  NVFP4 operand (the normalised bf16 activation is never stored);
* one NVFP4 GEMM for q/k/v (packed weights concatenated, each with its own scale) whose
  epilogue applies q_norm / k_norm and the rotary embedding per 128-column head, attention,
  then the activation quantiser and the o_proj GEMM whose epilogue applies the AdaLN gate
  and residual;
* cross-attention: RMSNorm -> NVFP4 -> q GEMM (q_norm in its epilogue); the encoder K/V
  (k_norm in the epilogue) of all layers come from one quantised copy of the embedded
  encoder states;
* MLP: one GEMM for gate/up with the SwiGLU epilogue, the activation quantiser, down GEMM
  with gate + residual.

Every DiT linear that the reference's low-precision export quantises (all but
``time_embed*``, acestep/engine/trt/fp8_onnx.py:101-104) runs in NVFP4; proj_in,
proj_out and the timestep MLPs stay bf16 on the tensor cores (``demon_bf16_linear``).
Every kernel here computes a row from that row alone, and the attention kernel walks each
sequence's key tiles in a fixed order (no split over the keys), so a sequence's output does
not depend on the batch it is computed in: the streaming ring and a single request give
identical bits.
Hot LoRA on a linear switches that projection to its own GEMM (LoRA ranks of fused
projections do not share one down-projection).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn
from . import nvfp4 as Q
from .attention import attention as _attention_kernel
from .nvfp4 import NVFP4Linear
from .rowops import adanorm_quantize, head_norm_rope, silu_mul_quantize

@dataclass
class DiTConfig:
    """Defaults of the 2B turbo checkpoint (configuration_acestep_v15.py:148-190)."""
    hidden_size: int = 2048
    intermediate_size: int = 6144
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    sliding_window: int = 128
    in_channels: int = 192
    audio_acoustic_hidden_dim: int = 64
    patch_size: int = 2
    encoder_hidden_size: int | None = None   # the reference embeds encoder states from hidden_size

    def __post_init__(self):
        if self.encoder_hidden_size is None:
            self.encoder_hidden_size = self.hidden_size
        if self.head_dim != 128:
            raise ValueError("demon_b200 DiT kernels are built for head_dim 128 (the reference's)")

    def layer_types(self):
        return ["sliding_attention" if (i + 1) % 2 else "full_attention" for i in range(self.num_hidden_layers)]


class RMSNorm(nn.Module):
    """Holds the Qwen3RMSNorm weight; the norm itself runs inside the fused row kernels."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps


def _attention(q, k, v, window: int | None):
    """softmax(q k^T / sqrt(128)) v over the GQA-shared heads, optional bidirectional band
    |i - j| <= window (the attention interface of AceStepAttention.forward, turbo.py:358-372,
    and its sliding-window mask, :110-112).  q [B, S, Hq, 128], k / v [B, L, Hk, 128]
    (strided views of the fused projection outputs are fine); returns [B, S, Hq, 128].

    The sm_100a attention kernel (demon_attention): each (sequence, q-head pair, 128-query
    block) is computed from that sequence alone, over its key tiles in a fixed order, so
    results do not depend on the batch.
    """
    return _attention_kernel(q, k, v, window)


class TimestepEmbedding(nn.Module):
    """turbo.py:207-261; the three linears stay bf16 (the reference never quantises time_embed)."""

    def __init__(self, in_channels: int, dim: int, scale: float = 1000):
        super().__init__()
        self.linear_1 = nn.Linear(in_channels, dim, bias=True)
        self.act1 = nn.SiLU()
        self.linear_2 = nn.Linear(dim, dim, bias=True)
        self.in_channels = in_channels
        self.act2 = nn.SiLU()
        self.time_proj = nn.Linear(dim, dim * 6)
        self.scale = scale

    def _freqs(self, device):
        cache = self.__dict__.setdefault("_freq_cache", {})
        if device not in cache:  # computed on the CPU as the reference does, then kept on the device
            half = self.in_channels // 2
            cache[device] = torch.exp(-math.log(10000) * torch.arange(0, half, dtype=torch.float32) / half).to(device)
        return cache[device]

    def forward(self, t):
        freqs = self._freqs(t.device)
        args = (t * self.scale)[:, None].float() * freqs[None]
        emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(t.dtype)
        temb = Q.bf16_linear(torch.nn.functional.silu(Q.bf16_linear(emb, self.linear_1.weight, self.linear_1.bias)),
                             self.linear_2.weight, self.linear_2.bias)
        proj = Q.bf16_linear(torch.nn.functional.silu(temb), self.time_proj.weight, self.time_proj.bias)
        return temb, proj.unflatten(1, (6, -1))


def _packed(lin: NVFP4Linear) -> Q.NVFP4Tensor:
    if lin.packed is None:
        lin.repack()
    return lin.packed


def _lora(lin: NVFP4Linear, xb: torch.Tensor | None, a: Q.NVFP4Tensor):
    """(lora_xa, lora_b) of the linear's active hot LoRAs, or (None, None)."""
    lo = lin.lora.active()
    if lo is None:
        return None, None
    if xb is None:
        raise RuntimeError("hot LoRA needs the bf16 input of the linear")
    A, B, scale = lo
    return Q.lora_down(xb, A, scale, a, _packed(lin)), B


def _has_lora(*lins) -> bool:
    return any(l.lora.active() is not None for l in lins)


def _gemm_head_norm(a, w, hn, rope, **kw):
    """NVFP4 GEMM whose first ``hn[0]`` output columns get the per-head RMSNorm (+ RoPE) of
    q / k.  The GEMM epilogue does it when the output width is a multiple of 256 (a warp then
    holds whole 128-column heads); otherwise the standalone head-norm kernel runs on the
    output (the same arithmetic)."""
    if hn is None or hn[0] == 0:
        return Q.gemm(a, w, **kw)
    if w.rows % 256 == 0:
        return Q.gemm(a, w, head_norm=hn, rope=rope, **kw)
    y = Q.gemm(a, w, **kw)
    hn_cols, hn_q, wq, wk, eps = hn
    rk = dict(cos=rope[0], sin=rope[1], S=rope[2]) if rope is not None else {}
    if hn_q:
        head_norm_rope(y, 0, hn_q // 128, wq, eps, **rk)
    if hn_cols > hn_q:
        head_norm_rope(y, hn_q, (hn_cols - hn_q) // 128, wk, eps, **rk)
    return y


class Attention(nn.Module):
    """AceStepAttention (turbo.py:263-378) with NVFP4 projections."""

    def __init__(self, cfg: DiTConfig, layer_idx: int, cross: bool = False):
        super().__init__()
        hd = cfg.head_dim
        self.cfg, self.cross, self.head_dim = cfg, cross, hd
        self.hq, self.hk = cfg.num_attention_heads, cfg.num_key_value_heads
        self.q_proj = NVFP4Linear(cfg.hidden_size, self.hq * hd, bias=False)
        self.k_proj = NVFP4Linear(cfg.hidden_size, self.hk * hd, bias=False)
        self.v_proj = NVFP4Linear(cfg.hidden_size, self.hk * hd, bias=False)
        self.o_proj = NVFP4Linear(self.hq * hd, cfg.hidden_size, bias=False)
        self.q_norm = RMSNorm(hd, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(hd, cfg.rms_norm_eps)
        self.window = cfg.sliding_window if (not cross and cfg.layer_types()[layer_idx] == "sliding_attention") \
            else None
        self._fused = None  # packed [q; k; v] (self) or [k; v] (cross)

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._fused = None

    def fused(self):
        if self._fused is None:
            parts = [self.k_proj, self.v_proj] if self.cross else [self.q_proj, self.k_proj, self.v_proj]
            self._fused = Q.fuse_weights([_packed(l) for l in parts])
        return self._fused

    def _norm_spec(self, lin):
        """The head-norm epilogue of one projection: q_norm on q_proj, k_norm on k_proj."""
        eps = self.q_norm.variance_epsilon
        if lin is self.q_proj:
            return (lin.out_features, lin.out_features, self.q_norm.weight, None, eps)
        if lin is self.k_proj:
            return (lin.out_features, 0, None, self.k_norm.weight, eps)
        return None

    def _proj(self, lins, a, xb, rope=None):
        """Columns of the listed projections side by side, q/k heads normalised (and rotated
        with ``rope``) in the GEMM epilogue: one fused GEMM, or one per linear when any has a
        hot LoRA."""
        if not _has_lora(*lins):
            specs = [self._norm_spec(l) for l in lins]
            hn_cols = sum(l.out_features for l, sp in zip(lins, specs) if sp is not None)
            hn_q = sum(l.out_features for l in lins if l is self.q_proj)
            hn = (hn_cols, hn_q, self.q_norm.weight, self.k_norm.weight, self.q_norm.variance_epsilon)
            return _gemm_head_norm(a, self.fused() if len(lins) > 1 else _packed(lins[0]), hn, rope)
        outs = []
        for l in lins:
            xa, lb = _lora(l, xb, a)
            sp = self._norm_spec(l)
            outs.append(_gemm_head_norm(a, _packed(l), sp, rope if sp else None, lora_xa=xa, lora_b=lb))
        return torch.cat(outs, 1)

    def self_attn(self, a, xb, h, gate, B, S, rope):
        hd, hq, hk = self.head_dim, self.hq, self.hk
        cos, sin = rope
        # the tables are cat(freqs, freqs).cos() / .sin() (DemonDiT._rope): equal halves
        qkv = self._proj([self.q_proj, self.k_proj, self.v_proj], a, xb, rope=(cos, sin, S, True))  # [M, (hq+2hk)*hd]
        ld = qkv.stride(0)
        q = qkv.as_strided((B, S, hq, hd), (S * ld, ld, hd, 1))
        k = qkv.as_strided((B, S, hk, hd), (S * ld, ld, hd, 1), hq * hd)
        v = qkv.as_strided((B, S, hk, hd), (S * ld, ld, hd, 1), (hq + hk) * hd)
        o = _attention(q, k, v, self.window).reshape(B * S, hq * hd)
        return self._out(o, h, gate, S)

    def cross_kv(self, enc_a, enc_b, B, L):
        """Encoder K (k_norm applied) and V of this layer: [B*L, 2 * hk * hd]."""
        return self._proj([self.k_proj, self.v_proj], enc_a, enc_b)

    def cross_attn(self, a, xb, h, kv, B, S, L):
        hd, hq, hk = self.head_dim, self.hq, self.hk
        xa, lb = _lora(self.q_proj, xb, a)
        q = _gemm_head_norm(a, _packed(self.q_proj), self._norm_spec(self.q_proj), None, lora_xa=xa, lora_b=lb)
        ld = kv.stride(0)
        k = kv.as_strided((B, L, hk, hd), (L * ld, ld, hd, 1))
        v = kv.as_strided((B, L, hk, hd), (L * ld, ld, hd, 1), hk * hd)
        o = _attention(q.view(B, S, hq, hd), k, v, None).reshape(B * S, hq * hd)
        return self._out(o, h, None, S)

    def _out(self, o, h, gate, S):
        oa = Q.quantize(o)
        xa, lb = _lora(self.o_proj, o, oa)
        return Q.gemm(oa, _packed(self.o_proj), residual=h, gate=gate, gate_rows=S, lora_xa=xa, lora_b=lb)


class MLP(nn.Module):
    """Qwen3MLP: down(silu(gate(x)) * up(x)), no biases."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.F = cfg.intermediate_size
        self.gate_proj = NVFP4Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = NVFP4Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = NVFP4Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)
        self._fused = None

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._fused = None

    def forward(self, a, xb, h, gate, S):
        down_lora = self.down_proj.lora.active() is not None
        if not _has_lora(self.gate_proj, self.up_proj):
            # one GEMM for gate and up (interleaved 128-row blocks) whose epilogue applies
            # silu(g) * u; h is then quantised for down_proj like any activation
            if self._fused is None:
                self._fused = Q.interleave_weights(_packed(self.gate_proj), _packed(self.up_proj))
            hb = Q.gemm(a, self._fused, silu_mul=True)
            ha = Q.quantize(hb)
        else:
            M = a.rows
            gu = torch.empty((M, 2 * self.F), dtype=torch.bfloat16, device=h.device)
            for i, l in enumerate((self.gate_proj, self.up_proj)):
                xa, lb = _lora(l, xb, a)
                Q.gemm(a, _packed(l), lora_xa=xa, lora_b=lb, out=gu[:, i * self.F:(i + 1) * self.F])
            hb = torch.empty((M, self.F), dtype=torch.bfloat16, device=h.device) if down_lora else None
            ha = silu_mul_quantize(gu, self.F, y=hb)
        xa = lb = None
        if down_lora:
            xa, lb = _lora(self.down_proj, hb, ha)
        return Q.gemm(ha, _packed(self.down_proj), residual=h, gate=gate, gate_rows=S, lora_xa=xa, lora_b=lb)


class DiTLayer(nn.Module):
    """AceStepDiTLayer (turbo.py:450-547)."""

    def __init__(self, cfg: DiTConfig, layer_idx: int):
        super().__init__()
        eps = cfg.rms_norm_eps
        self.eps = eps
        self.self_attn_norm = RMSNorm(cfg.hidden_size, eps)
        self.self_attn = Attention(cfg, layer_idx)
        self.cross_attn_norm = RMSNorm(cfg.hidden_size, eps)
        self.cross_attn = Attention(cfg, layer_idx, cross=True)
        self.mlp_norm = RMSNorm(cfg.hidden_size, eps)
        self.mlp = MLP(cfg)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, cfg.hidden_size) / cfg.hidden_size ** 0.5)

    def forward(self, h, tproj, kv, B, S, L, rope, ada=None):
        """``ada``: this layer's (gate, c_gate, 1 + scale, 1 + c_scale, shift, c_shift) when the
        model computed every layer's modulation at once (the same bf16 operations)."""
        if ada is None:
            # (shift, scale, gate, c_shift, c_scale, c_gate) = (table + temb).chunk(6, dim=1)  (turbo.py:503-505)
            mod = self.scale_shift_table + tproj                      # [B, 6, D] bf16
            shift, scale, gate, c_shift, c_scale, c_gate = mod.unbind(1)
            scale1, c_scale1 = 1 + scale, 1 + c_scale                 # bf16, as the reference's (1 + scale)
            shift, c_shift = shift.contiguous(), c_shift.contiguous()
        else:
            gate, c_gate, scale1, c_scale1, shift, c_shift = ada
        sa = self.self_attn
        xb = torch.empty_like(h) if _has_lora(sa.q_proj, sa.k_proj, sa.v_proj) else None
        a = adanorm_quantize(h, self.self_attn_norm.weight, self.eps, scale1, shift, S, y=xb)
        h = sa.self_attn(a, xb, h, gate, B, S, rope)
        ca = self.cross_attn
        xb = torch.empty_like(h) if _has_lora(ca.q_proj) else None
        a = adanorm_quantize(h, self.cross_attn_norm.weight, self.eps, y=xb)
        h = ca.cross_attn(a, xb, h, kv, B, S, L)
        mlp = self.mlp
        xb = torch.empty_like(h) if _has_lora(mlp.gate_proj, mlp.up_proj) else None
        a = adanorm_quantize(h, self.mlp_norm.weight, self.eps, c_scale1, c_shift, S, y=xb)
        return mlp(a, xb, h, c_gate, S)


class DemonDiT(nn.Module):
    """AceStepDiTModel with NVFP4 linears.  ``forward`` keeps the reference signature."""

    def __init__(self, cfg: "DiTConfig | dict | None" = None):
        super().__init__()
        if isinstance(cfg, dict):
            cfg = DiTConfig(**{k: v for k, v in cfg.items() if k in DiTConfig.__dataclass_fields__})
        cfg = cfg or DiTConfig()
        self.cfg = cfg
        d = cfg.hidden_size
        self.layers = nn.ModuleList([DiTLayer(cfg, i) for i in range(cfg.num_hidden_layers)])
        self.proj_in = nn.Sequential(nn.Identity(), nn.Conv1d(cfg.in_channels, d, cfg.patch_size, cfg.patch_size),
                                     nn.Identity())
        self.time_embed = TimestepEmbedding(256, d)
        self.time_embed_r = TimestepEmbedding(256, d)
        self.condition_embedder = NVFP4Linear(cfg.encoder_hidden_size, d, bias=True)
        self.norm_out = RMSNorm(d, cfg.rms_norm_eps)
        self.proj_out = nn.Sequential(nn.Identity(),
                                      nn.ConvTranspose1d(d, cfg.audio_acoustic_hidden_dim, cfg.patch_size,
                                                         cfg.patch_size), nn.Identity())
        self.scale_shift_table = nn.Parameter(torch.randn(1, 2, d) / d ** 0.5)
        # kept out of the module's buffers so that ``.to(torch.bfloat16)`` leaves it fp32, as the
        # reference's rotary embedding computes its angles in fp32 (Qwen3RotaryEmbedding)
        self._inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, dtype=torch.int64).float()
                                                   / cfg.head_dim))
        self._rope_cache: dict = {}
        self._conv_cache = None

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self._conv_cache = None
        Q.bump_generation()

    def _rope(self, S, device, dtype):
        key = (S, device, dtype)
        if key not in self._rope_cache:
            pos = torch.arange(S, device=device, dtype=torch.float32)
            freqs = pos[:, None] * self._inv_freq.to(device)[None, :]
            emb = torch.cat((freqs, freqs), dim=-1)
            self._rope_cache[key] = (emb.cos().to(dtype).contiguous(), emb.sin().to(dtype).contiguous())
        return self._rope_cache[key]

    def _convs(self):
        """proj_in / proj_out as linears over patches: Conv1d(k = stride = p) weight [D, C, p]
        -> [D, C * p] (patch feature index c * p + j); ConvTranspose1d weight [D, O, p] ->
        [O * p, D] with bias repeated per tap (one rounding, bias included)."""
        if self._conv_cache is None:
            ci, co = self.proj_in[1], self.proj_out[1]
            p = self.cfg.patch_size
            w_in = ci.weight.detach().reshape(ci.out_channels, -1).contiguous()
            w_out = co.weight.detach().reshape(co.in_channels, -1).t().contiguous()
            b_out = co.bias.detach().repeat_interleave(p).contiguous()
            self._conv_cache = (w_in, ci.bias.detach(), w_out, b_out)
        return self._conv_cache

    @torch.no_grad()
    def init_random_(self, seed: int = 0) -> "DemonDiT":
        """Seeded random weights (there are no checkpoints offline): N(0, 1/fan_in) linears and
        convolutions, norms 1, AdaLN tables N(0, 1/D), biases 0.  Drawn on the parameters'
        device (same seed and device type -> same weights)."""
        dev = next(self.parameters()).device
        g = torch.Generator(device=dev).manual_seed(seed)
        for name, p in self.named_parameters():
            shape = p.shape
            if name.endswith("norm.weight") or name.endswith("norm_out.weight"):
                p.data.fill_(1.0)
                continue
            if name.endswith(".bias"):
                p.data.zero_()
                continue
            if name.endswith("scale_shift_table"):
                std = 1.0 / shape[-1] ** 0.5
            else:
                fan_in = shape[0] if "proj_out" in name else shape[1] * (shape[2] if len(shape) > 2 else 1)
                std = 1.0 / fan_in ** 0.5
            p.data.copy_((torch.randn(shape, generator=g, device=dev) * std).to(p.dtype))
        for m in self.modules():
            if isinstance(m, NVFP4Linear):
                m.packed = None
            if isinstance(m, (Attention, MLP)):
                m._fused = None
        self._conv_cache = None
        Q.bump_generation()
        return self

    def encoder_kv(self, encoder_hidden_states):
        """condition_embedder and every layer's cross-attention K/V for encoder states [B, L, E]."""
        B, L, E = encoder_hidden_states.shape
        e2 = encoder_hidden_states.reshape(B * L, E).contiguous()
        ea = Q.quantize(e2)
        xa, lb = _lora(self.condition_embedder, e2, ea)
        enc = Q.gemm(ea, _packed(self.condition_embedder), bias=self.condition_embedder.bias, lora_xa=xa,
                     lora_b=lb)
        enc_a = Q.quantize(enc)
        return [layer.cross_attn.cross_kv(enc_a, enc, B, L) for layer in self.layers], L

    def forward(self, hidden_states, timestep, timestep_r, attention_mask=None, encoder_hidden_states=None,
                encoder_attention_mask=None, context_latents=None, use_cache=False, past_key_values=None,
                encoder_kv=None, **kw):
        """turbo.py:1310-1514.  ``encoder_kv``: the result of :meth:`encoder_kv` for these encoder
        states, to skip recomputing the cross-attention K/V (they depend on the condition only)."""
        cfg = self.cfg
        temb_t, proj_t = self.time_embed(timestep)
        temb_r, proj_r = self.time_embed_r(timestep - timestep_r)
        temb, tproj = temb_t + temb_r, proj_t + proj_r
        h = torch.cat([context_latents, hidden_states], dim=-1)
        T = h.shape[1]
        p = cfg.patch_size
        if T % p:
            h = torch.nn.functional.pad(h, (0, 0, 0, p - T % p))
        B, Tp, C = h.shape
        S = Tp // p
        w_in, b_in, w_out, b_out = self._convs()
        patches = h.view(B, S, p, C).transpose(2, 3).reshape(B * S, C * p)
        h = Q.bf16_linear(patches, w_in, b_in)                                    # [B*S, D]
        kv, L = encoder_kv if encoder_kv is not None else self.encoder_kv(encoder_hidden_states)
        rope = self._rope(S, h.device, h.dtype)
        # every layer's AdaLN modulation in three batched ops instead of five small ones per layer:
        # table + temb ([layers, B, 6, D] bf16), 1 + scale / 1 + c_scale, and the two shifts
        mods = torch.stack([l.scale_shift_table[0] for l in self.layers]).unsqueeze(1) + tproj.unsqueeze(0)
        scales1 = mods[:, :, 1::3] + 1                            # [layers, B, 2, D]: 1 + scale, 1 + c_scale
        shifts = mods[:, :, 0::3].contiguous()                    # [layers, B, 2, D]: shift, c_shift
        for i, (layer, kv_l) in enumerate(zip(self.layers, kv)):
            ada = (mods[i, :, 2], mods[i, :, 5], scales1[i, :, 0], scales1[i, :, 1], shifts[i, :, 0], shifts[i, :, 1])
            h = layer(h, tproj, kv_l, B, S, L, rope, ada)
        shift, scale = (self.scale_shift_table + temb.unsqueeze(1)).unbind(1)
        y = torch.empty_like(h)
        adanorm_quantize(h, self.norm_out.weight, self.norm_out.variance_epsilon, 1 + scale, shift.contiguous(), S,
                         quantize=False, y=y)
        o = Q.bf16_linear(y, w_out, b_out)                                        # [B*S, O*p]
        o = o.view(B, S, -1, p).transpose(2, 3).reshape(B, S * p, -1)
        return o[:, :T, :], past_key_values
