"""NVFP4 quantised linear: host side of the quantiser / GEMM / LoRA C ABI.

Drop-in for the DiT ``nn.Linear`` call sites of the reference
(acestep/models/modeling_acestep_v15_turbo.py:286-289 q/k/v/o, :34-35 and :538
the Qwen3 MLP gate/up/down): :class:`NVFP4Linear` keeps ``forward(x)`` with
``x [..., K] bf16 -> [..., N] bf16`` and the ``weight`` / ``bias`` state-dict
names, and adds the fused gated-residual epilogue used after ``o_proj`` and
the MLP (turbo.py:525-546) plus a hot LoRA whose strength is a kernel scalar
(the reference's LoRA contract, acestep/engine/lora.py:383-526, without the
weight rewrite of lora.py:811-833).

Every call goes through ``libdemon_b200.so``; there is no PyTorch fallback.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _native as nat


# Bumped whenever a packed weight or a hot-LoRA bank changes; captured CUDA graphs that
# bake in weight / LoRA pointers compare it before replaying.
_GENERATION = [0]


def weights_generation() -> int:
    return _GENERATION[0]


def bump_generation() -> None:
    _GENERATION[0] += 1


@dataclass
class NVFP4Tensor:
    """Packed NVFP4 operand: E2M1 codes, tcgen05-layout E4M3 block scales, fp32 global scale(s)."""
    codes: torch.Tensor   # uint8 [rows, K/2]
    sf: torch.Tensor      # uint8 [sf_bytes(rows, K)]
    gs: torch.Tensor      # float32 [1] or [rows]
    rows: int
    K: int
    per_row: bool = False    # gs holds one scale per row
    per_block: bool = False  # weight: gs holds one scale per 128-row block (fused projections)


def _check_cuda_bf16(x: torch.Tensor, name: str) -> None:
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (demon_b200 has no CPU path)")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {x.dtype}")


def quantize(x: torch.Tensor, gs_mode: int = nat.GS_PER_ROW, gs: torch.Tensor | None = None,
             stream=None) -> NVFP4Tensor:
    """Quantise bf16 ``x [M, K]`` (row stride may exceed K) to NVFP4.

    ``gs_mode``: GS_PER_ROW (default; one global scale per row, so a row's
    codes never depend on the rest of the batch), GS_DYNAMIC (one scale from
    the tensor absmax) or GS_STATIC (``gs`` given, float32 [1]).
    """
    _check_cuda_bf16(x, "x")
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("quantize expects a 2-D tensor with unit stride along K")
    M, K = x.shape
    dev = x.device
    codes = torch.empty((M, K // 2), dtype=torch.uint8, device=dev)
    sf = torch.empty((nat.sf_bytes(M, K),), dtype=torch.uint8, device=dev)
    if gs_mode == nat.GS_STATIC:
        if gs is None or gs.dtype != torch.float32 or gs.numel() != 1 or not gs.is_cuda:
            raise ValueError("GS_STATIC needs gs: float32 [1] CUDA tensor")
        g = gs
    else:
        g = torch.empty((M if gs_mode == nat.GS_PER_ROW else 1,), dtype=torch.float32, device=dev)
    nat.check(nat.load().demon_nvfp4_quantize(
        nat.ptr(x), M, K, x.stride(0), gs_mode, nat.ptr(g), nat.ptr(codes), nat.ptr(sf), nat.stream_ptr(stream)))
    return NVFP4Tensor(codes, sf, g, M, K, per_row=gs_mode == nat.GS_PER_ROW)


def pack_weight(w: torch.Tensor, stream=None) -> NVFP4Tensor:
    """Pack a bf16 weight ``[N, K]`` (torch Linear layout) with one per-tensor global scale.

    Plays the role of the reference's offline weight quantiser
    (acestep/engine/trt/fp8_onnx.py:115-149) for NVFP4.
    """
    return quantize(w.contiguous(), nat.GS_DYNAMIC, stream=stream)


def fuse_weights(parts: list) -> NVFP4Tensor:
    """Concatenate packed weights that read the same activation (q/k/v, MLP gate/up) along N.

    Codes and block scales concatenate as they are (every part has a multiple of 128 rows,
    the scale layout's row block); each part keeps its own per-tensor global scale, given to
    the GEMM as one scale per 128-column block of the fused output.
    """
    K = parts[0].K
    for t in parts:
        if t.K != K or t.rows % 128 or t.per_row or t.per_block or t.gs.numel() != 1:
            raise ValueError("fuse_weights: parts need equal K, rows % 128 == 0 and one global scale each")
    codes = torch.cat([t.codes for t in parts], 0)
    sf = torch.cat([t.sf for t in parts], 0)
    gs = torch.cat([t.gs.expand(t.rows // 128) for t in parts], 0).contiguous()
    return NVFP4Tensor(codes, sf, gs, sum(t.rows for t in parts), K, per_block=True)


def interleave_weights(gate: NVFP4Tensor, up: NVFP4Tensor) -> NVFP4Tensor:
    """Pack MLP gate and up projections for the GEMM's SwiGLU epilogue (``gemm(silu_mul=True)``):
    rows in blocks of 128 alternate gate, up (gate 0..127, up 0..127, gate 128..255, ...), each
    block keeping its part's global scale, so one 256-column tile holds the gate and up values
    of the same 128 output features."""
    K = gate.K
    for t in (gate, up):
        if t.K != K or t.rows != gate.rows or t.rows % 128 or t.per_row or t.per_block or t.gs.numel() != 1:
            raise ValueError("interleave_weights: gate and up need equal shapes, rows % 128 == 0, one scale each")
    nb = gate.rows // 128
    codes = torch.stack([gate.codes.view(nb, 128, K // 2), up.codes.view(nb, 128, K // 2)], 1)
    sf = torch.stack([gate.sf.view(nb, -1), up.sf.view(nb, -1)], 1)
    gs = torch.stack([gate.gs.expand(nb), up.gs.expand(nb)], 1)
    return NVFP4Tensor(codes.reshape(2 * gate.rows, K // 2).contiguous(), sf.reshape(-1).contiguous(),
                       gs.reshape(-1).contiguous(), 2 * gate.rows, K, per_block=True)


def bf16_linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """out = bf16(x @ w^T + bias) on the tensor cores, row by row independent of M.

    x bf16 [M, K] (unit stride along K), w bf16 [N, K], bias bf16 [N] or None.
    """
    _check_cuda_bf16(x, "x")
    _check_cuda_bf16(w, "w")
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("bf16_linear expects a 2-D x with unit stride along K")
    M, K = x.shape
    N = w.shape[0]
    w = w.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    nat.check(nat.load().demon_bf16_linear(nat.ptr(x), M, K, x.stride(0), nat.ptr(w), N, nat.ptr(bias),
                                           nat.ptr(out), out.stride(0), nat.stream_ptr(stream)))
    return out


def lora_down(x: torch.Tensor, lora_a: torch.Tensor, col_scale: torch.Tensor, a: NVFP4Tensor,
              w: NVFP4Tensor, stream=None) -> torch.Tensor:
    """xa = col_scale * (x @ lora_a^T) / (a_gs * w_gs), bf16 [M, r] (tcgen05 bf16 GEMM)."""
    _check_cuda_bf16(x, "x")
    _check_cuda_bf16(lora_a, "lora_a")
    M, K = x.shape
    r = lora_a.shape[0]
    xa = torch.empty((M, r), dtype=torch.bfloat16, device=x.device)
    nat.check(nat.load().demon_lora_down(
        nat.ptr(x), M, K, x.stride(0), nat.ptr(lora_a.contiguous()), r, nat.ptr(col_scale),
        nat.ptr(a.gs), int(a.per_row), nat.ptr(w.gs), nat.ptr(xa), nat.stream_ptr(stream)))
    return xa


def gemm(a: NVFP4Tensor, w: NVFP4Tensor, bias: torch.Tensor | None = None,
         residual: torch.Tensor | None = None, gate: torch.Tensor | None = None, gate_rows: int = 1,
         lora_xa: torch.Tensor | None = None, lora_b: torch.Tensor | None = None,
         out: torch.Tensor | None = None, head_norm: tuple | None = None, rope: tuple | None = None,
         silu_mul: bool = False, stream=None) -> torch.Tensor:
    """out = residual + gate * (alpha * (A W^T + lora) + bias), bf16 [M, N].

    ``silu_mul``: ``w`` from :func:`interleave_weights`; out = bf16(bf16(silu(g)) * u), bf16
    [M, N/2], with g and u the gate / up projections (Qwen3MLP's act_fn(gate) * up).

    ``head_norm = (hn_cols, hn_q_cols, w_q, w_k, eps)``: per-head RMSNorm of the output's
    first hn_cols columns (heads of 128; w_q for the first hn_q_cols, w_k after), and with
    ``rope = (cos, sin, S[, half])`` the rotary embedding after it (q/k projections of the DiT);
    ``half`` promises that the tables' two 64-column halves are equal (the standard
    rotate-half embedding), so that only the first half is read.
    """
    if a.K != w.K:
        raise ValueError(f"K mismatch: activations {a.K} vs weight {w.K}")
    M, N, K = a.rows, w.rows, a.K
    dev = a.codes.device
    if out is None:
        out = torch.empty((M, N // 2 if silu_mul else N), dtype=torch.bfloat16, device=dev)
    args = nat.DemonGemmArgs()
    args.silu_mul = int(bool(silu_mul))
    args.a_codes, args.a_sf, args.a_gs = nat.ptr(a.codes), nat.ptr(a.sf), nat.ptr(a.gs)
    args.a_gs_per_row = int(a.per_row)
    args.w_gs_per_block = int(w.per_block)
    args.w_codes, args.w_sf, args.w_gs = nat.ptr(w.codes), nat.ptr(w.sf), nat.ptr(w.gs)
    args.M, args.N, args.K = M, N, K
    args.out, args.ldo = nat.ptr(out), out.stride(0)
    args.bias = nat.ptr(bias)
    if residual is not None:
        args.residual, args.ldr = nat.ptr(residual), residual.stride(0)
    if gate is not None:
        args.gate, args.gate_rows, args.ld_gate = nat.ptr(gate), gate_rows, gate.stride(0)
    if lora_xa is not None:
        args.lora_xa, args.lora_b, args.lora_rank = nat.ptr(lora_xa), nat.ptr(lora_b), lora_xa.shape[1]
    if head_norm is not None:
        hn_cols, hn_q, wq, wk, eps = head_norm
        for wt in (wq, wk):
            if wt is not None and (wt.dtype != torch.bfloat16 or not wt.is_contiguous()):
                raise ValueError("head-norm weights must be contiguous bf16 [128]")
        args.hn_cols, args.hn_q_cols, args.hn_wq, args.hn_wk = hn_cols, hn_q, nat.ptr(wq), nat.ptr(wk)
        args.hn_eps = float(eps)
        if rope is not None:
            cos, sin, S = rope[:3]
            args.rope_cos, args.rope_sin, args.rope_S = nat.ptr(cos), nat.ptr(sin), int(S)
            args.rope_half = int(len(rope) > 3 and bool(rope[3]))
    nat.check(nat.load().demon_nvfp4_gemm(ctypes.byref(args), nat.stream_ptr(stream)))
    return out


@dataclass
class _LoRAEntry:
    A: torch.Tensor          # bf16 [r, K]  (PEFT lora_A)
    B: torch.Tensor          # bf16 [N, r]  (PEFT lora_B)
    strength: float = 1.0
    enabled: bool = True


@dataclass
class LoRABank:
    """Hot LoRAs of one linear, concatenated along the rank.

    The effective weight is ``W + sum_i s_i B_i A_i`` -- raw ``B @ A`` with no
    alpha / rank factor, exactly the reference's delta
    (acestep/engine/lora.py:316-319) and writeback (lora.py:824-833).  The
    strength of each LoRA is a per-rank-column scale of the down projection,
    so enable / disable / set_strength never touch the packed weight.  A strength change
    between two non-zero values rewrites that LoRA's segment of the device scale vector in
    place (stream-ordered), so captured CUDA graphs stay valid and the change costs one small
    fill at the next tick; adding, removing, enabling or zeroing a LoRA changes the
    concatenated operands and bumps the weights generation.
    """
    entries: dict = field(default_factory=dict)
    _cat: tuple | None = None

    @staticmethod
    def _contributes(e) -> bool:
        return e is not None and e.enabled and e.strength != 0.0

    def _changed(self) -> None:
        self._cat = None
        bump_generation()

    def set(self, lora_id: str, A: torch.Tensor, B: torch.Tensor, strength: float = 1.0) -> None:
        """Register (or replace) a LoRA.  One that contributes nothing (strength 0) leaves the
        concatenated operands, and so the captured graphs, as they are."""
        old = self.entries.get(lora_id)
        new = _LoRAEntry(A.to(torch.bfloat16).contiguous(), B.to(torch.bfloat16).contiguous(), float(strength))
        self.entries[lora_id] = new
        if self._contributes(old) or self._contributes(new):
            self._changed()

    def remove(self, lora_id: str) -> None:
        if self._contributes(self.entries.pop(lora_id, None)):
            self._changed()

    def set_strength(self, lora_id: str, strength: float) -> None:
        e = self.entries[lora_id]
        old, new = e.strength, float(strength)
        e.strength = new
        if old == new or not e.enabled or (old == 0.0 and new == 0.0):
            return
        if self._cat is not None and self._cat[0] is not None and old != 0.0 and new != 0.0:
            off = 0
            for x in self.entries.values():
                if x is e:
                    break
                if x.enabled and x.strength != 0.0:
                    off += x.A.shape[0]
            self._cat[2][off:off + e.A.shape[0]].fill_(new)   # same operands: graphs stay valid
            return
        self._changed()

    def enable(self, lora_id: str, enabled: bool = True) -> None:
        e = self.entries[lora_id]
        was = self._contributes(e)
        e.enabled = enabled
        if was != self._contributes(e):
            self._changed()

    def active(self):
        """(A_cat [R, K], B_cat [N, R], col_scale fp32 [R]) or None when no LoRA contributes."""
        if self._cat is None:
            live = [e for e in self.entries.values() if e.enabled and e.strength != 0.0]
            if not live:
                self._cat = (None,)
            else:
                A = torch.cat([e.A for e in live], 0)
                B = torch.cat([e.B for e in live], 1)
                scale = torch.cat([torch.full((e.A.shape[0],), e.strength, dtype=torch.float32) for e in live])
                r = A.shape[0]
                pad = (-r) % 16
                if pad:
                    A = torch.cat([A, A.new_zeros(pad, A.shape[1])], 0)
                    B = torch.cat([B, B.new_zeros(B.shape[0], pad)], 1)
                    scale = torch.cat([scale, scale.new_zeros(pad)])
                if A.shape[0] > 128:
                    raise ValueError(f"total LoRA rank {A.shape[0]} exceeds 128 for one linear")
                self._cat = (A.contiguous(), B.contiguous(), scale.to(A.device))
        return None if self._cat[0] is None else self._cat


class NVFP4Linear(torch.nn.Module):
    """Drop-in for ``nn.Linear`` backed by the NVFP4 quantiser + tcgen05 GEMM.

    ``weight`` (bf16 [N, K]) and ``bias`` keep their ``nn.Linear`` names; the
    packed operand is rebuilt by :meth:`repack` (done lazily on first forward
    and after ``load_state_dict``).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 keep_weight: bool = True):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = torch.nn.Parameter(
            torch.empty(out_features, in_features, dtype=torch.bfloat16, device=device), requires_grad=False)
        self.bias = (torch.nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16, device=device),
                                        requires_grad=False) if bias else None)
        self.keep_weight = keep_weight
        self.packed: NVFP4Tensor | None = None
        self.lora = LoRABank()

    @classmethod
    def from_linear(cls, lin: torch.nn.Linear, keep_weight: bool = True) -> "NVFP4Linear":
        m = cls(lin.in_features, lin.out_features, lin.bias is not None, device=lin.weight.device,
                keep_weight=keep_weight)
        with torch.no_grad():
            m.weight.copy_(lin.weight.to(torch.bfloat16))
            if lin.bias is not None:
                m.bias.copy_(lin.bias.to(torch.bfloat16))
        return m

    def repack(self) -> None:
        bump_generation()
        self.packed = pack_weight(self.weight.data)
        if not self.keep_weight:
            self.weight.data = torch.empty(0, dtype=torch.bfloat16, device=self.weight.device)

    def _load_from_state_dict(self, *args, **kwargs):
        super()._load_from_state_dict(*args, **kwargs)
        self.packed = None
        bump_generation()

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                out: torch.Tensor | None = None, a: NVFP4Tensor | None = None) -> torch.Tensor:
        """y = x W^T + b (+ hot LoRA), then optionally ``residual + bf16(y * gate)``.

        x: [..., K] bf16.  gate: [B, N] (one row per leading batch index, as the
        AdaLN gates of the DiT, turbo.py:525-546) or None.  residual: like the output.
        The plain call goes through the registered op ``torch.ops.demon_b200.nvfp4_linear``;
        a: ``quantize(x)`` when several linears share the input (q/k/v, gate/up) and
        ``out`` (a preallocated output) take the direct path to the same kernels.
        """
        if self.packed is None:
            self.repack()
        if a is None and out is None:
            lo = self.lora.active()
            A, B, cs = lo if lo is not None else (None, None, None)
            p = self.packed
            return torch.ops.demon_b200.nvfp4_linear(x, p.codes, p.sf, p.gs, self.bias, A, B, 1.0, residual, gate,
                                                     cs)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        if a is None:
            a = quantize(x2)
        lo = self.lora.active()
        xa = lb = None
        if lo is not None:
            A, B, scale = lo
            xa = lora_down(x2, A, scale, a, self.packed)
            lb = B
        res2 = residual.reshape(-1, self.out_features) if residual is not None else None
        gate2 = None
        gate_rows = 1
        if gate is not None:
            gate2 = gate.reshape(-1, self.out_features)
            gate_rows = x2.shape[0] // gate2.shape[0]
        out2 = out.reshape(-1, self.out_features) if out is not None else None
        y = gemm(a, self.packed, bias=self.bias, residual=res2, gate=gate2, gate_rows=gate_rows,
                 lora_xa=xa, lora_b=lb, out=out2)
        return y.reshape(*lead, self.out_features)


# ---------------------------------------------------------------------------
# torch.library op: the torch-op surface of the quantised linear
# ---------------------------------------------------------------------------

@torch.library.custom_op("demon_b200::nvfp4_linear", mutates_args=(), device_types="cuda")
def nvfp4_linear(x: torch.Tensor, w_codes: torch.Tensor, w_sf: torch.Tensor, w_gs: torch.Tensor,
                 bias: torch.Tensor | None = None, lora_A: torch.Tensor | None = None,
                 lora_B: torch.Tensor | None = None, lora_scale: float = 1.0,
                 residual: torch.Tensor | None = None, gate: torch.Tensor | None = None,
                 lora_col_scale: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + gate * (x W^T + bias + lora_scale * (x A^T) B^T)`` with W in NVFP4, as one op.

    The drop-in for the DiT's ``nn.Linear`` call sites (acestep/models/
    modeling_acestep_v15_turbo.py:286-289, 311-345, 377, 538) plus the gated residual after
    o_proj / the MLP (turbo.py:525-546) and the hot LoRA delta ``W + s B @ A``
    (acestep/engine/lora.py:316-319, 824-833) without rewriting W.

    x bf16 [..., K]; w_codes uint8 [N, K/2], w_sf uint8 (tcgen05 scale layout), w_gs fp32 [1]
    (or [N/128], one per 128-row block of a fused pack); bias bf16 [N]; lora_A bf16 [r, K] and
    lora_B bf16 [N, r] (PEFT layout, r % 16 == 0, r <= 128); residual bf16 [..., N]; gate bf16
    [B, N] with B dividing the rows of x (one gate row per sequence); lora_col_scale fp32 [r]
    multiplies lora_scale per rank column (several LoRAs concatenated along the rank, each
    with its strength, updated in place without re-capturing graphs).  CUDA only: there is no
    CPU kernel.  Returns bf16 [..., N].
    """
    K = x.shape[-1]
    N = w_codes.shape[0]
    if w_codes.shape[1] * 2 != K:
        raise ValueError(f"nvfp4_linear: w_codes {tuple(w_codes.shape)} do not match K={K}")
    if w_gs.numel() not in (1, N // 128):
        raise ValueError("nvfp4_linear: w_gs holds one scale, or one per 128-row block")
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or x2.stride(0) % 8:
        x2 = x2.contiguous()
    a = quantize(x2)
    w = NVFP4Tensor(w_codes, w_sf, w_gs, N, K, per_block=w_gs.numel() > 1)
    xa = lb = None
    if lora_A is not None:
        if lora_B is None:
            raise ValueError("nvfp4_linear: lora_A needs lora_B")
        r = lora_A.shape[0]
        scale = (lora_col_scale.float() * lora_scale if lora_col_scale is not None
                 else torch.full((r,), float(lora_scale), dtype=torch.float32, device=x.device))
        xa = lora_down(x2, lora_A, scale, a, w)
        lb = lora_B.contiguous()
    res2 = residual.reshape(-1, N) if residual is not None else None
    gate2, gate_rows = None, 1
    if gate is not None:
        gate2 = gate.reshape(-1, N)
        if x2.shape[0] % gate2.shape[0]:
            raise ValueError("nvfp4_linear: gate rows must divide the rows of x")
        gate_rows = x2.shape[0] // gate2.shape[0]
    y = gemm(a, w, bias=bias, residual=res2, gate=gate2, gate_rows=gate_rows, lora_xa=xa, lora_b=lb)
    return y.reshape(*x.shape[:-1], N)


@nvfp4_linear.register_fake
def _nvfp4_linear_fake(x, w_codes, w_sf, w_gs, bias=None, lora_A=None, lora_B=None, lora_scale=1.0,
                       residual=None, gate=None, lora_col_scale=None):
    return x.new_empty((*x.shape[:-1], w_codes.shape[0]), dtype=torch.bfloat16)
