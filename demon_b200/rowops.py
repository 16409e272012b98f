"""Host side of the DiT row kernels (``demon_adanorm_quantize``, ``demon_silu_mul_quantize``,
``demon_head_norm_rope`` in include/demon_b200.h).

Each returns the NVFP4 operand of the GEMM that follows (or updates its input in place);
rows are computed independently of the batch, so a slot's values never depend on which
other slots share the forward.  No PyTorch fallback: every call goes to libdemon_b200.so.
"""
from __future__ import annotations

import torch

from . import _native as nat
from .nvfp4 import NVFP4Tensor, _check_cuda_bf16


def _alloc_q(M: int, K: int, dev) -> NVFP4Tensor:
    return NVFP4Tensor(torch.empty((M, K // 2), dtype=torch.uint8, device=dev),
                       torch.empty((nat.sf_bytes(M, K),), dtype=torch.uint8, device=dev),
                       torch.empty((M,), dtype=torch.float32, device=dev), M, K, per_row=True)


def adanorm_quantize(x: torch.Tensor, norm_w: torch.Tensor, eps: float, scale1: torch.Tensor | None = None,
                     shift: torch.Tensor | None = None, rows_per_mod: int = 1, quantize: bool = True,
                     y: torch.Tensor | None = None, stream=None):
    """RMSNorm (+ AdaLN ``* (1 + scale) + shift``) of ``x [M, D]`` into an NVFP4 operand.

    ``scale1`` / ``shift``: bf16 [B, D] with ``rows_per_mod`` rows of x per entry (the
    sequence length).  Returns the NVFP4Tensor (``quantize``) and/or writes bf16 ``y``.
    """
    _check_cuda_bf16(x, "x")
    _check_cuda_bf16(norm_w, "norm_w")
    M, D = x.shape
    q = _alloc_q(M, D, x.device) if quantize else None
    mods = [t for t in (scale1, shift) if t is not None]
    for t in mods:
        _check_cuda_bf16(t, "modulation")
    for t in mods:
        # row m uses modulation row m // rows_per_mod: every such row must exist
        if t.dim() != 2 or t.shape[1] < D or rows_per_mod < 1 or t.shape[0] * rows_per_mod < M:
            raise ValueError(f"modulation {tuple(t.shape)} must be [ceil(M / rows_per_mod), >= D] "
                             f"for M={M}, D={D}, rows_per_mod={rows_per_mod}")
    multi = [t for t in mods if t.shape[0] > 1]   # a single row's stride is irrelevant
    ld_mod = multi[0].stride(0) if multi else (D if mods else 0)
    if any(t.stride(1) != 1 for t in mods) or any(t.stride(0) != ld_mod for t in multi):
        raise ValueError("scale1 and shift need the same row stride and unit column stride")
    nat.check(nat.load().demon_adanorm_quantize(
        nat.ptr(x), M, D, x.stride(0), nat.ptr(norm_w), nat.ptr(scale1), nat.ptr(shift), rows_per_mod, ld_mod,
        float(eps), nat.ptr(q.gs if q else None), nat.ptr(q.codes if q else None), nat.ptr(q.sf if q else None),
        nat.ptr(y), y.stride(0) if y is not None else 0, nat.stream_ptr(stream)))
    return q


def silu_mul_quantize(gu: torch.Tensor, F: int, y: torch.Tensor | None = None, stream=None) -> NVFP4Tensor:
    """NVFP4 of h = bf16(bf16(silu(gu[:, :F])) * gu[:, F:2F]) per row; ``y`` (bf16 [M, F],
    unit column stride) also receives h."""
    _check_cuda_bf16(gu, "gu")
    M = gu.shape[0]
    if y is not None:
        _check_cuda_bf16(y, "y")
        if y.shape[0] != M or y.shape[1] < F or y.stride(1) != 1:
            raise ValueError("silu_mul_quantize: y must be [M, >= F] with unit column stride")
    q = _alloc_q(M, F, gu.device)
    nat.check(nat.load().demon_silu_mul_quantize(nat.ptr(gu), M, F, gu.stride(0), nat.ptr(q.gs), nat.ptr(q.codes),
                                                 nat.ptr(q.sf), nat.ptr(y), y.stride(0) if y is not None else 0,
                                                 nat.stream_ptr(stream)))
    return q


def head_norm_rope(x: torch.Tensor, col0: int, heads: int, w: torch.Tensor, eps: float,
                   cos: torch.Tensor | None = None, sin: torch.Tensor | None = None, S: int = 1,
                   stream=None) -> None:
    """In place: per-head RMSNorm (weight ``w`` [128]) of ``heads`` heads starting at column
    ``col0`` of ``x [M, ld]``, then the rotary embedding when ``cos`` / ``sin`` [S, 128] are given."""
    _check_cuda_bf16(x, "x")
    M = x.shape[0]
    nat.check(nat.load().demon_head_norm_rope(nat.ptr(x), M, x.stride(0), col0, heads, nat.ptr(w), nat.ptr(cos),
                                              nat.ptr(sin), S, float(eps), nat.stream_ptr(stream)))
