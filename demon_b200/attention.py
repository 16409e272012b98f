"""Host side of the DiT attention kernel (``demon_attention`` in include/demon_b200.h).

``attention(q, k, v, window)`` is the attention core of AceStepAttention.forward
(acestep/models/modeling_acestep_v15_turbo.py:358-372): softmax(q k^T / sqrt(128)) v over the
GQA-shared K / V heads, bidirectional, optionally restricted to the band |i - j| <= window
(the sliding-window mask of lines 110-112 of the same file).  q / k / v are read through their
strides (the q / k / v column ranges of one fused projection output work as they are); the
result is a new contiguous [B, S, Hq, 128] tensor.  No PyTorch fallback: every call goes to
libdemon_b200.so.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

HEAD_DIM = 128


def _check(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda or t.dtype != torch.bfloat16 or t.dim() != 4:
        raise ValueError(f"{name} must be a 4-D bf16 CUDA tensor [B, rows, heads, 128]")
    if t.shape[3] != HEAD_DIM or t.stride(3) != 1 or (t.shape[2] > 1 and t.stride(2) != HEAD_DIM):
        raise ValueError(f"{name}: head_dim must be 128 with heads contiguous within a row "
                         f"(shape {tuple(t.shape)}, strides {t.stride()})")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int | None = None,
              scale: float | None = None, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """q [B, S, Hq, 128], k / v [B, L, Hk, 128] (bf16, Hq / Hk even) -> o [B, S, Hq, 128]."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check(t, n)
    B, S, Hq, _ = q.shape
    L, Hk = k.shape[1], k.shape[2]
    if tuple(v.shape) != tuple(k.shape) or k.shape[0] != B:
        raise ValueError(f"k {tuple(k.shape)} / v {tuple(v.shape)} do not match q {tuple(q.shape)}")
    if out is None:
        out = torch.empty(B, S, Hq, HEAD_DIM, dtype=torch.bfloat16, device=q.device)
    else:
        _check(out, "out")
        if tuple(out.shape) != (B, S, Hq, HEAD_DIM):
            raise ValueError(f"out must be [B, S, Hq, 128], got {tuple(out.shape)}")
    a = nat.DemonAttnArgs(
        q=nat.ptr(q), ldq=q.stride(1), sq=q.stride(0),
        k=nat.ptr(k), ldk=k.stride(1), sk=k.stride(0),
        v=nat.ptr(v), ldv=v.stride(1), sv=v.stride(0),
        o=nat.ptr(out), ldo=out.stride(1), so=out.stride(0),
        B=B, S=S, L=L, Hq=Hq, Hk=Hk, head_dim=HEAD_DIM, window=-1 if window is None else int(window),
        scale=float(HEAD_DIM ** -0.5 if scale is None else scale))
    nat.check(nat.load().demon_attention(ctypes.byref(a), nat.stream_ptr(stream)))
    return out
