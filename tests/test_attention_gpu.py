"""GPU parity of the sm_100a attention kernel (``demon_attention``) against an fp32 reference.

The reference is the attention of AceStepAttention.forward restated in fp32 PyTorch
(acestep/models/modeling_acestep_v15_turbo.py:358-372 and its bidirectional band |i - j| <=
window, lines 110-112): scores q k^T / sqrt(128) over the GQA-shared heads, -inf outside the
band, softmax, times v.  The kernel rounds the probabilities to bf16 before the P V product
(as FlashAttention and cuDNN do) and its output to bf16, so the bar is a relative Frobenius
error of at most 1e-2 per case (observed a few 1e-3) and no element off by more than 2 % of
the largest output magnitude.  Cases: the DiT's sliding-window (128) and global self-attention
and its cross attention over 256 encoder rows, sequence lengths that are not multiples of 128,
a single short block, strided q / k / v views of one fused projection output, and logits
large enough to exercise the lazy rescaling of the running maximum.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 1e-2
MAX_ABS_FRAC = 2e-2


def reference(q, k, v, window):
    """fp32 attention: q [B, S, Hq, D], k / v [B, L, Hk, D] -> [B, S, Hq, D]."""
    B, S, Hq, D = q.shape
    L, Hk = k.shape[1], k.shape[2]
    G = Hq // Hk
    qf = q.float().transpose(1, 2)                                   # [B, Hq, S, D]
    kf = k.float().transpose(1, 2).repeat_interleave(G, dim=1)       # [B, Hq, L, D]
    vf = v.float().transpose(1, 2).repeat_interleave(G, dim=1)
    s = qf @ kf.transpose(-1, -2) * D ** -0.5
    if window is not None:
        i = torch.arange(S, device=q.device)[:, None]
        j = torch.arange(L, device=q.device)[None, :]
        s = s.masked_fill((i - j).abs() > window, float("-inf"))
    return (s.softmax(-1) @ vf).transpose(1, 2)


def check(o, ref, label):
    err = float((o.float() - ref).norm() / ref.norm())
    mx = float((o.float() - ref).abs().max() / ref.abs().max())
    assert torch.isfinite(o).all(), label
    assert err <= REL_FRO_TOL and mx <= MAX_ABS_FRAC, f"{label}: rel Frobenius {err:.2e}, max {mx:.2e}"
    return err


def fused_qkv(B, S, hq, hk, g, dev, scale=1.0):
    """q / k / v as strided views of one [B*S, (hq + 2 hk) * 128] projection output."""
    qkv = (torch.randn(B * S, (hq + 2 * hk) * 128, generator=g) * scale).to(torch.bfloat16).to(dev)
    ld = qkv.stride(0)
    q = qkv.as_strided((B, S, hq, 128), (S * ld, ld, 128, 1))
    k = qkv.as_strided((B, S, hk, 128), (S * ld, ld, 128, 1), hq * 128)
    v = qkv.as_strided((B, S, hk, 128), (S * ld, ld, 128, 1), (hq + hk) * 128)
    return q, k, v


@pytest.mark.parametrize("B,S,hq,hk,window", [
    (2, 750, 16, 8, 128),    # DiT sliding-window layer (T = 1500 frames -> 750 tokens)
    (2, 750, 16, 8, None),   # DiT global layer
    (3, 300, 4, 2, 128),     # ragged tail, band covering the whole short sequence
    (1, 77, 2, 1, None),     # one partial block
    (2, 1000, 4, 1, 64),     # G = 4 (two head pairs per kv head), narrow band
    (1, 513, 8, 4, 200),     # band not aligned to the 128-key tiles
])
def test_self_attention_matches_fp32(cuda, B, S, hq, hk, window):
    from demon_b200 import _native as nat
    from demon_b200.attention import attention
    g = torch.Generator().manual_seed(B * 1000 + S + hq)
    q, k, v = fused_qkv(B, S, hq, hk, g, cuda)
    o = attention(q, k, v, window)
    torch.cuda.synchronize()
    assert nat.device_status() == (0, 0)
    check(o, reference(q, k, v, window), f"self B={B} S={S} window={window}")


def test_cross_attention_matches_fp32(cuda):
    """The DiT's cross attention: 750 queries over 256 encoder rows (K / V of one [B*L, 2 hk *
    128] projection)."""
    from demon_b200.attention import attention
    g = torch.Generator().manual_seed(11)
    B, S, L, hq, hk = 3, 750, 256, 16, 8
    q = torch.randn(B, S, hq, 128, generator=g).to(torch.bfloat16).to(cuda)
    kv = torch.randn(B * L, 2 * hk * 128, generator=g).to(torch.bfloat16).to(cuda)
    ld = kv.stride(0)
    k = kv.as_strided((B, L, hk, 128), (L * ld, ld, 128, 1))
    v = kv.as_strided((B, L, hk, 128), (L * ld, ld, 128, 1), hk * 128)
    o = attention(q, k, v, None)
    check(o, reference(q, k, v, None), "cross")


def test_large_logits_rescale(cuda):
    """q and k scaled so that row maxima grow by far more than 2^8 from one key tile to the
    next: the running offset is raised and the accumulator rescaled in place."""
    from demon_b200.attention import attention
    g = torch.Generator().manual_seed(12)
    B, S, hq, hk = 2, 640, 4, 2
    q, k, v = fused_qkv(B, S, hq, hk, g, cuda)
    ramp = torch.linspace(0.2, 6.0, S, device=cuda).to(torch.bfloat16)  # later keys dominate
    k = (k.float() * ramp[None, :, None, None]).to(torch.bfloat16)
    q = (q.float() * 3).to(torch.bfloat16)
    for window in (None, 128):
        o = attention(q, k, v, window)
        check(o, reference(q, k, v, window), f"rescale window={window}")


def test_matches_cudnn_and_is_batch_invariant(cuda):
    """Against PyTorch's cuDNN SDPA (the library path this kernel replaces) on the DiT's global
    layer, and a sequence's rows do not depend on the batch it is computed in."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from demon_b200.attention import attention
    g = torch.Generator().manual_seed(13)
    B, S, hq, hk = 4, 750, 16, 8
    q, k, v = fused_qkv(B, S, hq, hk, g, cuda)
    o = attention(q, k, v, None)
    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
        ref = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), enable_gqa=True).transpose(1, 2)
    check(o, ref.float(), "vs cuDNN")
    one = attention(q[2:3], k[2:3], v[2:3], None)
    assert torch.equal(one, o[2:3])


def test_rejects_bad_arguments(cuda):
    from demon_b200 import _native as nat
    from demon_b200.attention import attention
    q = torch.zeros(1, 128, 3, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(1, 128, 1, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(nat.DemonError, match="even"):
        attention(q, k, k, None)                    # G = 3
    q = torch.zeros(1, 100, 2, 128, dtype=torch.bfloat16, device=cuda)
    k = torch.zeros(1, 64, 1, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(nat.DemonError, match="S == L"):
        attention(q, k, k, 16)                      # band over a different key length
