"""GPU checks of the DiT row kernels, the bf16 linear and fused-projection GEMMs.

References are plain PyTorch fp32 restatements of the reference's eager op sequence
(Qwen3RMSNorm, AdaLN modulation, SiLU * up, apply_rotary_pos_emb in
acestep/models/modeling_acestep_v15_turbo.py), each intermediate the reference keeps in
bf16 rounded to bf16.  Sums of squares are accumulated in another order than torch's, so a
result may differ by one bf16 ulp where the rounding of x * rsqrt(.) is close to a tie:
the bar is >= 99 % of elements bit-identical and none more than one ulp apart.  NVFP4
outputs are checked bit-exactly against the CPU oracle quantiser run on the kernel's own
bf16 values.
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu


def bf(x):
    return x.to(torch.bfloat16).float()


def ulp_check(got, ref, frac=0.99):
    got, ref = got.float().cpu(), ref.float().cpu()
    same = (got == ref)
    assert same.float().mean().item() >= frac, same.float().mean().item()
    gb = got.to(torch.bfloat16).view(torch.int16).int()
    rb = ref.to(torch.bfloat16).view(torch.int16).int()
    assert (gb - rb).abs().max().item() <= 1


def rms_ref(x, w, eps):
    xf = x.float()
    r = torch.rsqrt((xf.double() ** 2).mean(-1, keepdim=True) + eps).float()
    return bf(w.float() * bf(xf * r))


def make_x(M, K, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    if outliers:
        idx = torch.randperm(K, generator=g)[: max(1, K // 100)]
        x[:, idx] *= 20
    return x.to(torch.bfloat16)


def oracle_quant_of(y_bf16_cpu):
    bits = y_bf16_cpu.contiguous().view(torch.int16).numpy().view(np.uint16)
    return O.quantize(bits, O.GS_PER_ROW)


@pytest.mark.parametrize("M,D,B", [(300, 2048, 2), (300, 2048, 20), (300, 2048, 100), (77, 256, 1), (130, 6144, 5)])
def test_adanorm_quantize(cuda, M, D, B):
    """B modulation rows over M rows (S = ceil(M / B) rows each).  At D = 2048 a CTA of the
    staged kernel covers 16 rows and stages two modulation rows: S = 15 (B = 20) is the smallest
    S it takes, S = 3 (B = 100) goes to the per-warp form."""
    from demon_b200.rowops import adanorm_quantize
    S = -(-M // B)
    g = torch.Generator().manual_seed(M + D)
    x = make_x(M, D, 1)
    w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    scale1 = (1 + 0.3 * torch.randn(B, D, generator=g)).to(torch.bfloat16)
    shift = (0.3 * torch.randn(B, D, generator=g)).to(torch.bfloat16)
    eps = 1e-6
    y = torch.empty(M, D, dtype=torch.bfloat16, device=cuda)
    q = adanorm_quantize(x.to(cuda), w.to(cuda), eps, scale1.to(cuda), shift.to(cuda), S, y=y)
    bidx = torch.arange(M) // S
    ref = bf(bf(rms_ref(x, w, eps) * scale1.float()[bidx]) + shift.float()[bidx])
    ulp_check(y, ref)
    codes, sf_swz, _, gs = oracle_quant_of(y.cpu())
    assert np.array_equal(q.codes.cpu().numpy(), codes)
    assert np.array_equal(q.sf.cpu().numpy(), sf_swz)
    assert np.array_equal(q.gs.cpu().numpy(), gs)
    # batch invariance: one row alone gives the same bits
    y1 = torch.empty(1, D, dtype=torch.bfloat16, device=cuda)
    r = M - 1
    q1 = adanorm_quantize(x[r:r + 1].to(cuda), w.to(cuda), eps, scale1[bidx[r]:bidx[r] + 1].to(cuda),
                          shift[bidx[r]:bidx[r] + 1].to(cuda), 1, y=y1)
    assert torch.equal(y1[0], y[r])
    assert torch.equal(q1.codes[0], q.codes[r])


def test_adanorm_plain_norm_bf16_only(cuda):
    from demon_b200.rowops import adanorm_quantize
    x = make_x(64, 512, 3)
    w = torch.linspace(0.5, 1.5, 512).to(torch.bfloat16)
    y = torch.empty(64, 512, dtype=torch.bfloat16, device=cuda)
    q = adanorm_quantize(x.to(cuda), w.to(cuda), 1e-6, quantize=False, y=y)
    assert q is None
    ulp_check(y, rms_ref(x, w, 1e-6))


@pytest.mark.parametrize("M,F", [(200, 6144), (33, 512)])
def test_silu_mul_quantize(cuda, M, F):
    from demon_b200.rowops import silu_mul_quantize
    g = torch.Generator().manual_seed(F)
    gu = (2 * torch.randn(M, 2 * F, generator=g)).to(torch.bfloat16)
    y = torch.empty(M, F, dtype=torch.bfloat16, device=cuda)
    q = silu_mul_quantize(gu.to(cuda), F, y=y)
    gf, uf = gu[:, :F].float(), gu[:, F:].float()
    h = bf(bf(gf / (1 + torch.exp(-gf))) * uf)
    ulp_check(y, h)                    # silu in fp32 then two bf16 roundings, as torch's eager ops
    codes, sf_swz, sf_lin, gs = oracle_quant_of(h.to(torch.bfloat16))
    # codes follow h; h itself may differ by one ulp where exp rounds differently
    same = (q.codes.cpu().numpy() == codes).mean()
    assert same >= 0.99, same
    deq = O.dequantize(q.codes.cpu().numpy(), O.unswizzle_sf(q.sf.cpu().numpy(), M, F), q.gs.cpu().numpy())
    ref = O.dequantize(codes, sf_lin, gs)
    assert np.linalg.norm(deq - ref) / np.linalg.norm(ref) < 1e-2


@pytest.mark.parametrize("rope", [True, False])
def test_head_norm_rope(cuda, rope):
    from demon_b200.rowops import head_norm_rope
    M, S, hq, hk = 90, 45, 4, 2
    ld = (hq + 2 * hk) * 128
    g = torch.Generator().manual_seed(7)
    x = (3 * torch.randn(M, ld, generator=g)).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    emb = torch.cat([pos[:, None] * inv[None]] * 2, -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    xd = x.to(cuda)
    kw = dict(cos=cos.to(cuda), sin=sin.to(cuda), S=S) if rope else {}
    head_norm_rope(xd, 0, hq, wq.to(cuda), 1e-6, **kw)
    head_norm_rope(xd, hq * 128, hk, wk.to(cuda), 1e-6, **kw)

    def ref_heads(xh, w):
        n = rms_ref(xh, w, 1e-6)                       # [M, H, 128]
        if not rope:
            return n
        c = cos.float()[torch.arange(M) % S][:, None]
        s = sin.float()[torch.arange(M) % S][:, None]
        rot = torch.cat([-n[..., 64:], n[..., :64]], -1)
        return bf(bf(n * c) + bf(rot * s))
    ref_q = ref_heads(x[:, :hq * 128].view(M, hq, 128), wq).reshape(M, -1)
    ref_k = ref_heads(x[:, hq * 128:(hq + hk) * 128].view(M, hk, 128), wk).reshape(M, -1)
    out = xd.cpu()
    ulp_check(out[:, :hq * 128], ref_q)
    ulp_check(out[:, hq * 128:(hq + hk) * 128], ref_k)
    assert torch.equal(out[:, (hq + hk) * 128:], x[:, (hq + hk) * 128:])  # v untouched


def test_fused_projection_gemm_equals_separate(cuda):
    from demon_b200 import nvfp4 as Q
    M, K = 300, 2048
    x = make_x(M, K, 11).to(cuda)
    ws = [(torch.randn(n, K) * s).to(torch.bfloat16).to(cuda) for n, s in ((2048, 0.02), (1024, 0.5), (1024, 3.0))]
    packs = [Q.pack_weight(w) for w in ws]
    a = Q.quantize(x)
    fused = Q.gemm(a, Q.fuse_weights(packs))
    sep = torch.cat([Q.gemm(a, p) for p in packs], 1)
    assert torch.equal(fused, sep)


@pytest.mark.parametrize("M,K,N", [(300, 384, 2048), (7, 2048, 12288), (129, 2048, 128), (64, 256, 192)])
def test_bf16_linear(cuda, M, K, N):
    from demon_b200 import nvfp4 as Q
    g = torch.Generator().manual_seed(M + N)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16)
    y = Q.bf16_linear(x.to(cuda), w.to(cuda), b.to(cuda))
    ref = x.double() @ w.double().t() + b.double()
    rel = float((y.cpu().double() - ref).norm() / ref.norm())
    assert rel < 4e-3, rel  # bf16 output rounding: 2^-9 relative at most, ~1e-3 rms
    y1 = Q.bf16_linear(x[M - 1:].to(cuda), w.to(cuda), b.to(cuda))
    assert torch.equal(y1[0], y[M - 1])          # a row does not depend on the batch


@pytest.mark.parametrize("rope", [True, False])
def test_gemm_head_norm_epilogue(cuda, rope):
    """q/k head RMSNorm (+ RoPE) in the GEMM epilogue equals the GEMM followed by the
    standalone head-norm kernel (same arithmetic; the sum of squares runs in another order)."""
    from demon_b200 import nvfp4 as Q
    from demon_b200.rowops import head_norm_rope
    M, K, S, hq, hk = 300, 2048, 150, 4, 2
    N = (hq + 2 * hk) * 128
    g = torch.Generator().manual_seed(21)
    x = make_x(M, K, 5).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    wq = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda)
    wk = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda)
    pos = torch.arange(S, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    emb = torch.cat([pos[:, None] * inv[None]] * 2, -1)
    cos, sin = emb.cos().to(torch.bfloat16).to(cuda), emb.sin().to(torch.bfloat16).to(cuda)
    a, pw = Q.quantize(x), Q.pack_weight(w)
    rp = (cos, sin, S) if rope else None
    fused = Q.gemm(a, pw, head_norm=((hq + hk) * 128, hq * 128, wq, wk, 1e-6), rope=rp)
    ref = Q.gemm(a, pw)
    kw = dict(cos=cos, sin=sin, S=S) if rope else {}
    head_norm_rope(ref, 0, hq, wq, 1e-6, **kw)
    head_norm_rope(ref, hq * 128, hk, wk, 1e-6, **kw)
    ulp_check(fused[:, :(hq + hk) * 128], ref[:, :(hq + hk) * 128])
    assert torch.equal(fused[:, (hq + hk) * 128:], ref[:, (hq + hk) * 128:])


@pytest.mark.parametrize("M,F,bias", [(300, 512, False), (7, 6144, False), (129, 1024, True)])
def test_gemm_silu_epilogue(cuda, M, F, bias):
    """The gate/up GEMM with the SwiGLU epilogue (interleaved weight blocks) gives exactly the
    h of GEMM + demon_silu_mul_quantize, and quantising it gives the same NVFP4 operand."""
    from demon_b200 import nvfp4 as Q
    from demon_b200.rowops import silu_mul_quantize
    K = 2048
    g = torch.Generator().manual_seed(M + F)
    x = make_x(M, K, 9).to(cuda)
    wg = (torch.randn(F, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda)
    wu = (torch.randn(F, K, generator=g) * 0.3).to(torch.bfloat16).to(cuda)
    a, pg, pu = Q.quantize(x), Q.pack_weight(wg), Q.pack_weight(wu)
    bg = bu = None
    if bias:
        bg = (0.5 * torch.randn(F, generator=g)).to(torch.bfloat16).to(cuda)
        bu = (0.5 * torch.randn(F, generator=g)).to(torch.bfloat16).to(cuda)
    b_cat = torch.cat([bg, bu]) if bias else None
    b_il = torch.stack([bg.view(-1, 128), bu.view(-1, 128)], 1).reshape(-1) if bias else None
    gu = Q.gemm(a, Q.fuse_weights([pg, pu]), bias=b_cat)
    y = torch.empty(M, F, dtype=torch.bfloat16, device=cuda)
    ref_q = silu_mul_quantize(gu, F, y=y)
    h = Q.gemm(a, Q.interleave_weights(pg, pu), bias=b_il, silu_mul=True)
    assert h.shape == (M, F)
    assert torch.equal(h, y)
    hq = Q.quantize(h)
    assert torch.equal(hq.codes, ref_q.codes)
    assert torch.equal(hq.sf, ref_q.sf)
    assert torch.equal(hq.gs, ref_q.gs)
    # and against the definition on the GEMM's own gate / up values
    gf, uf = gu[:, :F].float().cpu(), gu[:, F:].float().cpu()
    ulp_check(h, bf(bf(gf / (1 + torch.exp(-gf))) * uf))


def test_adanorm_rejects_short_modulation(cuda):
    """Row m reads modulation row m // rows_per_mod: a table with too few rows is refused on the
    host before any launch (the C ABI is given only its pointer and row pitch)."""
    from demon_b200.rowops import adanorm_quantize
    M, D, S = 1500, 2048, 750
    x = torch.zeros(M, D, dtype=torch.bfloat16, device=cuda)
    w = torch.ones(D, dtype=torch.bfloat16, device=cuda)
    short = torch.ones(1, D, dtype=torch.bfloat16, device=cuda)   # needs M / S = 2 rows
    with pytest.raises(ValueError, match="modulation"):
        adanorm_quantize(x, w, 1e-6, short, short, S)
    ok = torch.ones(2, D, dtype=torch.bfloat16, device=cuda)
    adanorm_quantize(x, w, 1e-6, ok, ok, S)
