"""GPU parity of the NVFP4 quantiser and block-scaled GEMM against the CPU oracle.

Bars (north star): codes and block scales bit-exact against the oracle
quantiser; GEMM output within relative Frobenius error 1e-2 of the fp32/fp64
dequantise-then-matmul (the reference's refit-merged weights for LoRA).
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 1e-2  # north-star tolerance for the GEMM


def make_x(M, K, seed, outlier_frac=0.01, outlier_scale=20.0):
    """Config-1 activations: N(0,1) with 1% of K channels scaled x20, bf16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    n_out = max(1, int(K * outlier_frac))
    idx = torch.randperm(K, generator=g)[:n_out]
    x[:, idx] *= outlier_scale
    return x.to(torch.bfloat16)


def make_w(N, K, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(N, K, generator=g) * std).to(torch.bfloat16)


def bits(t_bf16_cpu):
    return t_bf16_cpu.view(torch.int16).numpy().view(np.uint16)


def rel_fro(y, ref):
    y = y.double()
    ref = ref.double()
    return float((y - ref).norm() / ref.norm().clamp_min(1e-300))


@pytest.mark.parametrize("M,K", [(1, 64), (37, 192), (128, 256), (300, 2048), (1500, 2048), (129, 6144)])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_quantize_bit_exact(cuda, M, K, mode):
    from demon_b200 import nvfp4
    x = make_x(M, K, seed=M * 7 + K + mode)
    gs_static = np.array([0.37 / 2688.0], np.float32)
    ref_codes, ref_swz, ref_lin, ref_gs = O.quantize(bits(x), mode, gs_static if mode == 0 else None)
    gs = torch.from_numpy(gs_static).to(cuda) if mode == 0 else None
    q = nvfp4.quantize(x.to(cuda), gs_mode=mode, gs=gs)
    torch.cuda.synchronize()
    assert np.array_equal(q.codes.cpu().numpy(), ref_codes)
    assert np.array_equal(q.sf.cpu().numpy(), ref_swz)
    assert np.array_equal(q.gs.cpu().numpy().view(np.uint32), ref_gs.view(np.uint32))


def test_quantize_edge_values(cuda):
    """Ties of E2M1, E4M3 subnormal / saturating scales, zero blocks, +-0."""
    from demon_b200 import nvfp4
    K = 256
    rows = []
    # every E2M1 tie point and neighbours, scaled so the block absmax is 6 (scale 1 after g)
    ties = [0.0, -0.0, 0.25, 0.2499, 0.2501, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -5.0, -6.0]
    rows.append(np.array(ties * (K // 16), np.float32))
    rows.append(np.zeros(K, np.float32))                          # all-zero row
    r = np.zeros(K, np.float32); r[::16] = 1e-30; rows.append(r)  # tiny blocks -> zero scale
    rng = np.random.default_rng(5)
    for e in range(-20, 20, 3):                                    # scales across the E4M3 range
        rows.append((rng.standard_normal(K) * 2.0 ** e).astype(np.float32))
    x = np.stack(rows)
    xb = O.f32_to_bf16_bits(x)
    xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    for mode, g in ((0, np.array([1.0 / 6.0 / 448.0 * 6.0], np.float32)), (1, None), (2, None)):
        ref_codes, ref_swz, _, ref_gs = O.quantize(xb, mode, g)
        q = nvfp4.quantize(xt.to(cuda), gs_mode=mode, gs=torch.from_numpy(g).to(cuda) if g is not None else None)
        assert np.array_equal(q.codes.cpu().numpy(), ref_codes), f"codes mode {mode}"
        assert np.array_equal(q.sf.cpu().numpy(), ref_swz), f"scales mode {mode}"


@pytest.mark.parametrize("K", [2048, 6144])
def test_quantize_nan_values(cuda, K):
    """NaN elements do not count towards any absmax (row or block) and get code 0 -- the
    quantiser's slow path, taken by a whole warp when one of its lanes holds a NaN; rows
    without a NaN next to them take the fast path.  Bit-exact against the oracle."""
    from demon_b200 import nvfp4
    rng = np.random.default_rng(K)
    M = 40
    x = (rng.standard_normal((M, K)) * 2.0).astype(np.float32)
    mask = rng.random((M, K)) < 0.003
    mask[::5] = False                     # some rows hold no NaN at all
    x[mask] = np.nan
    xb = O.f32_to_bf16_bits(x)
    xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    for mode in (1, 2):
        ref_codes, ref_swz, _, ref_gs = O.quantize(xb, mode, None)
        q = nvfp4.quantize(xt.to(cuda), gs_mode=mode)
        assert np.array_equal(q.codes.cpu().numpy(), ref_codes), f"codes mode {mode}"
        assert np.array_equal(q.sf.cpu().numpy(), ref_swz), f"scales mode {mode}"
        assert np.array_equal(q.gs.cpu().numpy().view(np.uint32), np.asarray(ref_gs, np.float32).view(np.uint32))


def _dequant_ref(q_codes, q_sf, gs, rows, K):
    lin = O.unswizzle_sf(q_sf, rows, K)
    return torch.from_numpy(O.dequantize(q_codes, lin, gs))


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (1, 256, 512), (200, 384, 1024), (1500, 6144, 2048),
                                   (750, 2048, 6144)])
def test_gemm_matches_dequant_matmul(cuda, M, N, K):
    from demon_b200 import nvfp4
    x = make_x(M, K, seed=11 + M)
    w = make_w(N, K, seed=13 + N)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(3)) * 0.1).to(torch.bfloat16)
    a = nvfp4.quantize(x.to(cuda))
    wp = nvfp4.pack_weight(w.to(cuda))
    y = nvfp4.gemm(a, wp, bias=bias.to(cuda))
    torch.cuda.synchronize()
    A = _dequant_ref(a.codes.cpu().numpy(), a.sf.cpu().numpy(), a.gs.cpu().numpy(), M, K)
    W = _dequant_ref(wp.codes.cpu().numpy(), wp.sf.cpu().numpy(), wp.gs.cpu().numpy(), N, K)
    ref = A.double() @ W.double().T + bias.double()
    err = rel_fro(y.cpu(), ref)
    assert err <= REL_FRO_TOL, err
    assert err < 5e-3  # bf16 output rounding is the only expected error
    assert torch.isfinite(y).all()


def test_gemm_epilogue_gate_residual(cuda):
    from demon_b200 import nvfp4
    B, S, K, N = 3, 100, 512, 256
    M = B * S
    x = make_x(M, K, seed=21)
    w = make_w(N, K, seed=22)
    g = torch.Generator().manual_seed(23)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    gate = (torch.randn(B, N, generator=g)).to(torch.bfloat16)
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    a = nvfp4.quantize(x.to(cuda))
    wp = nvfp4.pack_weight(w.to(cuda))
    y = nvfp4.gemm(a, wp, bias=bias.to(cuda), residual=res.to(cuda), gate=gate.to(cuda), gate_rows=S)
    A = _dequant_ref(a.codes.cpu().numpy(), a.sf.cpu().numpy(), a.gs.cpu().numpy(), M, K)
    W = _dequant_ref(wp.codes.cpu().numpy(), wp.sf.cpu().numpy(), wp.gs.cpu().numpy(), N, K)
    lin = A.double() @ W.double().T + bias.double()
    ref = res.double() + gate.double().repeat_interleave(S, 0) * lin
    assert rel_fro(y.cpu(), ref) < 5e-3


@pytest.mark.parametrize("rank,N", [(64, 2048), (16, 256), (96, 384)])
def test_gemm_lora_matches_merged_weights(cuda, rank, N):
    """Fused LoRA epilogue vs the reference's merged weight W + s * B @ A (lora.py:316-319, 824-833)."""
    from demon_b200 import nvfp4
    M, K = 300, 1024
    x = make_x(M, K, seed=31)
    w = make_w(N, K, seed=32)
    g = torch.Generator().manual_seed(33)
    A_ = (torch.randn(rank, K, generator=g) * 0.01).to(torch.bfloat16)
    B_ = (torch.randn(N, rank, generator=g) * 0.01).to(torch.bfloat16)
    lin = nvfp4.NVFP4Linear(K, N, bias=False, device=cuda)
    with torch.no_grad():
        lin.weight.copy_(w.to(cuda))
    xc = x.to(cuda)
    y0 = lin(xc).cpu()
    lin.lora.set("l0", A_.to(cuda), B_.to(cuda), strength=0.0)
    assert torch.equal(lin(xc).cpu(), y0)  # strength 0 is a no-op (lora.py:503-526)
    a = nvfp4.quantize(xc)
    Aq = _dequant_ref(a.codes.cpu().numpy(), a.sf.cpu().numpy(), a.gs.cpu().numpy(), M, K).double()
    Wq = _dequant_ref(lin.packed.codes.cpu().numpy(), lin.packed.sf.cpu().numpy(),
                      lin.packed.gs.cpu().numpy(), N, K).double()
    delta = B_.double() @ A_.double()
    for s in (0.25, 1.0):
        lin.lora.set_strength("l0", s)
        y = lin(xc).cpu()
        ref = Aq @ Wq.T + x.double() @ (s * delta).T
        err = rel_fro(y, ref)
        assert err <= REL_FRO_TOL, (s, err)
    lin.lora.remove("l0")
    assert torch.equal(lin(xc).cpu(), y0)


def test_lora_path_alone(cuda):
    """Zero base weight: the output is the LoRA product only (bf16 xa + bf16 MMA)."""
    from demon_b200 import nvfp4
    M, K, N, rank = 257, 2048, 512, 64
    x = make_x(M, K, seed=51)
    g = torch.Generator().manual_seed(52)
    A_ = (torch.randn(rank, K, generator=g) * 0.01).to(torch.bfloat16)
    B_ = (torch.randn(N, rank, generator=g) * 0.01).to(torch.bfloat16)
    lin = nvfp4.NVFP4Linear(K, N, bias=False, device=cuda)
    with torch.no_grad():
        lin.weight.zero_()
    lin.lora.set("a", A_[:48].to(cuda), B_[:, :48].to(cuda), strength=0.7)
    lin.lora.set("b", A_[48:].to(cuda), B_[:, 48:].to(cuda), strength=-1.5)
    y = lin(x.to(cuda)).cpu()
    d = 0.7 * B_[:, :48].double() @ A_[:48].double() - 1.5 * B_[:, 48:].double() @ A_[48:].double()
    ref = x.double() @ d.T
    assert rel_fro(y, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(1500, 6144, 2048), (300, 2048, 6144), (129, 384, 256)])
def test_gemm_matches_cublaslt_nvfp4(cuda, M, N, K):
    """An independent implementation on the same packed operands: cuBLASLt's block-scaled NVFP4
    GEMM (through torch._scaled_mm; E2M1 codes, E4M3 scales in the same 128x4-chunk layout, no
    global scales).  demon's output divided by its alpha = a_gs[m] * w_gs must agree to the bf16
    rounding of the two outputs."""
    from demon_b200 import nvfp4
    if not hasattr(torch, "float4_e2m1fn_x2"):
        pytest.skip("this torch has no NVFP4 dtype")
    x = make_x(M, K, seed=M + N).to(cuda)
    w = make_w(N, K, seed=K).to(cuda)
    a, pw = nvfp4.quantize(x), nvfp4.pack_weight(w)
    y = nvfp4.gemm(a, pw)
    try:
        ref = torch._scaled_mm(a.codes.view(torch.float4_e2m1fn_x2), pw.codes.view(torch.float4_e2m1fn_x2).t(),
                               a.sf.view(torch.float8_e4m3fn), pw.sf.view(torch.float8_e4m3fn),
                               out_dtype=torch.bfloat16)
    except (RuntimeError, TypeError) as e:  # a torch / cuBLASLt build without the NVFP4 path
        pytest.skip(f"cuBLASLt NVFP4 GEMM unavailable: {e}")
    alpha = a.gs.view(-1, 1).float() * pw.gs.view(1, -1).float()
    d = y.float() / alpha
    assert rel_fro(d.cpu(), ref.float().cpu()) < 5e-3


def test_gemm_rows_are_batch_invariant(cuda):
    """A row's output does not depend on the other rows of the batch (stream == batch)."""
    from demon_b200 import nvfp4
    K, N = 2048, 2048
    x = make_x(512, K, seed=41).to(cuda)
    w = nvfp4.pack_weight(make_w(N, K, seed=42).to(cuda))
    full = nvfp4.gemm(nvfp4.quantize(x), w)
    part = nvfp4.gemm(nvfp4.quantize(x[100:229].contiguous()), w)
    assert torch.equal(full[100:229], part)


def test_gemm_rejects_bad_shapes(cuda):
    from demon_b200 import nvfp4, _native
    x = make_x(64, 320, seed=1).to(cuda)  # K % 64 == 0 but K % 256 != 0
    a = nvfp4.quantize(x)
    w = nvfp4.pack_weight(make_w(128, 320, seed=2).to(cuda))
    with pytest.raises(_native.DemonError):
        nvfp4.gemm(a, w)
    assert _native.device_status() == (0, 0)
