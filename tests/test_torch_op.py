"""The torch.library op ``demon_b200::nvfp4_linear`` (the torch-op surface of the linear).

CPU: the op is registered under torch.ops.demon_b200 with a fake (meta) kernel, so shape
propagation works without a GPU, and it has no CPU kernel (no fallback path).
GPU: the op gives exactly the bits of the direct C-ABI path (quantise + LoRA down-projection
+ GEMM epilogue), and ``NVFP4Linear.forward`` goes through it.
"""
import pytest
import torch

from demon_b200 import nvfp4


def _fake_args(dev="cuda"):
    x = torch.empty(3, 5, 256, dtype=torch.bfloat16, device=dev)
    wc = torch.empty(384, 128, dtype=torch.uint8, device=dev)
    return x, wc, torch.empty(384 * 16, dtype=torch.uint8, device=dev), torch.empty(1, device=dev)


def test_op_is_registered_with_a_fake_kernel():
    from torch._subclasses.fake_tensor import FakeTensorMode
    assert hasattr(torch.ops.demon_b200, "nvfp4_linear")
    with FakeTensorMode():
        y = torch.ops.demon_b200.nvfp4_linear(*_fake_args())
        assert y.shape == (3, 5, 384) and y.dtype == torch.bfloat16
        A = torch.empty(16, 256, dtype=torch.bfloat16, device="cuda")
        B = torch.empty(384, 16, dtype=torch.bfloat16, device="cuda")
        res = torch.empty(3, 5, 384, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.demon_b200.nvfp4_linear(*_fake_args(), None, A, B, 0.5, res, None)
        assert y.shape == (3, 5, 384)


def test_op_has_no_cpu_kernel():
    x, wc, sf, gs = _fake_args("cpu")
    with pytest.raises(NotImplementedError):
        torch.ops.demon_b200.nvfp4_linear(x, wc, sf, gs)


@pytest.mark.gpu
def test_op_matches_direct_path_and_backs_the_module(cuda):
    g = torch.Generator().manual_seed(5)
    B, S, K, N, r = 3, 100, 1024, 512, 32
    x = torch.randn(B, S, K, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    bias = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).to(cuda)
    A = (torch.randn(r, K, generator=g) * 0.01).to(torch.bfloat16).to(cuda)
    Bl = (torch.randn(N, r, generator=g) * 0.01).to(torch.bfloat16).to(cuda)
    res = torch.randn(B, S, N, generator=g).to(torch.bfloat16).to(cuda)
    gate = torch.randn(B, N, generator=g).to(torch.bfloat16).to(cuda)
    pw = nvfp4.pack_weight(w)
    x2 = x.reshape(-1, K)
    a = nvfp4.quantize(x2)
    cs = torch.full((r,), 0.7, dtype=torch.float32, device=cuda)
    xa = nvfp4.lora_down(x2, A, cs, a, pw)
    direct = nvfp4.gemm(a, pw, bias=bias, residual=res.reshape(-1, N), gate=gate, gate_rows=S, lora_xa=xa,
                        lora_b=Bl).reshape(B, S, N)
    op = torch.ops.demon_b200.nvfp4_linear(x, pw.codes, pw.sf, pw.gs, bias, A, Bl, 0.7, res, gate)
    assert torch.equal(op, direct)
    op2 = torch.ops.demon_b200.nvfp4_linear(x, pw.codes, pw.sf, pw.gs, bias, A, Bl, 1.0, res, gate, cs)
    assert torch.equal(op2, direct)
    plain = torch.ops.demon_b200.nvfp4_linear(x, pw.codes, pw.sf, pw.gs, bias)
    assert torch.equal(plain, nvfp4.gemm(a, pw, bias=bias).reshape(B, S, N))
    # the module's forward is the op
    lin = nvfp4.NVFP4Linear(K, N, bias=True, device=cuda)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(bias)
    lin.lora.set("l", A, Bl, strength=0.7)
    calls = []
    orig = torch.ops.demon_b200.nvfp4_linear

    class Spy:
        def __call__(self, *args):
            calls.append(len(args))
            return orig(*args)
    try:
        torch.ops.demon_b200.nvfp4_linear = Spy()
        y = lin(x, residual=res, gate=gate)
    finally:
        torch.ops.demon_b200.nvfp4_linear = orig
    assert calls, "NVFP4Linear.forward did not go through torch.ops.demon_b200.nvfp4_linear"
    assert torch.equal(y, direct)
