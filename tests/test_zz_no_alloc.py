"""The allocation-free NVFP4 linear (demon_nvfp4_linear_noalloc).

Callers that cannot allocate device memory while the layer runs -- a TensorRT
plugin's enqueue(), or a real-time thread that must not block in cudaMalloc --
use this entry point: it keeps the quantised activation in a fixed array
inside the library instead of buffers the caller provides.  This test calls it
through the C ABI twice in a row (the second call reuses the array the first
one left behind) and checks each result against the regular entry points
(demon_nvfp4_quantize + demon_nvfp4_gemm).  Both paths run the same two kernels
with the same per-row scales on the same shapes, so the outputs must be
bit-identical; the relative Frobenius error the other GEMM tests use (1e-2) is
only reported in the failure message.  It also checks that a call larger than
the array, or with an argument only the GEMM rejects, fails on the host and
enqueues no kernel at all (so the array keeps the previous call's contents).

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import warnings

import pytest
import torch

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 1e-2


def _linear_noalloc(lib, x, w, bias, out, N=None, ldo=None):
    from demon_b200 import _native as nat
    M, K = x.shape
    return lib.demon_nvfp4_linear_noalloc(
        ctypes.c_void_p(x.data_ptr()), M, K, x.stride(0), ctypes.c_void_p(w.codes.data_ptr()),
        ctypes.c_void_p(w.sf.data_ptr()), ctypes.c_void_p(w.gs.data_ptr()), w.rows if N is None else N,
        ctypes.c_void_p(bias.data_ptr() if bias is not None else 0), ctypes.c_void_p(out.data_ptr()),
        out.stride(0) if ldo is None else ldo, ctypes.c_void_p(nat.stream_ptr()))


def _rel_fro(y, ref):
    return float((y.double() - ref.double()).norm() / ref.double().norm())


def _case(cuda, g, M, K, N):
    from demon_b200 import nvfp4
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    w = nvfp4.pack_weight((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda))
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    return x, w, bias


def test_noalloc_linear_matches_regular_path_twice(cuda):
    from demon_b200 import _native as nat
    from demon_b200 import nvfp4
    lib = nat.load()
    g = torch.Generator().manual_seed(77)
    cases = [(1500, 2048, 6144), (700, 6144, 2048)]  # second call: different shape, same array
    for M, K, N in cases:
        x, w, bias = _case(cuda, g, M, K, N)
        ref = nvfp4.gemm(nvfp4.quantize(x), w, bias=bias)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        rc = _linear_noalloc(lib, x, w, bias, out)
        assert rc == nat.DEMON_OK, nat.last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        err = _rel_fro(out, ref)
        assert torch.equal(out, ref), f"noalloc differs from the regular path (rel. Frobenius {err:.2e})"
        assert err <= REL_FRO_TOL
    assert nat.device_status() == (0, 0)


def test_noalloc_linear_rejects_oversized_calls(cuda):
    from demon_b200 import _native as nat
    from demon_b200 import nvfp4
    lib = nat.load()
    K, N = 6144, 128
    M = 8_388_608 // K + 1  # one row past the array's activation limit
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    w = nvfp4.pack_weight(torch.zeros(N, K, dtype=torch.bfloat16, device=cuda))
    out = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda)
    rc = _linear_noalloc(lib, x, w, None, out)
    assert rc == nat.DEMON_ERR_INVALID
    assert "scratch" in nat.last_error()
    assert lib.demon_nvfp4_noalloc_scratch_bytes() == (4 << 20) + (640 << 10) + 65536 * 4


def _kernel_nodes_enqueued(fn):
    """Runs fn() under stream capture and returns the number of graph nodes it enqueued."""
    from cuda.bindings import runtime as rt
    graph = torch.cuda.CUDAGraph(keep_graph=True)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")  # torch may warn that the captured graph is empty
        with torch.cuda.graph(graph):
            rc = fn()
    err, _, n = rt.cudaGraphGetNodes(rt.cudaGraph_t(init_value=graph.raw_cuda_graph()), 0)
    assert err == rt.cudaError_t.cudaSuccess
    return rc, int(n)


def test_noalloc_rejected_call_launches_nothing(cuda):
    """A call that only the GEMM half rejects (N not a multiple of 128; an unaligned row
    pitch of the output) fails on the host before the quantiser runs: nothing is enqueued,
    and the array still holds the previous call's operand."""
    from demon_b200 import _native as nat
    from demon_b200 import nvfp4
    lib = nat.load()
    g = torch.Generator().manual_seed(78)
    M, K, N = 640, 2048, 1024
    x, w, bias = _case(cuda, g, M, K, N)
    first = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    assert _linear_noalloc(lib, x, w, bias, first) == nat.DEMON_OK, nat.last_error()  # address looked up
    torch.cuda.synchronize()
    x2, w2, _ = _case(cuda, g, M, K, 64)
    out2 = torch.empty(M, 1024, dtype=torch.bfloat16, device=cuda)
    rc, nodes = _kernel_nodes_enqueued(lambda: _linear_noalloc(lib, x2, w, None, out2, N=64))
    assert rc == nat.DEMON_ERR_INVALID and nodes == 0, (rc, nodes, nat.last_error())
    rc, nodes = _kernel_nodes_enqueued(lambda: _linear_noalloc(lib, x2, w, None, out2, ldo=1028))
    assert rc == nat.DEMON_ERR_INVALID and nodes == 0, (rc, nodes, nat.last_error())
    again = torch.empty_like(first)
    assert _linear_noalloc(lib, x, w, bias, again) == nat.DEMON_OK
    torch.cuda.synchronize()
    assert torch.equal(again, first)
    assert torch.equal(first, nvfp4.gemm(nvfp4.quantize(x), w, bias=bias))
    assert nat.device_status() == (0, 0)
