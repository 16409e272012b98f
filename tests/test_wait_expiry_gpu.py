"""The GEMM's bounded device-side waits, run out on purpose and recovered from.

Every mbarrier wait of the NVFP4 GEMM gives up after a time limit: the CTA then records
DEMON_DEV_TIMEOUT in the library's status word, stops issuing work, waits (bounded) for the
copies it already issued, frees its tensor memory and returns, so a stuck pipeline ends with
an error the host can read instead of hanging the GPU.  ``demon_test_arm_gemm_stall`` makes
this happen without any fault: for one launch, the first CTA (pair) waits at most a few
milliseconds and never issues the loads of its first stage -- no copy is in flight for them,
nothing waits on another GPU, nothing traps.  The test checks that the status word reports
the timeout, that the launch came back, and that the next launches on the same device are
exact again (the context stays usable).
"""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV_TIMEOUT = 0x1


def _operands(cuda, M, N, K, seed):
    from demon_b200 import nvfp4
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    return nvfp4.quantize(x), nvfp4.pack_weight(w)


@pytest.mark.parametrize("M,N,K", [(1024, 512, 2048),   # CTA pairs (N % 256 == 0)
                                   (1024, 384, 1024)])  # one-CTA 128-wide tiles
def test_gemm_wait_expiry_reports_timeout_and_recovers(cuda, M, N, K):
    from demon_b200 import _native as nat
    from demon_b200 import nvfp4
    lib = nat.load()
    a, w = _operands(cuda, M, N, K, seed=M + N)
    ref = nvfp4.gemm(a, w)
    assert nat.device_status() == (0, 0)
    nat.check(lib.demon_test_arm_gemm_stall(ctypes.c_int64(5_000_000)))  # 5 ms per wait
    t0 = time.perf_counter()
    nvfp4.gemm(a, w)                         # the armed launch: its first CTA gives up
    bits, where = nat.device_status()        # synchronises the stream
    dt = time.perf_counter() - t0
    assert bits & DEV_TIMEOUT, (bits, where)
    assert where != 0
    assert dt < 5.0, dt                      # ended on its own within a few wait limits
    # the context is intact and the hook was one-shot: the next launches are exact
    for _ in range(2):
        again = nvfp4.gemm(a, w)
        torch.cuda.synchronize()
        assert torch.equal(again, ref)
    assert nat.device_status() == (0, 0)


def test_arm_gemm_stall_checks_its_argument(cuda):
    from demon_b200 import _native as nat
    lib = nat.load()
    assert lib.demon_test_arm_gemm_stall(ctypes.c_int64(10)) == nat.DEMON_ERR_INVALID
    assert lib.demon_test_arm_gemm_stall(ctypes.c_int64(0)) == nat.DEMON_OK
