"""CPU checks of the C-ABI library: it builds, loads, exports every symbol that
include/demon_b200.h declares, and its struct layouts match the ctypes binding.
No compute entry point is called here (there is no GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "demon_b200.h").read_text()
    return sorted(set(re.findall(r"DEMON_API\s+[\w\s\*]+?\b(demon_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from demon_b200 import _build, _native
    _build.build()
    return _native.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("demon_nvfp4_quantize", "demon_nvfp4_gemm", "demon_lora_down", "demon_ode_step"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    from demon_b200 import _native
    so = ctypes.CDLL(str(_native.LIB_PATH))
    for s in declared_symbols():
        assert hasattr(so, s), f"{s} declared in include/demon_b200.h but not exported"
    assert set(declared_symbols()) <= set(_native.EXPORTED) | {"demon_struct_sizes"}


def test_struct_layouts_match(lib):
    from demon_b200 import _native
    g, o = ctypes.c_int64(), ctypes.c_int64()
    assert lib.demon_struct_sizes(ctypes.byref(g), ctypes.byref(o)) == 0
    assert g.value == ctypes.sizeof(_native.DemonGemmArgs)
    assert o.value == ctypes.sizeof(_native.DemonOdeSlot)


def test_host_only_entry_points(lib):
    assert lib.demon_abi_version() == 1
    assert lib.demon_nvfp4_sf_bytes(1500, 2048) == 1536 * 128
    assert lib.demon_nvfp4_sf_bytes(1, 64) == 128 * 4
    # the bounded-wait test hook validates its limit on the host (and 0 disarms it)
    assert lib.demon_test_arm_gemm_stall(ctypes.c_int64(10)) == 1
    assert lib.demon_test_arm_gemm_stall(ctypes.c_int64(5_000_000)) == 0
    assert lib.demon_test_arm_gemm_stall(ctypes.c_int64(0)) == 0


def test_compute_entry_points_fail_cleanly_without_gpu(lib):
    """With no usable device the entry points return an error code, not a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from demon_b200 import _native
    rc = lib.demon_nvfp4_quantize(None, 16, 64, 64, 2, None, None, None, None)
    assert rc != 0
    assert _native.last_error()


def test_product_package_does_not_import_oracle():
    """The product path never routes through the oracle (test infrastructure only)."""
    for p in (ROOT / "demon_b200").rglob("*.py"):
        src = p.read_text()
        assert "oracle" not in re.findall(r"^\s*(?:from|import)\s+(\w+)", src, re.M), p
