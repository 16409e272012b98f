"""ctypes binding of the C ABI in ``include/demon_b200.h``.

The shared library ``demon_b200/libdemon_b200.so`` is the only compute path of
this package: there is no CPU or PyTorch fallback.  If the library is missing
or fails to load, every entry point raises.  Device buffers are torch tensors;
only raw pointers, sizes and the current CUDA stream cross the boundary.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdemon_b200.so"

DEMON_OK, DEMON_ERR_INVALID, DEMON_ERR_CUDA, DEMON_ERR_TIMEOUT, DEMON_ERR_UNSUPPORTED = range(5)
GS_STATIC, GS_DYNAMIC, GS_PER_ROW = 0, 1, 2
ODE_MAX_COND = 4

# flags of DemonOdeSlot (include/demon_b200.h)
ODE_X0PATH = 1 << 0
ODE_MASK = 1 << 1
ODE_CFG = 1 << 2
ODE_MOM_INIT = 1 << 3
ODE_RESCALE = 1 << 4
ODE_X0_TARGET = 1 << 5
ODE_FINAL = 1 << 6
ODE_SDE_CURVE = 1 << 7
ODE_SDE_BARE = 1 << 8
ODE_ONC = 1 << 9
ODE_CACHE_NEG = 1 << 10
ODE_DEC_OUT = 1 << 11
ODE_DEC_MASK = 1 << 12
ODE_VS = 1 << 13
ODE_DCW_LO = 1 << 14
ODE_DCW_HI = 1 << 15
ODE_DCW_PIX = 1 << 16

EXPORTED = (
    "demon_abi_version", "demon_struct_sizes", "demon_last_error", "demon_device_status",
    "demon_nvfp4_sf_bytes", "demon_nvfp4_quantize", "demon_nvfp4_gemm", "demon_lora_down",
    "demon_ode_step", "demon_ode_prepare", "demon_ode_cluster_size", "demon_nvfp4_noalloc_scratch_bytes",
    "demon_nvfp4_linear_noalloc", "demon_test_arm_gemm_stall",
    "demon_bf16_linear", "demon_adanorm_quantize", "demon_silu_mul_quantize", "demon_head_norm_rope",
    "demon_attention", "demon_attention_args_size",
)

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class DemonGemmArgs(ctypes.Structure):
    _fields_ = [
        ("a_codes", _vp), ("a_sf", _vp), ("a_gs", _vp), ("a_gs_per_row", _i32), ("w_gs_per_block", _i32),
        ("w_codes", _vp), ("w_sf", _vp), ("w_gs", _vp),
        ("M", _i64), ("N", _i64), ("K", _i64),
        ("out", _vp), ("ldo", _i64), ("bias", _vp), ("residual", _vp), ("ldr", _i64),
        ("gate", _vp), ("gate_rows", _i64), ("ld_gate", _i64),
        ("lora_xa", _vp), ("lora_b", _vp), ("lora_rank", _i64),
        ("hn_cols", _i64), ("hn_q_cols", _i64), ("rope_S", _i64), ("hn_wq", _vp), ("hn_wk", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp), ("hn_eps", _f32), ("silu_mul", _i32), ("rope_half", _i32),
    ]


class DemonOdeSlot(ctypes.Structure):
    _fields_ = [
        ("xt", _vp),
        ("v_pos", _vp * ODE_MAX_COND), ("w_pos", _vp * ODE_MAX_COND),
        ("v_neg", _vp * ODE_MAX_COND), ("w_neg", _vp * ODE_MAX_COND),
        ("n_pos", _i32), ("n_neg", _i32),
        ("neg_cache", _vp), ("momentum", _vp),
        ("guidance", _vp), ("guidance_s", _f32),
        ("apg_mom", _vp), ("apg_mom_s", _f32),
        ("rescale", _vp), ("rescale_s", _f32),
        ("vscale", _vp), ("vscale_s", _f32),
        ("sdc", _vp), ("sdc_s", _f32),
        ("onc", _vp), ("onc_s", _f32),
        ("x0_coef", _vp), ("x0_coef_s", _f32),
        ("x0_coef_mul", _f32), ("mask_s", _f32),
        ("mask", _vp), ("mask_orig", _vp), ("mask_noise", _vp), ("source", _vp), ("x0_target", _vp),
        ("noise", _vp), ("dec_out", _vp),
        ("mask_s_next", _f32), ("t_curr", _f32), ("t_next", _f32), ("flags", _i32),
        ("seed", ctypes.c_uint64), ("step", ctypes.c_uint64),
        ("dcw_lo", _vp), ("dcw_lo_s", _f32), ("dcw_hi", _vp), ("dcw_hi_s", _f32),
    ]


class DemonAttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("ldq", _i64), ("sq", _i64),
        ("k", _vp), ("ldk", _i64), ("sk", _i64),
        ("v", _vp), ("ldv", _i64), ("sv", _i64),
        ("o", _vp), ("ldo", _i64), ("so", _i64),
        ("B", _i32), ("S", _i32), ("L", _i32), ("Hq", _i32), ("Hk", _i32), ("head_dim", _i32), ("window", _i32),
        ("scale", _f32),
    ]


class DemonError(RuntimeError):
    """A C-ABI call returned a non-zero status (message from demon_last_error)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"demon_b200 error {code}: {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the native library (raises if it is absent: no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m demon_b200._build` "
                "(demon_b200 has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        L.demon_abi_version.restype = ctypes.c_int
        L.demon_struct_sizes.argtypes = [ctypes.POINTER(_i64), ctypes.POINTER(_i64)]
        L.demon_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        L.demon_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint), _vp]
        L.demon_nvfp4_sf_bytes.restype = _i64
        L.demon_nvfp4_sf_bytes.argtypes = [_i64, _i64]
        L.demon_nvfp4_quantize.argtypes = [_vp, _i64, _i64, _i64, ctypes.c_int, _vp, _vp, _vp, _vp]
        L.demon_nvfp4_gemm.argtypes = [ctypes.POINTER(DemonGemmArgs), _vp]
        L.demon_test_arm_gemm_stall.argtypes = [_i64]
        L.demon_lora_down.argtypes = [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, ctypes.c_int, _vp, _vp, _vp]
        L.demon_ode_step.argtypes = [_vp, _i32, _i64, _i64, _vp, _vp]
        L.demon_ode_prepare.argtypes = [_vp, _i32, _i64, _i64, _vp, _vp]
        L.demon_ode_cluster_size.argtypes = [_i32, _i64, ctypes.POINTER(_i32)]
        L.demon_nvfp4_linear_noalloc.argtypes = [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _vp]
        L.demon_bf16_linear.argtypes = [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp, _i64, _vp]
        L.demon_adanorm_quantize.argtypes = [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp,
                                             _vp, _i64, _vp]
        L.demon_silu_mul_quantize.argtypes = [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp]
        L.demon_head_norm_rope.argtypes = [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _f32, _vp]
        L.demon_attention.argtypes = [ctypes.POINTER(DemonAttnArgs), _vp]
        for name in EXPORTED:
            getattr(L, name).restype = (_i64 if name in ("demon_nvfp4_sf_bytes", "demon_nvfp4_noalloc_scratch_bytes",
                                                         "demon_attention_args_size") else ctypes.c_int)
        g, o = _i64(), _i64()
        L.demon_struct_sizes(ctypes.byref(g), ctypes.byref(o))
        if g.value != ctypes.sizeof(DemonGemmArgs) or o.value != ctypes.sizeof(DemonOdeSlot):
            raise RuntimeError(
                f"ABI mismatch: C sizeof(DemonGemmArgs)={g.value} vs {ctypes.sizeof(DemonGemmArgs)}, "
                f"sizeof(DemonOdeSlot)={o.value} vs {ctypes.sizeof(DemonOdeSlot)}")
        if L.demon_attention_args_size() != ctypes.sizeof(DemonAttnArgs):
            raise RuntimeError(f"ABI mismatch: C sizeof(DemonAttnArgs)={L.demon_attention_args_size()} vs "
                               f"{ctypes.sizeof(DemonAttnArgs)}")
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().demon_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != DEMON_OK:
        raise DemonError(rc, last_error())


def ptr(t) -> int:
    """Device pointer of a torch tensor (or 0 for None)."""
    return 0 if t is None else int(t.data_ptr())


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def device_status(stream=None) -> tuple[int, int]:
    """Read and clear the device status word: (DEMON_DEV_* bits, first failing site)."""
    out = (ctypes.c_uint * 2)()
    check(load().demon_device_status(out, stream_ptr(stream)))
    return int(out[0]), int(out[1])


def ode_cluster_size(n_slots: int, T: int) -> int:
    """CTAs per slot cluster that the ODE launches use for n_slots x T on the current device."""
    out = _i32()
    check(load().demon_ode_cluster_size(n_slots, T, ctypes.byref(out)))
    return out.value


def sf_bytes(rows: int, K: int) -> int:
    return int(load().demon_nvfp4_sf_bytes(rows, K))
