"""NVFP4 oracle: ctypes wrapper over oracle/nvfp4_ref.c plus an independent
numpy restatement used to cross-check it.

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package (demon_b200/).

The reference (daydreamlive/DEMON) has no NVFP4 quantiser; the conventions
pinned from it are the absmax floor 1e-12 (acestep/engine/trt/fp8_onnx.py:67),
the E4M3 max 448 and the clamp-then-RNE-cast (fp8_onnx.py:61, :115-149;
acestep/engine/trt/lora_refit.py:598-601).  The E4M3 block-scale cast in
:func:`quantize_numpy` is torch's ``float8_e4m3fn`` cast, the reference's own
conversion, so agreement between the two restatements pins the C encoder to
the reference's rounding.  E2M1 rounding has no reference implementation
("parity unpinned" for that half of the format).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
LIB_PATH = BUILD / "libnvfp4_oracle.so"

GS_STATIC, GS_DYNAMIC, GS_PER_ROW = 0, 1, 2
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C oracle with gcc (no fast-math, no FP contraction)."""
    src = HERE / "nvfp4_ref.c"
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return LIB_PATH
    BUILD.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    subprocess.check_call([
        "gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off",
        "-fno-fast-math", "-o", str(tmp), str(src), "-lm",
    ])
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(build()))
        L.demon_oracle_e4m3_encode.restype = ctypes.c_uint8
        L.demon_oracle_e4m3_encode.argtypes = [ctypes.c_float]
        L.demon_oracle_e4m3_decode.restype = ctypes.c_float
        L.demon_oracle_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.demon_oracle_e2m1_encode.restype = ctypes.c_uint8
        L.demon_oracle_e2m1_encode.argtypes = [ctypes.c_float]
        L.demon_oracle_global_scale.restype = ctypes.c_float
        L.demon_oracle_global_scale.argtypes = [ctypes.c_float]
        L.demon_oracle_sf_offset.restype = ctypes.c_int64
        L.demon_oracle_sf_offset.argtypes = [ctypes.c_int64] * 3
        L.demon_oracle_sf_bytes.restype = ctypes.c_int64
        L.demon_oracle_sf_bytes.argtypes = [ctypes.c_int64] * 2
        L.demon_oracle_quantize.restype = ctypes.c_int
        L.demon_oracle_quantize.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.demon_oracle_dequant.restype = None
        L.demon_oracle_dequant.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def sf_bytes(rows: int, K: int) -> int:
    return ((rows + 127) // 128) * 128 * (K // 16)


def quantize(x_bf16_bits: np.ndarray, gs_mode: int = GS_PER_ROW, gs: np.ndarray | None = None):
    """Quantise bf16 activations (uint16 bit patterns, [M, K]) with the C oracle.

    Returns (codes [M, K/2] u8, sf_swizzled [sf_bytes] u8, sf_linear [M, K/16] u8,
    gs fp32 ([1] or [M])).
    """
    x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16)
    M, K = x.shape
    codes = np.zeros((M, K // 2), np.uint8)
    sf_swz = np.zeros(sf_bytes(M, K), np.uint8)
    sf_lin = np.zeros((M, K // 16), np.uint8)
    if gs_mode == GS_STATIC:
        assert gs is not None
        g = np.ascontiguousarray(np.asarray(gs, np.float32).reshape(1))
    else:
        g = np.zeros(M if gs_mode == GS_PER_ROW else 1, np.float32)
    rc = lib().demon_oracle_quantize(_ptr(x), M, K, K, gs_mode, _ptr(g), _ptr(codes), _ptr(sf_swz), _ptr(sf_lin))
    if rc != 0:
        raise ValueError(f"oracle quantize rejected M={M} K={K} mode={gs_mode}")
    return codes, sf_swz, sf_lin, g


def dequantize(codes: np.ndarray, sf_lin: np.ndarray, gs: np.ndarray) -> np.ndarray:
    M = codes.shape[0]
    K = codes.shape[1] * 2
    out = np.zeros((M, K), np.float32)
    codes = np.ascontiguousarray(codes)
    sf_lin = np.ascontiguousarray(sf_lin)
    g = np.ascontiguousarray(gs, np.float32)
    lib().demon_oracle_dequant(_ptr(codes), _ptr(sf_lin), _ptr(g), int(g.size > 1), M, K, _ptr(out))
    return out


def swizzle_sf(sf_lin: np.ndarray) -> np.ndarray:
    """Row-major [rows, K/16] block scales -> tcgen05 128x4-chunk layout."""
    rows, nkb = sf_lin.shape
    K = nkb * 16
    out = np.zeros(sf_bytes(rows, K), np.uint8)
    m = np.arange(rows)[:, None]
    kb = np.arange(nkb)[None, :]
    r = m % 128
    off = ((m // 128) * (K // 64) + kb // 4) * 512 + (r % 32) * 16 + (r // 32) * 4 + (kb % 4)
    out[off.ravel()] = sf_lin.ravel()
    return out


def unswizzle_sf(sf_swz: np.ndarray, rows: int, K: int) -> np.ndarray:
    m = np.arange(rows)[:, None]
    kb = np.arange(K // 16)[None, :]
    r = m % 128
    off = ((m // 128) * (K // 64) + kb // 4) * 512 + (r % 32) * 16 + (r // 32) * 4 + (kb % 4)
    return sf_swz[off]


# ---------------------------------------------------------------------------
# Independent numpy restatement (different algorithm for E2M1 rounding; the
# E4M3 cast is torch's float8_e4m3fn, i.e. the reference's conversion).
# ---------------------------------------------------------------------------

def _e4m3_torch(s: np.ndarray) -> np.ndarray:
    import torch
    t = torch.from_numpy(np.ascontiguousarray(s, np.float32)).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy().copy(), t.float().numpy()


def _e2m1_nearest_even(v: np.ndarray) -> np.ndarray:
    """Nearest E2M1 code by explicit distance comparison; ties pick the even code."""
    a = np.minimum(np.abs(v.astype(np.float64)), 6.0)
    a = np.where(np.isnan(a), 0.0, a)
    d = np.abs(a[..., None] - E2M1_VALUES.astype(np.float64))      # [..., 8]
    best = np.argmin(d, axis=-1)
    dmin = np.take_along_axis(d, best[..., None], -1)[..., 0]
    # a tie can only be with the next code up; prefer the even one
    nxt = np.minimum(best + 1, 7)
    dn = np.take_along_axis(d, nxt[..., None], -1)[..., 0]
    tie = (dn == dmin) & (nxt != best)
    mag = np.where(tie & (best % 2 == 1), nxt, best)
    sign = (v < 0) & (mag != 0)
    return (mag | (sign.astype(np.int64) << 3)).astype(np.uint8)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def quantize_numpy(x_bf16_bits: np.ndarray, gs_mode: int = GS_PER_ROW, gs=None):
    x = bf16_bits_to_f32(np.asarray(x_bf16_bits, np.uint16))
    M, K = x.shape
    f32 = np.float32
    absx = np.abs(x)
    if gs_mode == GS_STATIC:
        g = np.full((M, 1), np.asarray(gs, f32).reshape(-1)[0], f32)
        g_out = np.asarray(gs, f32).reshape(1)
    elif gs_mode == GS_DYNAMIC:
        amax = f32(np.nanmax(absx)) if M else f32(0)
        g0 = f32(max(amax, f32(1e-12)) / f32(2688.0))
        g = np.full((M, 1), g0, f32)
        g_out = np.array([g0], f32)
    else:
        amax = np.nanmax(absx, axis=1).astype(f32)
        g = (np.maximum(amax, f32(1e-12)) / f32(2688.0)).astype(f32)[:, None]
        g_out = g[:, 0].copy()
    xb = x.reshape(M, K // 16, 16)
    amax_b = np.nanmax(np.abs(xb), axis=2).astype(f32)
    denom = (f32(6.0) * g).astype(f32)
    s = (amax_b / denom).astype(f32)
    s = np.where(s <= f32(448.0), s, f32(448.0)).astype(f32)
    sb_bits, sbf = _e4m3_torch(s)
    scale = (sbf * g).astype(f32)
    with np.errstate(divide="ignore", invalid="ignore"):
        rs = (f32(1.0) / scale).astype(f32)
        v = (xb * rs[..., None]).astype(f32)  # zero-scale blocks give 0*inf here; masked below
    codes = _e2m1_nearest_even(v)
    codes = np.where((sbf == 0)[..., None], np.uint8(0), codes).reshape(M, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, sb_bits.astype(np.uint8), g_out
