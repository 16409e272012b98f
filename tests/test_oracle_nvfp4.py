"""CPU checks of the NVFP4 oracle (oracle/nvfp4_ref.c) -- no GPU.

The E4M3 block-scale encoder is pinned to torch's float8_e4m3fn cast (the
reference's conversion, acestep/engine/trt/fp8_onnx.py:144-146) over a dense
and a log-uniform sample of [0, 448]; the whole quantiser is cross-checked
against an independent numpy restatement; known answers come from
tests/golden/nvfp4_kat.json (tests/golden/make_nvfp4_kat.py)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O

KAT = json.loads((Path(__file__).resolve().parent / "golden" / "nvfp4_kat.json").read_text())


def test_e4m3_encoder_matches_torch_cast():
    rng = np.random.default_rng(0)
    vals = np.concatenate([np.linspace(0, 448, 100001, dtype=np.float32),
                           (2.0 ** rng.uniform(-24, np.log2(448), 300000)).astype(np.float32)])
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    enc = np.frompyfunc(lambda v: O.lib().demon_oracle_e4m3_encode(float(v)), 1, 1)
    got = enc(vals[::7]).astype(np.uint8)
    assert np.array_equal(got, ref[::7])


def test_e4m3_decode_roundtrip():
    for b in range(0x7F):
        v = O.lib().demon_oracle_e4m3_decode(b)
        assert O.lib().demon_oracle_e4m3_encode(v) == b


def test_e2m1_known_answers():
    for v, code in KAT["e2m1"]:
        assert O.lib().demon_oracle_e2m1_encode(v) == code, v


def test_e4m3_known_answers():
    for v, b in KAT["e4m3"]:
        assert O.lib().demon_oracle_e4m3_encode(v) == b, v


def test_quant_known_answers():
    bits = np.array(KAT["quant_input_bf16_bits"], np.uint16)
    for mode, exp in KAT["quant"].items():
        c, _, lin, gs = O.quantize(bits, int(mode))
        assert c.tolist() == exp["codes"]
        assert lin.tolist() == exp["sf"]
        assert gs.view(np.uint32).tolist() == exp["gs_bits"]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("M,K", [(7, 64), (130, 256), (64, 2048)])
def test_c_oracle_matches_numpy_restatement(mode, M, K):
    rng = np.random.default_rng(M * K + mode)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[:, rng.choice(K, max(1, K // 100), replace=False)] *= 20
    x[0, :16] = 0.0
    if M > 3:
        x[3] *= 1e-30
    bits = O.f32_to_bf16_bits(x)
    gs = np.array([0.02], np.float32) if mode == 0 else None
    c, swz, lin, g = O.quantize(bits, mode, gs)
    c2, sb2, g2 = O.quantize_numpy(bits, mode, gs)
    assert np.array_equal(c, c2) and np.array_equal(lin, sb2) and np.array_equal(g, g2)
    assert np.array_equal(O.unswizzle_sf(swz, M, K), lin)
    assert np.array_equal(O.swizzle_sf(lin), swz)


def test_dequantisation_error_is_fp4_sized():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((256, 1024)).astype(np.float32)
    bits = O.f32_to_bf16_bits(x)
    c, _, lin, gs = O.quantize(bits, O.GS_PER_ROW)
    xd = O.dequantize(c, lin, gs)
    xf = O.bf16_bits_to_f32(bits)
    rel = np.linalg.norm(xd - xf) / np.linalg.norm(xf)
    assert 0.05 < rel < 0.12  # E2M1 with 16-element E4M3 blocks: ~9% per element on N(0,1)
