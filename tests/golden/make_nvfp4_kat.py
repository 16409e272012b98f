"""Write tests/golden/nvfp4_kat.json: known answers for the NVFP4 format.

- e2m1: every tie point and its neighbours -> expected code, from the format
  definition (magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even code,
  saturating at 6, zero always code 0);
- e4m3: values -> byte from torch's float8_e4m3fn cast (the conversion the
  reference uses, acestep/engine/trt/fp8_onnx.py:144-146), after the
  clamp-to-448 the reference applies (lora_refit.py:598-601);
- quant: two small bf16 blocks quantised by the oracle (regression vectors).

    python tests/golden/make_nvfp4_kat.py
"""
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

# value -> (magnitude code) by the format definition
E2M1_TABLE = [
    (0.0, 0), (0.1, 0), (0.25, 0), (0.2501, 1), (0.5, 1), (0.7499, 1), (0.75, 2), (1.0, 2), (1.25, 2),
    (1.2501, 3), (1.5, 3), (1.7499, 3), (1.75, 4), (2.0, 4), (2.5, 4), (2.5001, 5), (3.0, 5), (3.4999, 5),
    (3.5, 6), (4.0, 6), (5.0, 6), (5.0001, 7), (6.0, 7), (7.0, 7), (1e9, 7),
]


def main():
    from oracle import nvfp4_oracle as O
    e2m1 = []
    for v, mag in E2M1_TABLE:
        e2m1.append([v, mag])
        e2m1.append([-v, (mag | 8) if mag else 0])
    vals = np.array([0.0, 2 ** -10, 2 ** -9, 1.5 * 2 ** -9, 2.5 * 2 ** -9, 2 ** -6, 0.0146484375, 0.1, 1.0, 1.0625,
                     1.1875, 3.3, 100.0, 240.0, 447.0, 448.0], np.float32)
    e4m3 = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((4, 64)) * np.array([1, 1e-3, 30, 1e-8])[:, None]).astype(np.float32)
    bits = O.f32_to_bf16_bits(x)
    quant = {}
    for mode in (1, 2):
        c, swz, lin, gs = O.quantize(bits, mode)
        quant[str(mode)] = {"codes": c.tolist(), "sf": lin.tolist(), "gs_bits": gs.view(np.uint32).tolist()}
    out = {"e2m1": e2m1, "e4m3": [[float(v), int(b)] for v, b in zip(vals, e4m3)],
           "quant_input_bf16_bits": bits.tolist(), "quant": quant}
    (HERE / "nvfp4_kat.json").write_text(json.dumps(out))


if __name__ == "__main__":
    main()
