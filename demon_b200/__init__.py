"""demon_b200 -- B200-native (sm_100a) hot path of the DEMON streaming diffusion engine.

The package holds the host side of the C ABI in ``include/demon_b200.h``:

- :mod:`demon_b200.nvfp4`  NVFP4 quantiser, block-scaled tcgen05 GEMM with fused
  bias / hot-LoRA / gated-residual epilogue, and the drop-in ``NVFP4Linear``;
- :mod:`demon_b200.ode`    the fused per-slot ODE step and its slot descriptors;
- :mod:`demon_b200.stream` the ring-buffer tick that drives both.

All compute runs in ``libdemon_b200.so`` (built by ``python -m demon_b200._build``);
nothing falls back to a CPU or PyTorch implementation.
"""
from . import _native  # noqa: F401

__all__ = ["_native"]
