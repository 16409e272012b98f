"""The hot-LoRA writeback driven by the reference's own LoRA manager (CPU).

``NVFP4LoRAManager`` below is the reference-side binding a maintainer adds: a subclass of
the reference's ``LoRAManagerBase`` (acestep/engine/lora.py:71-691) whose ``_apply_to_engine``
(lora.py:114-121) hands each enabled LoRA's ``A`` / ``B`` and strength to the NVFP4 linears'
banks (``demon_b200.lora.apply_to_decoder``) instead of rewriting weights.  The reference's
lifecycle (register, enable with and without a strength, set_lora_strength, disable,
re-enable, remove) runs unchanged; after every step each linear's effective delta
``sum_i s_i B_i @ A_i`` must equal what the reference's ``EagerLoRAManager`` wrote into an
fp32 twin of the decoder (live weight - base), within fp32 rounding.  Also checked: a
strength-0 enable adds nothing, a disable keeps the strength for the next enable, two
LoRAs add, and a strength change between non-zero values is an in-place update (captured
CUDA graphs stay valid).

Needs the reference checkout (importable in the build container, absent on GPU boxes):
skipped when it is not found.
"""
import os
import sys
from pathlib import Path

import pytest
import torch

REF = Path(os.environ.get("DEMON_REFERENCE", "/root/reference"))
if not (REF / "acestep" / "engine" / "lora.py").exists():
    pytest.skip("reference checkout not available", allow_module_level=True)
sys.path.insert(0, str(REF))
sys.dont_write_bytecode = True
try:
    from acestep.engine.lora import EagerLoRAManager, LoRAManagerBase, LoRAState  # noqa: E402
except Exception as e:  # pragma: no cover - depends on the container's packages
    pytest.skip(f"reference LoRA manager not importable: {e!r}", allow_module_level=True)

from demon_b200 import nvfp4  # noqa: E402
from demon_b200.lora import (apply_to_decoder, drop_lora, effective_delta, load_lora_pairs,  # noqa: E402
                              lora_param_names)

SHAPES = {"layers.0.self_attn.q_proj": (256, 256), "layers.0.mlp.down_proj": (256, 512),
          "layers.1.self_attn.o_proj": (256, 256)}


class NVFP4LoRAManager(LoRAManagerBase):
    """LoRAManagerBase backend for a decoder of NVFP4 linears (no weight rewrite)."""

    def __init__(self, decoder):
        self._decoder = decoder
        self._linears = lora_param_names(decoder)
        self._param_dtype = {n: torch.bfloat16 for n in self._linears}
        self._param_numel = {n: m.in_features * m.out_features for n, m in self._linears.items()}
        super().__init__()

    def _compute_deltas(self, lora_path):
        # keep the low-rank factors: the GEMM epilogue applies them, nothing is materialised
        return load_lora_pairs(lora_path, set(self._linears))

    def _on_disabled(self, entry):
        drop_lora(self._linears, entry.lora_id)   # release the factors (GPU memory on a GPU decoder)

    def _apply_to_engine(self, param_names):
        apply_to_decoder(self._decoder, param_names,
                         [(e.lora_id, e.state == LoRAState.ENABLED, e.strength, e.deltas or {})
                          for e in self._loras.values()], linears=self._linears)


def _tree(make):
    root = torch.nn.Module()
    for path, (n, k) in SHAPES.items():
        mod = root
        parts = path.split(".")
        for p in parts[:-1]:
            if not hasattr(mod, p):
                mod.add_module(p, torch.nn.Module())
            mod = getattr(mod, p)
        mod.add_module(parts[-1], make(n, k))
    return root


def _write_lora(path, targets, rank, seed):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    t = {}
    for name in targets:
        n, k = SHAPES[name]
        t[f"base_model.model.{name}.lora_A.weight"] = (torch.randn(rank, k, generator=g) * 0.05).to(torch.bfloat16)
        t[f"base_model.model.{name}.lora_B.weight"] = (torch.randn(n, rank, generator=g) * 0.05).to(torch.bfloat16)
    save_file(t, str(path))


def _check(ours, eager_twin):
    for path in SHAPES:
        lin = ours.get_submodule(path)
        want = eager_twin.get_submodule(path).weight.detach().double()   # base is zero: live = delta
        got = effective_delta(lin)
        if got is None:
            assert torch.count_nonzero(want) == 0, path
        else:
            assert torch.allclose(got, want, rtol=1e-5, atol=1e-7), (path, (got - want).abs().max())


def test_reference_lifecycle_drives_the_nvfp4_banks(tmp_path):
    pa, pb = tmp_path / "loraA.safetensors", tmp_path / "loraB.safetensors"
    _write_lora(pa, ["layers.0.self_attn.q_proj", "layers.0.mlp.down_proj"], rank=16, seed=1)
    _write_lora(pb, ["layers.0.self_attn.q_proj", "layers.1.self_attn.o_proj"], rank=32, seed=2)
    ours = _tree(lambda n, k: nvfp4.NVFP4Linear(k, n, bias=False, device="cpu"))
    twin = _tree(lambda n, k: torch.nn.Linear(k, n, bias=False))
    with torch.no_grad():
        for p in twin.parameters():
            p.zero_()
    mine, ref = NVFP4LoRAManager(ours), EagerLoRAManager(twin, device=torch.device("cpu"))

    def both(fn):
        fn(mine)
        fn(ref)
        _check(ours, twin)

    both(lambda m: m.register_lora(str(pa)))
    both(lambda m: m.register_lora(str(pb)))
    both(lambda m: m.enable_lora("loraA", strength=0.0))        # a placeholder: contributes nothing
    assert all(effective_delta(ours.get_submodule(p)) is None for p in SHAPES)
    both(lambda m: m.set_lora_strength("loraA", 0.5))
    both(lambda m: m.enable_lora("loraB", strength=-1.0))       # two LoRAs add
    gen = nvfp4.weights_generation()
    both(lambda m: m.set_lora_strength("loraA", 1.0))
    assert nvfp4.weights_generation() == gen                    # in place: graphs stay valid
    both(lambda m: m.disable_lora("loraA"))
    assert mine.get_lora("loraA").strength == 1.0               # kept across disable
    both(lambda m: m.enable_lora("loraA"))                      # back at 1.0
    both(lambda m: m.set_lora_strength("loraB", 0.0))
    both(lambda m: m.remove_lora("loraA"))
    both(lambda m: m.remove_all())
    assert all(not ours.get_submodule(p).lora.entries for p in SHAPES)
