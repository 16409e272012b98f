"""Hot-LoRA writeback for a decoder of NVFP4 linears.

The reference's LoRA manager (acestep/engine/lora.py:71-691, ``LoRAManagerBase``) owns the
catalog and lifecycle and leaves one method to its backend: ``_apply_to_engine(param_names)``
(lora.py:114-121), which must make every listed weight equal ``base + sum_i s_i * B_i @ A_i``
over the ENABLED LoRAs (the eager backend rewrites ``param.data``, lora.py:811-833; the
TensorRT backend refits and re-quantises, 1.2 s).  Here no weight is rewritten: each
linear's :class:`~demon_b200.nvfp4.LoRABank` holds the enabled LoRAs' ``A`` / ``B`` and
strengths, and the GEMM adds ``sum_i s_i (x A_i^T) B_i^T`` in its epilogue.  A manager
subclass therefore keeps each LoRA's ``(A, B)`` pairs instead of the full-rank ``B @ A`` the
base class materialises (:func:`load_lora_pairs`) and calls :func:`apply_to_decoder` from
``_apply_to_engine``.

Semantics kept from the reference: the delta is raw ``B @ A`` (no alpha / rank factor,
lora.py:316-319); a strength-0 or disabled LoRA contributes nothing; strengths of several
LoRAs add; a strength change between two non-zero values is an in-place scalar update that
keeps captured CUDA graphs valid.
"""
from __future__ import annotations

from typing import Dict, Iterable, Mapping, Set, Tuple

import torch

from .nvfp4 import NVFP4Linear


def lora_param_names(decoder: torch.nn.Module) -> Dict[str, NVFP4Linear]:
    """Decoder-relative weight names of every NVFP4 linear (``layers.3.self_attn.q_proj.weight``,
    the names ``decoder.named_parameters()`` and PEFT LoRA keys use) -> the linear."""
    return {f"{name}.weight": m for name, m in decoder.named_modules() if isinstance(m, NVFP4Linear)}


def load_lora_pairs(path: str, param_names: Set[str]) -> Tuple[Dict[str, Tuple[torch.Tensor, torch.Tensor]], int]:
    """The PEFT ``lora_A`` / ``lora_B`` tensors of a LoRA safetensors file per weight name, with
    the key mapping of the reference's ``_compute_deltas`` (lora.py:283-302: the
    ``base_model.model.`` prefix dropped, ``.lora_A.weight`` / ``.lora_B.weight`` -> ``.weight``);
    weights not in ``param_names`` are skipped.  Returns (pairs, bytes of the kept tensors)."""
    from safetensors.torch import load_file
    raw = load_file(path)
    halves: Dict[str, Dict[str, torch.Tensor]] = {}
    for key, t in raw.items():
        k = key.replace("base_model.model.", "")
        if ".lora_A.weight" in k:
            halves.setdefault(k.replace(".lora_A.weight", ".weight"), {})["A"] = t
        elif ".lora_B.weight" in k:
            halves.setdefault(k.replace(".lora_B.weight", ".weight"), {})["B"] = t
    pairs, nbytes = {}, 0
    for name, ab in halves.items():
        if "A" in ab and "B" in ab and name in param_names:
            A, B = ab["A"].to(torch.bfloat16).contiguous(), ab["B"].to(torch.bfloat16).contiguous()
            pairs[name] = (A, B)
            nbytes += A.numel() * A.element_size() + B.numel() * B.element_size()
    return pairs, nbytes


def apply_to_decoder(decoder: torch.nn.Module, param_names: Iterable[str],
                     loras: Iterable[Tuple[str, bool, float, Mapping[str, Tuple[torch.Tensor, torch.Tensor]]]],
                     linears: Dict[str, NVFP4Linear] | None = None) -> None:
    """``_apply_to_engine`` for a decoder of NVFP4 linears.

    ``loras``: every catalogued LoRA as ``(lora_id, enabled, strength, pairs)`` with ``pairs``
    its ``{weight name: (A [r, K], B [N, r])}``.  For each listed weight the linear's bank ends
    up holding exactly the enabled LoRAs that have a pair for it, at their strengths; a LoRA
    whose pair is already in the bank only gets its strength updated."""
    lins = linears if linears is not None else lora_param_names(decoder)
    loras = list(loras)
    for name in param_names:
        lin = lins.get(name)
        if lin is None:
            continue
        bank = lin.lora
        for lora_id, enabled, strength, pairs in loras:
            pair = pairs.get(name) if (enabled and pairs) else None
            if pair is None:
                if lora_id in bank.entries:
                    bank.remove(lora_id)
                continue
            A, B = pair
            e = bank.entries.get(lora_id)
            dev = lin.weight.device
            if e is not None and e.A.shape == A.shape and e.B.shape == B.shape and e.enabled:
                if e.strength != float(strength):
                    bank.set_strength(lora_id, strength)
            else:
                bank.set(lora_id, A.to(dev), B.to(dev), strength=strength)


def drop_lora(linears: Mapping[str, NVFP4Linear], lora_id: str) -> None:
    """Remove one LoRA from every bank that holds it: the ``_on_disabled`` hook of a manager
    subclass (lora.py:132-136), which the reference calls whenever a LoRA leaves ENABLED --
    also for a strength-0 LoRA, whose disable refits nothing but whose factors are held."""
    for lin in linears.values():
        if lora_id in lin.lora.entries:
            lin.lora.remove(lora_id)


def effective_delta(lin: NVFP4Linear) -> torch.Tensor | None:
    """``sum_i s_i * B_i @ A_i`` of a linear's bank in fp64 (what the epilogue adds), or None."""
    act = lin.lora.active()
    if act is None:
        return None
    A, B, scale = act
    return (B.double().cpu() * scale.double().cpu()[None, :]) @ A.double().cpu()
