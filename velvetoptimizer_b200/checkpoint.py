"""Checkpoint interchange for the MoE / FFN layers.

* The Python reference saves ``torch.save`` dicts whose ``model_state_dict`` holds every
  layer's FFN under ``layers.{i}.ffn.`` (python/train.py:147-202, loaded by
  python/generate.py:27-48); ``layer_state_dicts`` cuts those out so they load into
  ``MoELayer`` / ``FeedForward`` unchanged.
* The Rust twins (Candle ``crates/vesper-core/src/flylora.rs:66-67``, tch
  ``crates/vesper-cli/src/tch_model.rs:47-48``) name the LoRA linears ``lora_b_down`` /
  ``lora_b_up`` and keep no ``proj_a`` buffer; ``to_rust_names`` / ``from_rust_names``
  convert between the two conventions.
* ``stack_experts`` / ``unstack_experts`` convert a MoE layer's per-expert state_dict to the
  stacked ``[E, ...]`` tensors the C ABI's ``vmoe_weights`` takes, and back.
"""
from __future__ import annotations

import re

import torch

_LORA = (("lora_down", "lora_b_down"), ("lora_up", "lora_b_up"))


def to_rust_names(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Python-reference keys -> Candle/tch keys (``proj_a`` buffers are dropped)."""
    out = {}
    for k, v in sd.items():
        if k.endswith(".proj_a"):
            continue
        for py, rs in _LORA:
            k = k.replace(f".{py}.", f".{rs}.")
        out[k] = v
    return out


def from_rust_names(sd: dict[str, torch.Tensor],
                    proj_a_from: dict[str, torch.Tensor] | None = None) -> dict[str, torch.Tensor]:
    """Candle/tch keys -> Python-reference keys.

    ``proj_a`` (unused by the forward, model.py:107-113) is taken from ``proj_a_from`` (e.g.
    a freshly built module's state_dict) when given, else left out (load with strict=False).
    """
    out = {}
    for k, v in sd.items():
        for py, rs in _LORA:
            k = k.replace(f".{rs}.", f".{py}.")
        out[k] = v
    if proj_a_from:
        for k, v in proj_a_from.items():
            if k.endswith(".proj_a"):
                out.setdefault(k, v)
    return out


def layer_state_dicts(model_sd: dict[str, torch.Tensor]) -> dict[int, dict[str, torch.Tensor]]:
    """Per-layer FFN state_dicts (``layers.{i}.ffn.*`` with the prefix removed)."""
    layers: dict[int, dict[str, torch.Tensor]] = {}
    pat = re.compile(r"^layers\.(\d+)\.ffn\.(.+)$")
    for k, v in model_sd.items():
        m = pat.match(k)
        if m:
            layers.setdefault(int(m.group(1)), {})[m.group(2)] = v
    return layers


_EXPERT_KEYS = {
    "gate_w": "gate_proj.base.weight", "gate_b": "gate_proj.base.bias",
    "up_w": "up_proj.base.weight", "up_b": "up_proj.base.bias",
    "down_w": "down_proj.weight", "down_b": "down_proj.bias",
    "gate_lora_down_w": "gate_proj.lora_down.weight", "gate_lora_down_b": "gate_proj.lora_down.bias",
    "gate_lora_up_w": "gate_proj.lora_up.weight", "gate_lora_up_b": "gate_proj.lora_up.bias",
    "up_lora_down_w": "up_proj.lora_down.weight", "up_lora_down_b": "up_proj.lora_down.bias",
    "up_lora_up_w": "up_proj.lora_up.weight", "up_lora_up_b": "up_proj.lora_up.bias",
}


def stack_experts(moe_sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """A MoELayer state_dict -> the stacked tensors of the C ABI (``vmoe_weights`` names)."""
    E = 1 + max(int(m.group(1)) for k in moe_sd if (m := re.match(r"experts\.(\d+)\.", k)))
    out = {"router_w": moe_sd["router.weight"], "router_b": moe_sd["router.bias"]}
    for name, key in _EXPERT_KEYS.items():
        out[name] = torch.stack([moe_sd[f"experts.{e}.{key}"] for e in range(E)])
    return out


def unstack_experts(stacked: dict[str, torch.Tensor],
                    proj_a_from: dict[str, torch.Tensor] | None = None) -> dict[str, torch.Tensor]:
    """The inverse of ``stack_experts`` (``proj_a`` copied from ``proj_a_from`` if given)."""
    sd = {"router.weight": stacked["router_w"], "router.bias": stacked["router_b"]}
    E = stacked["gate_w"].shape[0]
    for name, key in _EXPERT_KEYS.items():
        for e in range(E):
            sd[f"experts.{e}.{key}"] = stacked[name][e]
    if proj_a_from:
        for k, v in proj_a_from.items():
            if k.endswith(".proj_a"):
                sd[k] = v
    return sd
