"""MoE layer configuration: the MoE knobs of the reference's VesperConfig.

Field names and defaults follow python/vesper/config.py (FlyLoRA :17-19, ERA gamma :22,
MoE :33-36) so a reference ``VesperConfig`` can be passed wherever an ``MoEConfig`` is
accepted; ``validate`` raises like ``VesperConfig.validate`` (config.py:89-94).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class MoEConfig:
    hidden_size: int = 768
    intermediate_size: int = 3072
    moe_num_experts: int = 8
    moe_top_k: int = 2
    moe_aux_loss_weight: float = 0.01
    flylora_rank: int = 16
    flylora_alpha: float = 32.0
    flylora_sparsity: float = 0.25
    era_gamma: float = 0.1
    # tokens an expert may take per forward; 0 keeps every token (the reference has no
    # capacity limit, so 0 is the parity setting)
    moe_capacity: int = 0

    @classmethod
    def from_any(cls, cfg) -> "MoEConfig":
        """Accept an MoEConfig or any object with VesperConfig's attribute names."""
        if isinstance(cfg, cls):
            return cfg
        names = [f for f in cls.__dataclass_fields__]
        kw = {n: getattr(cfg, n) for n in names if hasattr(cfg, n)}
        return cls(**kw)

    def validate(self) -> None:
        # VesperConfig.validate, MoE part (python/vesper/config.py:91-94)
        assert 1 <= self.moe_top_k <= self.moe_num_experts
        assert self.moe_num_experts >= 2
        assert self.moe_capacity >= 0
        assert self.hidden_size > 0 and self.intermediate_size > 0

    @property
    def lora_scaling(self) -> float:
        # FlyLoRALinear.scaling (python/vesper/model.py:102)
        return self.flylora_alpha / self.flylora_rank if self.flylora_rank > 0 else 0.0
