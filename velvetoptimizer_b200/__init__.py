"""B200-native (sm_100a) Mixture-of-Experts FFN forward for VelvetOptimizer.

Public surface:
  * ``MoELayer`` — drop-in for the reference ``vesper.model.MoELayer``;
  * ``FeedForward`` — drop-in for the reference dense ``vesper.model.FeedForward``;
  * ``MoEConfig`` — the MoE knobs of ``VesperConfig``;
  * ``torch.ops.vesper_moe.forward`` — the custom op over the C ABI (include/vesper_moe.h).
"""
from .config import MoEConfig
from .moe import ExpertFFN, FeedForward, FlyLoRALinear, MoELayer

__all__ = ["MoEConfig", "MoELayer", "FeedForward", "ExpertFFN", "FlyLoRALinear"]
