"""Seeded synthetic inputs for the MoE FFN forward path (test infrastructure).

This module is part of the ORACLE: only tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it.  It never runs on the product path.

The reference publishes no dataset for this path; every input is synthetic, drawn the
way the reference initialises a fresh model:

* ``x ~ N(0, 1)``;
* every ``nn.Linear`` weight ``~ N(0, 0.02)`` with zero bias, as
  ``VesperLM._init_weights`` does (python/vesper/model.py:456-467);
* "FlyLoRA off" means ``lora_up.weight = 0`` and ``lora_up.bias = 0``, which makes the
  low-rank term of ``FlyLoRALinear.forward`` (python/vesper/model.py:123-126) exactly 0;
* the skewed-router case adds a per-expert router bias ``b_e = log(zipf_pmf(e + 1))``
  so expert popularity falls off like Zipf(alpha).

All draws come from one ``numpy.random.Generator(PCG64(seed))`` in a fixed order, so
the same arrays are rebuilt on any machine with the same numpy.
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict

import numpy as np


@dataclass
class MoECase:
    """Shape and option set of one MoE layer forward (names follow VesperConfig)."""

    tokens: int                 # T = batch * seq
    hidden: int                 # H = hidden_size
    inter: int                  # I = intermediate_size (expert d_ff)
    experts: int                # E = moe_num_experts
    top_k: int                  # K = moe_top_k
    batch: int = 1              # B (only the [B, S, H] view uses it)
    era_gamma: float = 0.1      # VesperConfig.era_gamma (python/vesper/config.py:22)
    lora_rank: int = 16         # VesperConfig.flylora_rank (config.py:17)
    lora_alpha: float = 32.0    # VesperConfig.flylora_alpha (config.py:18)
    lora_on: bool = False       # FlyLoRA branch active (non-zero lora_up)
    zipf_alpha: float = 0.0     # > 0: Zipf-skewed router bias
    bias_std: float = 0.0       # > 0: non-zero Linear biases (exercise the bias path)
    weight_std: float = 0.02
    router_std: float | None = None  # None: weight_std; 0.0: an all-tied router
    seed: int = 0

    @property
    def seq(self) -> int:
        assert self.tokens % self.batch == 0
        return self.tokens // self.batch

    @property
    def lora_scaling(self) -> float:
        # FlyLoRALinear.scaling = alpha / rank (python/vesper/model.py:102)
        return self.lora_alpha / self.lora_rank

    def to_dict(self) -> dict:
        return asdict(self)


def zipf_router_bias(experts: int, alpha: float) -> np.ndarray:
    """Router bias b_e = log(pmf(e+1)) of a Zipf(alpha) law truncated to E experts."""
    ranks = np.arange(1, experts + 1, dtype=np.float64)
    pmf = ranks ** (-alpha)
    pmf /= pmf.sum()
    return np.log(pmf).astype(np.float32)


def make_inputs(case: MoECase) -> dict[str, np.ndarray]:
    """Build x and every weight of one MoE layer as fp32 numpy arrays.

    Layout follows ``nn.Linear`` ([out, in] row-major, y = x W^T + b), stacked over
    experts:

    ======  ==============  =========================================================
    key     shape           reference parameter
    ======  ==============  =========================================================
    x       [T, H]          hidden states (``MoELayer.forward`` input, flattened)
    w_r     [E, H]          ``router.weight``           (model.py:314)
    b_r     [E]             ``router.bias``
    w_g     [E, I, H]       ``experts.e.gate_proj.base.weight``  (model.py:116)
    b_g     [E, I]          ``experts.e.gate_proj.base.bias``
    w_u     [E, I, H]       ``experts.e.up_proj.base.weight``
    b_u     [E, I]          ``experts.e.up_proj.base.bias``
    a_g     [E, r, H]       ``experts.e.gate_proj.lora_down.weight`` (model.py:116)
    ba_g    [E, r]          ``experts.e.gate_proj.lora_down.bias``
    l_g     [E, I, r]       ``experts.e.gate_proj.lora_up.weight``   (model.py:117)
    bl_g    [E, I]          ``experts.e.gate_proj.lora_up.bias``
    a_u ..  (same for up_proj)
    w_d     [E, H, I]       ``experts.e.down_proj.weight`` (model.py:290)
    b_d     [E, H]          ``experts.e.down_proj.bias``
    ======  ==============  =========================================================
    """
    c = case
    rng = np.random.default_rng(c.seed)
    T, H, I, E, r = c.tokens, c.hidden, c.inter, c.experts, c.lora_rank
    f32 = np.float32

    def normal(shape, std):
        if std == 0.0:
            return np.zeros(shape, dtype=f32)
        return (rng.standard_normal(shape, dtype=f32) * f32(std)).astype(f32)

    rstd = c.weight_std if c.router_std is None else c.router_std
    out: dict[str, np.ndarray] = {}
    out["x"] = rng.standard_normal((T, H), dtype=f32)
    out["w_r"] = normal((E, H), rstd)
    out["b_r"] = normal((E,), c.bias_std)
    if c.zipf_alpha > 0:
        out["b_r"] = (out["b_r"] + zipf_router_bias(E, c.zipf_alpha)).astype(f32)
    for p in ("g", "u"):
        out[f"w_{p}"] = normal((E, I, H), c.weight_std)
        out[f"b_{p}"] = normal((E, I), c.bias_std)
        out[f"a_{p}"] = normal((E, r, H), c.weight_std)
        out[f"ba_{p}"] = normal((E, r), c.bias_std)
        lstd = c.weight_std if c.lora_on else 0.0
        out[f"l_{p}"] = normal((E, I, r), lstd)
        out[f"bl_{p}"] = normal((E, I), c.bias_std if c.lora_on else 0.0)
    out["w_d"] = normal((E, H, I), c.weight_std)
    out["b_d"] = normal((E, H), c.bias_std)
    return out


def make_norm_inputs(case: MoECase, eps: float = 1e-6) -> dict[str, np.ndarray]:
    """Residual-stream input and LayerNorm parameters for the fused pre-norm block.

    x = 2 * N(0,1) + a per-token offset N(0,1) + a per-channel offset N(0,0.5), so the mean
    subtraction matters; ln_w = 1 + N(0,0.1), ln_b = N(0,0.1); eps as config.layer_norm_eps
    (python/vesper/config.py:26).  Seeded from the case (its seed + 1000).
    """
    rng = np.random.default_rng(case.seed + 1000)
    f32 = np.float32
    T, H = case.tokens, case.hidden
    base = make_inputs(case)["x"]
    x = (f32(2.0) * base + rng.standard_normal((T, 1), dtype=f32)
         + f32(0.5) * rng.standard_normal((1, H), dtype=f32)).astype(f32)
    return {"x": x,
            "ln_w": (f32(1.0) + f32(0.1) * rng.standard_normal(H, dtype=f32)).astype(f32),
            "ln_b": (f32(0.1) * rng.standard_normal(H, dtype=f32)).astype(f32),
            "eps": np.asarray(eps, dtype=f32)}


def backward_inputs(case: MoECase) -> tuple[np.ndarray, np.float32]:
    """(dout ~ N(0,1) [T,H], daux) of the backward cases, seeded from the case (seed + 2000)."""
    rng = np.random.default_rng(case.seed + 2000)
    return rng.standard_normal((case.tokens, case.hidden), dtype=np.float32), np.float32(0.37)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) >> 16
    out = (u.astype(np.uint32) << 16).view(np.float32)
    # NaN stays NaN (not produced by these generators, kept for completeness)
    return np.where(np.isnan(a), a, out).reshape(a.shape)


def bf16_inputs(inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """The same arrays rounded to bf16 (what a bf16 device run actually sees)."""
    return {k: round_bf16(v) for k, v in inputs.items()}


# The workloads the bench and the parity tests are sized on.
WORKLOADS = {
    # fp32 correctness case, runs in the reference PyTorch on CPU
    "c1_fp32": MoECase(tokens=512, batch=2, hidden=768, inter=3072, experts=8, top_k=2),
    # decode-shaped, bf16
    "c2_decode": MoECase(tokens=64, batch=64, hidden=2048, inter=8192, experts=8, top_k=2),
    # prefill, bf16, near-uniform router
    "c3_prefill": MoECase(tokens=32768, batch=8, hidden=2048, inter=8192, experts=8, top_k=2),
    # fine-grained, Zipf-skewed, FlyLoRA rank 16
    "c4_skewed": MoECase(tokens=32768, batch=8, hidden=2048, inter=1024, experts=64, top_k=8,
                         lora_on=True, zipf_alpha=1.2),
    # expert-parallel layer, per-GPU token count
    "c5_ep": MoECase(tokens=65536, batch=16, hidden=4096, inter=2048, experts=64, top_k=4),
}
