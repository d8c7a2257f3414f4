"""Checkpoint interchange (CPU): reference layer extraction, Rust naming, stacked experts."""
import torch

from velvetoptimizer_b200 import FeedForward, MoEConfig, MoELayer
from velvetoptimizer_b200 import checkpoint as C

CFG = MoEConfig(hidden_size=32, intermediate_size=48, moe_num_experts=3, moe_top_k=2,
                flylora_rank=4, flylora_alpha=8.0)


def _model_sd():
    """A VesperLM-shaped state_dict: layer 0 dense FFN, layer 1 MoE (python/vesper/model.py:402-405)."""
    torch.manual_seed(0)
    ffn, moe = FeedForward(CFG), MoELayer(CFG)
    sd = {"embeddings.weight": torch.zeros(10, 32)}
    sd.update({f"layers.0.ffn.{k}": v for k, v in ffn.state_dict().items()})
    sd.update({f"layers.1.ffn.{k}": v for k, v in moe.state_dict().items()})
    sd["layers.1.attention.q_proj.weight"] = torch.zeros(32, 32)
    return sd, ffn, moe


def test_layer_state_dicts_load_unchanged():
    sd, ffn, moe = _model_sd()
    layers = C.layer_state_dicts(sd)
    assert sorted(layers) == [0, 1]
    f2, m2 = FeedForward(CFG), MoELayer(CFG)
    f2.load_state_dict(layers[0])
    m2.load_state_dict(layers[1])
    assert torch.equal(m2.experts[2].down_proj.weight, moe.experts[2].down_proj.weight)


def test_rust_names_round_trip():
    _, _, moe = _model_sd()
    sd = moe.state_dict()
    rs = C.to_rust_names(sd)
    assert "experts.0.gate_proj.lora_b_down.weight" in rs
    assert not any(k.endswith("proj_a") for k in rs)
    back = C.from_rust_names(rs, proj_a_from=sd)
    assert set(back) == set(sd) and all(torch.equal(back[k], sd[k]) for k in sd)


def test_stack_unstack_round_trip():
    _, _, moe = _model_sd()
    sd = moe.state_dict()
    st = C.stack_experts(sd)
    assert st["gate_w"].shape == (3, 48, 32) and st["down_w"].shape == (3, 32, 48)
    assert torch.equal(st["up_lora_up_w"][1], sd["experts.1.up_proj.lora_up.weight"])
    back = C.unstack_experts(st, proj_a_from=sd)
    assert set(back) == set(sd) and all(torch.equal(back[k], sd[k]) for k in sd)
    # the module's own stacking agrees with the checkpoint helper
    mine = moe.stacked_weights(torch.float32)
    assert all(torch.equal(mine[k], st[k]) for k in st)
