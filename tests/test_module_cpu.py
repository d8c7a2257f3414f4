"""CPU: the layers' repack-on-change check (no GPU calls).

Every forward compares a key of (data pointer, version) per parameter with the key the
packed weights were built from.  The parameter list behind the key is cached; these tests
pin that every way of changing a weight still changes the key.
"""
import torch
import torch.nn as nn

from velvetoptimizer_b200 import FeedForward, MoEConfig, MoELayer


def small_layer():
    cfg = MoEConfig(hidden_size=32, intermediate_size=48, moe_num_experts=4, moe_top_k=2)
    return MoELayer(cfg)


def test_param_list_matches_parameters():
    layer = small_layer()
    assert layer._param_list() == list(layer.parameters())
    assert layer._param_list() is layer._param_list()  # cached between calls


def test_in_place_update_changes_key():
    layer = small_layer()
    k0 = layer._weight_key()
    with torch.no_grad():
        layer.experts[2].down_proj.weight.add_(1.0)
    assert layer._weight_key() != k0


def test_load_state_dict_changes_key():
    layer = small_layer()
    k0 = layer._weight_key()
    sd = {k: v.clone() + 1 for k, v in layer.state_dict().items()}
    layer.load_state_dict(sd)
    assert layer._weight_key() != k0


def test_data_assignment_changes_key():
    layer = small_layer()
    k0 = layer._weight_key()
    layer.router.weight.data = torch.zeros_like(layer.router.weight)
    assert layer._weight_key() != k0


def test_parameter_replacement_rebuilds_list():
    layer = small_layer()
    layer._weight_key()
    new = nn.Parameter(torch.zeros_like(layer.router.bias))
    layer.router.bias = new
    assert any(p is new for p in layer._param_list())
    assert layer._param_list() == list(layer.parameters())


def test_submodule_replacement_rebuilds_list():
    layer = small_layer()
    layer._weight_key()
    layer.experts[1] = type(layer.experts[1])(layer.config)
    assert layer._param_list() == list(layer.parameters())
    assert all(any(p is q for q in layer._param_list()) for p in layer.experts[1].parameters())


def test_feedforward_uses_the_same_check():
    cfg = MoEConfig(hidden_size=32, intermediate_size=48, moe_num_experts=4, moe_top_k=2)
    ffn = FeedForward(cfg)
    k0 = ffn._weight_key()
    with torch.no_grad():
        ffn.up_proj.base.weight.mul_(2.0)
    assert ffn._weight_key() != k0
    assert ffn._param_list() == list(ffn.parameters())
