"""CPU: the layers' repack-on-change check (no GPU calls).

Every forward compares a key of (data pointer, version) per parameter with the key the
packed weights were built from.  The parameter list behind the key is cached; these tests
pin that every way of changing a weight still changes the key.
"""
import pytest
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


class _DataWriteOptimizer(torch.optim.Optimizer):
    """Writes its update through ``p.data`` as VelvetOptimizer does
    (python/vesper/optimizer.py:176,212): the parameter's version does not change."""

    def __init__(self, params, lr=0.1):
        super().__init__(params, dict(lr=lr))

    @torch.no_grad()
    def step(self, closure=None):
        for group in self.param_groups:
            for p in group["params"]:
                if p.grad is not None:
                    p.data.copy_(p.data.float() - group["lr"] * p.grad.float())


def test_optimizer_step_through_data_changes_key():
    layer = small_layer()
    k0 = layer._weight_key()
    opt = _DataWriteOptimizer(layer.parameters())
    for p in layer.parameters():
        p.grad = torch.ones_like(p)
    versions = [p._version for p in layer.parameters()]
    opt.step()
    assert [p._version for p in layer.parameters()] == versions  # invisible to versions
    assert layer._weight_key() != k0


def test_reference_velvet_optimizer_step_changes_key():
    """The reference's own optimizer (its PyTorch update path on CPU) through the layer."""
    import sys

    import pytest

    from tests.golden_io import reference_python_dir
    ref = reference_python_dir()
    if ref is None:
        pytest.skip("no reference checkout beside this repository")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from vesper.optimizer import VelvetOptimizer
    layer = small_layer()
    opt = VelvetOptimizer(layer.parameters(), lr=1e-2)
    assert opt._kernel_backend == "pytorch"  # CPU: the p.data.copy_ update
    k0 = layer._weight_key()
    for p in layer.parameters():
        p.grad = torch.full_like(p, 0.5)
    before = layer.router.weight.detach().clone()
    opt.step()
    assert not torch.equal(before, layer.router.weight.detach())
    assert layer._weight_key() != k0


def test_mark_weights_dirty_changes_key():
    layer = small_layer()
    k0 = layer._weight_key()
    layer.router.weight.data.add_(1.0)  # neither version nor pointer moves
    assert layer._weight_key() == k0
    layer.mark_weights_dirty()
    assert layer._weight_key() != k0


def test_registration_hooks_ignore_other_modules():
    from velvetoptimizer_b200 import moe
    layer = small_layer()
    layer._param_list()
    g0 = moe._STRUCTURE_GEN[0]
    other = nn.Sequential(nn.Linear(4, 4), nn.ReLU())  # registers modules and parameters
    other[0].weight = nn.Parameter(torch.zeros(4, 4))
    assert moe._STRUCTURE_GEN[0] == g0
    layer.router.weight = nn.Parameter(torch.zeros_like(layer.router.weight))
    assert moe._STRUCTURE_GEN[0] > g0


def test_hooks_installed_by_the_first_layer_not_at_import():
    import subprocess
    import sys
    code = ("import torch\n"
            "from velvetoptimizer_b200 import moe, MoEConfig, MoELayer\n"
            "assert not moe._HOOKS\n"
            "MoELayer(MoEConfig(hidden_size=16, intermediate_size=16, moe_num_experts=2, "
            "moe_top_k=1))\n"
            "assert len(moe._HOOKS) == 3\n")
    import os
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=repo, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_native_pairs_match_the_parameters():
    """The native helper returns every parameter's (data pointer, version), 16 bytes each,
    and the key moves with an in-place write."""
    import struct

    from velvetoptimizer_b200 import moe
    if moe._native_pairs is None:
        pytest.skip("the host helper is not built")
    layer = small_layer()
    plist = layer._param_list()
    raw = moe._native_pairs(plist)
    vals = struct.unpack(f"{2 * len(plist)}Q", raw)
    assert all(vals[2 * i] == p.data_ptr() and vals[2 * i + 1] == p._version
               for i, p in enumerate(plist))
    with torch.no_grad():
        plist[-1].add_(1.0)
    assert moe._native_pairs(plist) != raw
    with pytest.raises(TypeError):
        moe._native_pairs([1, 2])
