"""CPU-only checks of the C-ABI library and the host-side layer (no GPU calls)."""
import ctypes
import json
import os
import re

import pytest
import torch

from velvetoptimizer_b200 import MoEConfig, MoELayer, _lib
from velvetoptimizer_b200.build import LIB

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "vesper_moe.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"VMOE_API\s+(?:int|const char\s*\*)\s+(vmoe_\w+)\s*\(", text)))


def test_library_built_and_loads():
    assert os.path.exists(LIB)
    lib = _lib.load()
    assert lib.vmoe_abi_version() == 1


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert len(syms) >= 13
    lib = ctypes.CDLL(LIB)
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.EXPORTED)


def test_status_strings():
    lib = _lib.load()
    assert lib.vmoe_status_string(0) == b"ok"
    assert lib.vmoe_status_string(_lib.VMOE_ERR_INVALID_ARG) == b"invalid argument"
    assert lib.vmoe_stage_name(0) == b"router"
    assert lib.vmoe_stage_name(99) == b""


def _create(**kw):
    base = dict(hidden=64, inter=128, num_experts=4, top_k=2, lora_rank=16, lora_scaling=2.0,
                era_gamma=0.1, dtype=_lib.VMOE_F32, capacity=0)
    base.update(kw)
    cfg = _lib.VmoeConfig(**base)
    h = ctypes.c_void_p()
    rc = _lib.load().vmoe_create(ctypes.byref(cfg), 0, ctypes.byref(h))
    return rc, h


@pytest.mark.parametrize("kw,code", [
    (dict(top_k=5), _lib.VMOE_ERR_INVALID_ARG),        # top_k > E   (config.py:92)
    (dict(top_k=0), _lib.VMOE_ERR_INVALID_ARG),
    (dict(num_experts=1, top_k=1), _lib.VMOE_ERR_INVALID_ARG),  # E >= 2 (config.py:94)
    (dict(hidden=0), _lib.VMOE_ERR_INVALID_ARG),
    (dict(dtype=7), _lib.VMOE_ERR_INVALID_ARG),
    (dict(capacity=-1), _lib.VMOE_ERR_INVALID_ARG),
    (dict(hidden=60), _lib.VMOE_ERR_UNSUPPORTED_SHAPE),
    (dict(num_experts=512, top_k=2), _lib.VMOE_ERR_UNSUPPORTED_SHAPE),
    (dict(num_experts=64, top_k=40), _lib.VMOE_ERR_UNSUPPORTED_SHAPE),
])
def test_create_rejects_bad_config(kw, code):
    rc, h = _create(**kw)
    assert rc == code
    assert not h.value


@pytest.mark.parametrize("ep_size,ep_rank,kw,code", [
    (3, 0, {}, _lib.VMOE_ERR_INVALID_ARG),          # 4 experts over 3 ranks
    (2, 2, {}, _lib.VMOE_ERR_INVALID_ARG),          # rank out of range
    (2, 0, dict(capacity=8), _lib.VMOE_ERR_UNSUPPORTED_SHAPE),
    (2, 0, dict(dtype=_lib.VMOE_BF16, hidden=128), _lib.VMOE_ERR_UNSUPPORTED_SHAPE),
])
def test_create_ep_rejects_bad_partition(ep_size, ep_rank, kw, code):
    base = dict(hidden=64, inter=128, num_experts=4, top_k=2, lora_rank=16, lora_scaling=2.0,
                era_gamma=0.1, dtype=_lib.VMOE_F32, capacity=0)
    base.update(kw)
    cfg = _lib.VmoeConfig(**base)
    h = ctypes.c_void_p()
    assert _lib.load().vmoe_create_ep(ctypes.byref(cfg), 0, ep_size, ep_rank, ctypes.byref(h)) == code
    assert not h.value


def test_null_arguments_rejected():
    lib = _lib.load()
    assert lib.vmoe_create(None, 0, None) == _lib.VMOE_ERR_INVALID_ARG
    assert lib.vmoe_destroy(None) == _lib.VMOE_ERR_INVALID_ARG
    assert lib.vmoe_forward(None, None, 0, None, None, None, None, None, None, None, 0,
                            None) == _lib.VMOE_ERR_INVALID_ARG
    assert lib.vmoe_set_weights(None, None, None) == _lib.VMOE_ERR_INVALID_ARG


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_create_without_gpu_is_a_clean_error():
    rc, h = _create()
    assert rc == _lib.VMOE_ERR_CUDA and not h.value


def test_state_dict_keys_match_reference(golden_dir):
    ref = json.load(open(os.path.join(golden_dir, "state_dict_keys.json")))
    cfg = MoEConfig(**ref["config"])
    m = MoELayer(cfg)
    got = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert got == ref["keys"]


def test_feedforward_state_dict_keys_match_reference(golden_dir):
    from velvetoptimizer_b200 import FeedForward
    ref = json.load(open(os.path.join(golden_dir, "state_dict_keys.json")))
    m = FeedForward(MoEConfig(**ref["config"]))
    assert {k: list(v.shape) for k, v in m.state_dict().items()} == ref["ffn_keys"]


def test_config_validation_mirrors_reference():
    with pytest.raises(AssertionError):
        MoELayer(MoEConfig(moe_num_experts=4, moe_top_k=5))
    with pytest.raises(AssertionError):
        MoELayer(MoEConfig(moe_num_experts=1, moe_top_k=1))


def test_cpu_tensors_are_refused():
    m = MoELayer(MoEConfig(hidden_size=64, intermediate_size=128, moe_num_experts=4, moe_top_k=2))
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 3, 64))
