"""GPU: the host-buffer forward (vmoe_forward_host) against the device forward and goldens.

The chunked copy-in / forward / copy-out pipeline must give outputs bit-identical to
vmoe_forward on the same tokens (every token's routing, GEMM rows and combine order are
independent of the chunk it lands in) and the aux loss of the whole batch (within 1e-6
relative: the chunks' probability sums are added in a different order).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, bf16_inputs, make_inputs
from tests.abi_runner import AbiLayer
from tests.golden_io import load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def host_run(layer, x_host: torch.Tensor, chunks: int):
    h = layer.handle
    T = x_host.shape[0]
    dev = torch.device("cuda", layer.device)
    ws = torch.empty(h.host_workspace_size(T, chunks), dtype=torch.uint8, device=dev)
    out = torch.empty(x_host.shape, dtype=x_host.dtype, pin_memory=x_host.is_pinned())
    aux = torch.full((), 7.0, dtype=torch.float32, pin_memory=True)
    s = torch.cuda.current_stream(dev)
    h.forward_host(x_host.data_ptr(), T, out.data_ptr(), aux.data_ptr(), chunks, ws.data_ptr(),
                   ws.numel(), s.cuda_stream)
    s.synchronize()
    assert h.device_status(s.cuda_stream) == 0
    return out, float(aux)


@pytest.mark.parametrize("chunks", [0, 1, 3, 16])
def test_host_forward_bit_identical_bf16(chunks):
    case = MoECase(tokens=3000, hidden=256, inter=384, experts=8, top_k=2, bias_std=0.02, seed=5)
    p = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, p, "bf16")
    dev = torch.device("cuda", 0)
    x_dev = torch.from_numpy(p["x"]).to(dev, torch.bfloat16)
    ref = layer.run_device(x_dev)
    torch.cuda.synchronize()
    out, aux = host_run(layer, x_dev.cpu().pin_memory(), chunks)
    assert torch.equal(out, ref["out"].cpu())
    ref_aux = float(ref["aux"].item())
    assert abs(aux - ref_aux) <= 1e-6 * abs(ref_aux)


def test_host_forward_fp32_golden():
    case, g = load_golden("c1_fp32")
    p = make_inputs(case)
    layer = AbiLayer(case, p, "f32")
    x = torch.from_numpy(np.ascontiguousarray(p["x"])).float().pin_memory()
    out, aux = host_run(layer, x, 2)
    assert O.norm_rel_err(out.numpy(), g["out"]) < 1e-5
    assert abs(aux - float(g["aux"])) <= 1e-5 * abs(float(g["aux"]))


def test_host_forward_pageable_and_empty():
    case = MoECase(tokens=257, hidden=128, inter=256, experts=4, top_k=2, seed=2)
    p = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, p, "bf16")
    dev = torch.device("cuda", 0)
    x_dev = torch.from_numpy(p["x"]).to(dev, torch.bfloat16)
    ref = layer.run_device(x_dev)
    torch.cuda.synchronize()
    out, _ = host_run(layer, x_dev.cpu(), 2)  # pageable host memory: correct, not overlapped
    assert torch.equal(out, ref["out"].cpu())
    _, aux = host_run(layer, x_dev.cpu()[:0], 0)
    assert np.isnan(aux)


def test_module_forward_host_matches_forward():
    from velvetoptimizer_b200 import MoEConfig, MoELayer
    cfg = MoEConfig(hidden_size=256, intermediate_size=512, moe_num_experts=8, moe_top_k=2)
    torch.manual_seed(0)
    layer = MoELayer(cfg).cuda().to(torch.bfloat16)
    x = torch.randn(4, 600, 256).to(torch.bfloat16)
    with torch.no_grad():
        out_d, aux_d = layer(x.cuda())
    out_h, aux_h = layer.forward_host(x.pin_memory(), chunks=4)
    assert out_h.device.type == "cpu"
    assert torch.equal(out_h, out_d.cpu())
    assert abs(float(aux_h) - float(aux_d)) <= 1e-6 * abs(float(aux_d))


@pytest.mark.parametrize("chunks", [2, 5])
def test_host_forward_carry_skewed_many_experts(chunks):
    # 64 experts, Zipf-skewed: small experts' segments are carried from chunk to chunk
    # (and the last chunk pads them), large ones split into whole tiles plus a remainder
    case = MoECase(tokens=6000, hidden=256, inter=256, experts=64, top_k=4, zipf_alpha=1.2,
                   bias_std=0.02, seed=11)
    p = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, p, "bf16")
    dev = torch.device("cuda", 0)
    x_dev = torch.from_numpy(p["x"]).to(dev, torch.bfloat16)
    ref = layer.run_device(x_dev)
    torch.cuda.synchronize()
    out, aux = host_run(layer, x_dev.cpu().pin_memory(), chunks)
    assert torch.equal(out, ref["out"].cpu())
    ref_aux = float(ref["aux"].item())
    assert abs(aux - ref_aux) <= 1e-6 * abs(ref_aux)


def test_host_forward_capacity_is_one_batch():
    # a token capacity applies to the whole batch, so the host forward must not cut it into
    # chunks that would each drop their own late tokens
    case = MoECase(tokens=1500, hidden=128, inter=256, experts=4, top_k=2, seed=3)
    p = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, p, "bf16", capacity=500)
    dev = torch.device("cuda", 0)
    x_dev = torch.from_numpy(p["x"]).to(dev, torch.bfloat16)
    ref = layer.run_device(x_dev)
    torch.cuda.synchronize()
    out, _ = host_run(layer, x_dev.cpu().pin_memory(), 4)
    assert torch.equal(out, ref["out"].cpu())
