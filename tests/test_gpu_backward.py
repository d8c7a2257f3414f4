"""GPU: the MoE backward (vmoe_set_training / vmoe_forward_train / vmoe_backward).

Against the oracle backward (numpy fp32 autograd restatement, itself pinned to the
reference's autograd goldens at 1e-5) on the same bf16-rounded inputs and the GPU's own
routing, within the bf16 tolerance (2e-2 norm-relative): dx, the router's and every
expert's weight and bias gradients, and through the module also the FlyLoRA factors'.
Also: the training forward equals the inference forward bit for bit, reruns are
bit-identical, and edge shapes (K = 1, K = E, empty experts, ragged sizes, H and I off the
tile grid).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, backward_inputs, bf16_inputs, make_inputs, round_bf16
from tests.abi_runner import AbiLayer
from velvetoptimizer_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 2e-2
GRAD_KEYS = {"router_w": "dw_r", "router_b": "db_r", "gate_w": "dw_g", "gate_b": "db_g",
             "up_w": "dw_u", "up_b": "db_u", "down_w": "dw_d", "down_b": "db_d"}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def train_step(layer: AbiLayer, x_np, dout_np, daux):
    """forward_train + backward through the C ABI; numpy results."""
    c = layer.case
    h = layer.handle
    dev = torch.device("cuda", layer.device)
    s = torch.cuda.current_stream(dev)
    h.set_training(True, s.cuda_stream)
    x = torch.from_numpy(np.ascontiguousarray(x_np)).to(dev, torch.bfloat16)
    T = x.shape[0]
    saved_b, scratch_b = h.train_workspace_size(T)
    saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
    scratch = torch.empty(scratch_b, dtype=torch.uint8, device=dev)
    out = torch.empty_like(x)
    logits = torch.empty((T, c.experts), dtype=torch.float32, device=dev)
    aux = torch.empty((1,), dtype=torch.float32, device=dev)
    h.forward_train(x.data_ptr(), T, out.data_ptr(), logits.data_ptr(), aux.data_ptr(),
                    saved.data_ptr(), saved_b, s.cuda_stream)
    dout = torch.from_numpy(np.ascontiguousarray(dout_np)).to(dev, torch.bfloat16)
    daux_t = torch.tensor([daux], dtype=torch.float32, device=dev)
    E, H, I = c.experts, c.hidden, c.inter
    f = dict(device=dev, dtype=torch.float32)
    g = {"router_w": torch.full((E, H), np.nan, **f), "router_b": torch.full((E,), np.nan, **f),
         "gate_w": torch.full((E, I, H), np.nan, **f), "gate_b": torch.full((E, I), np.nan, **f),
         "up_w": torch.full((E, I, H), np.nan, **f), "up_b": torch.full((E, I), np.nan, **f),
         "down_w": torch.full((E, H, I), np.nan, **f), "down_b": torch.full((E, H), np.nan, **f)}
    dx = torch.empty_like(x)
    vg = _lib.VmoeGrads(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in g.items()})
    h.backward(x.data_ptr(), dout.data_ptr(), T, daux_t.data_ptr(), dx.data_ptr(), vg,
               saved.data_ptr(), saved_b, scratch.data_ptr(), scratch_b, s.cuda_stream)
    s.synchronize()
    assert h.device_status(s.cuda_stream) == 0
    r = {k: v.cpu().numpy() for k, v in g.items()}
    r["dx"] = dx.float().cpu().numpy()
    r["out"] = out.float().cpu().numpy()
    r["logits"] = logits.cpu().numpy()
    r["aux"] = float(aux.item())
    return r


CASES = {
    "e8k2_lora_bias": MoECase(tokens=300, hidden=256, inter=384, experts=8, top_k=2,
                              lora_on=True, bias_std=0.05, seed=61),
    "e16k4_h320": MoECase(tokens=200, hidden=320, inter=256, experts=16, top_k=4, seed=62),
    "e4k1": MoECase(tokens=129, hidden=128, inter=128, experts=4, top_k=1, bias_std=0.05, seed=63),
    "e16k1_empty_experts": MoECase(tokens=5, hidden=128, inter=128, experts=16, top_k=1, seed=64),
    "e2k2_k_eq_e": MoECase(tokens=64, hidden=128, inter=256, experts=2, top_k=2, seed=65),
    "e64k4_t1000": MoECase(tokens=1000, hidden=512, inter=256, experts=64, top_k=4, seed=66),
}


@pytest.mark.parametrize("name", list(CASES))
def test_backward_against_oracle(name):
    case = CASES[name]
    p = bf16_inputs(make_inputs(case))
    dout, daux = backward_inputs(case)
    dout = round_bf16(dout)
    layer = AbiLayer(case, p, "bf16")
    ref_fwd = layer.run(p["x"])  # the inference forward (and the GPU's routing)
    r = train_step(layer, p["x"], dout, daux)
    # the training forward is the inference forward
    assert np.array_equal(r["out"], ref_fwd["out"])
    assert r["aux"] == float(ref_fwd["aux"])
    assert np.array_equal(r["logits"], ref_fwd["logits"])
    ora = O.moe_backward(p, case, dout, daux, force_idx=ref_fwd["topk_idx"])
    errs = {"dx": O.norm_rel_err(r["dx"], ora["dx"])}
    for k, ok in GRAD_KEYS.items():
        assert np.isfinite(r[k]).all(), k
        errs[k] = O.norm_rel_err(r[k], ora[ok])
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, (bad, errs)
    # determinism: a second step is bit-identical
    r2 = train_step(layer, p["x"], dout, daux)
    for k in list(GRAD_KEYS) + ["dx"]:
        assert np.array_equal(r[k], r2[k]), k
    layer.close()


def test_backward_rejects_fp32_and_missing_training():
    case = CASES["e4k1"]
    p = make_inputs(case)
    layer = AbiLayer(case, p, "f32")
    s = torch.cuda.current_stream().cuda_stream
    with pytest.raises(_lib.VmoeError):
        layer.handle.set_training(True, s)
    layer.close()
    lb = AbiLayer(case, bf16_inputs(p), "bf16")
    dev = torch.device("cuda", 0)
    x = torch.zeros((case.tokens, case.hidden), dtype=torch.bfloat16, device=dev)
    saved_b, _ = lb.handle.train_workspace_size(case.tokens)
    saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
    with pytest.raises(_lib.VmoeError):  # vmoe_set_training not called
        lb.handle.forward_train(x.data_ptr(), case.tokens, x.data_ptr(), None, None,
                                saved.data_ptr(), saved_b, s)
    lb.close()


def test_module_autograd_against_oracle():
    """MoELayer (fp32 parameters, bf16 activations, as under the reference's bf16 autocast):
    loss.backward() fills every parameter's .grad, FlyLoRA factors included."""
    from velvetoptimizer_b200 import MoEConfig, MoELayer
    case = CASES["e8k2_lora_bias"]
    inp = make_inputs(case)
    ib = bf16_inputs(inp)
    cfg = MoEConfig(hidden_size=case.hidden, intermediate_size=case.inter,
                    moe_num_experts=case.experts, moe_top_k=case.top_k,
                    flylora_rank=case.lora_rank, flylora_alpha=case.lora_alpha,
                    era_gamma=case.era_gamma)
    m = MoELayer(cfg)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    sd = dict(m.state_dict())
    sd["router.weight"], sd["router.bias"] = t(ib["w_r"]), t(ib["b_r"])
    for e in range(case.experts):
        for q, nm in (("g", "gate_proj"), ("u", "up_proj")):
            pre = f"experts.{e}.{nm}"
            sd[f"{pre}.base.weight"], sd[f"{pre}.base.bias"] = t(ib[f"w_{q}"][e]), t(ib[f"b_{q}"][e])
            sd[f"{pre}.lora_down.weight"], sd[f"{pre}.lora_down.bias"] = t(ib[f"a_{q}"][e]), t(ib[f"ba_{q}"][e])
            sd[f"{pre}.lora_up.weight"], sd[f"{pre}.lora_up.bias"] = t(ib[f"l_{q}"][e]), t(ib[f"bl_{q}"][e])
        sd[f"experts.{e}.down_proj.weight"] = t(ib["w_d"][e])
        sd[f"experts.{e}.down_proj.bias"] = t(ib["b_d"][e])
    m.load_state_dict(sd)
    m = m.cuda()
    dout, daux = backward_inputs(case)
    dout = round_bf16(dout)
    x = torch.from_numpy(ib["x"]).reshape(1, case.tokens, case.hidden).cuda().to(torch.bfloat16)
    x.requires_grad_(True)
    out, aux, logits = m(x, return_router_logits=True)
    loss = (out.float() * torch.from_numpy(dout).cuda().reshape(out.shape)).sum() + float(daux) * aux
    loss.backward()
    probs = O.softmax(logits.detach().reshape(-1, case.experts).cpu().numpy())
    _, idx = O.topk_lowest_index(probs, case.top_k)
    ora = O.moe_backward(ib, case, dout, daux, force_idx=idx)
    errs = {"dx": O.norm_rel_err(x.grad.float().reshape(-1, case.hidden).cpu().numpy(), ora["dx"]),
            "dw_r": O.norm_rel_err(m.router.weight.grad.cpu().numpy(), ora["dw_r"]),
            "db_r": O.norm_rel_err(m.router.bias.grad.cpu().numpy(), ora["db_r"])}
    for q, nm in (("g", "gate_proj"), ("u", "up_proj")):
        for key, get in ((f"dw_{q}", lambda pr: pr.base.weight), (f"db_{q}", lambda pr: pr.base.bias),
                         (f"da_{q}", lambda pr: pr.lora_down.weight), (f"dba_{q}", lambda pr: pr.lora_down.bias),
                         (f"dl_{q}", lambda pr: pr.lora_up.weight), (f"dbl_{q}", lambda pr: pr.lora_up.bias)):
            got = np.stack([get(getattr(e, nm)).grad.cpu().numpy() for e in m.experts])
            errs[key] = O.norm_rel_err(got, ora[key])
    errs["dw_d"] = O.norm_rel_err(np.stack([e.down_proj.weight.grad.cpu().numpy() for e in m.experts]), ora["dw_d"])
    errs["db_d"] = O.norm_rel_err(np.stack([e.down_proj.bias.grad.cpu().numpy() for e in m.experts]), ora["db_d"])
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, (bad, errs)
    assert m.experts[0].gate_proj.proj_a.grad is None  # a buffer
    m.close()


def test_pair_and_single_cta_weight_gradients_agree(monkeypatch):
    """The CTA-pair weight-gradient GEMM (default) against the single-CTA one."""
    case = CASES["e8k2_lora_bias"]
    p = bf16_inputs(make_inputs(case))
    dout, daux = backward_inputs(case)
    dout = round_bf16(dout)
    layer = AbiLayer(case, p, "bf16")
    monkeypatch.setenv("VMOE_PAIR_WGRAD", "0")
    single = train_step(layer, p["x"], dout, daux)
    monkeypatch.setenv("VMOE_PAIR_WGRAD", "1")
    pair = train_step(layer, p["x"], dout, daux)
    for k in GRAD_KEYS:
        assert O.norm_rel_err(pair[k], single[k]) < 1e-6, k
    assert np.array_equal(pair["dx"], single["dx"])
    layer.close()
