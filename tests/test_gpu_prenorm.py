"""GPU: the fused pre-norm block (vmoe_set_norm + vmoe_forward_residual).

out = x + MoE(LayerNorm(x)), the FFN half of the reference's TransformerLayer.forward
(python/vesper/model.py:418-425), with the LayerNorm folded into the router's and the
dispatch's reads and the residual add into the combine.  Checked against the reference's
own outputs (fp32 goldens, 1e-5) and the oracle (bf16, 2e-2 on the GPU's routing), on both
routers: the tensor-core router (bf16, E <= 64: row statistics from MMAs on the x tile,
folded weights) and the CUDA-core router (fp32, or E > 64: statistics pass, normalised
loads).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, bf16_inputs, make_inputs, make_norm_inputs, round_bf16
from tests.abi_runner import AbiLayer
from tests.golden_io import ln_golden_names, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def run_residual(layer, x_np, ln_w, ln_b, eps, inplace=False):
    c = layer.case
    dev = torch.device("cuda", layer.device)
    s = torch.cuda.current_stream(dev)
    w = torch.from_numpy(ln_w).to(dev, layer.tdtype)
    b = torch.from_numpy(ln_b).to(dev, layer.tdtype)
    layer.handle.set_norm(w.data_ptr(), b.data_ptr(), float(eps), s.cuda_stream)
    x = torch.from_numpy(np.ascontiguousarray(x_np)).to(dev, layer.tdtype)
    T = x.shape[0]
    need = layer.handle.workspace_size(T)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
    out = x if inplace else torch.empty_like(x)
    r = {"logits": torch.empty((T, c.experts), dtype=torch.float32, device=dev),
         "idx": torch.empty((T, c.top_k), dtype=torch.int32, device=dev),
         "w": torch.empty((T, c.top_k), dtype=torch.float32, device=dev),
         "counts": torch.empty((c.experts,), dtype=torch.int32, device=dev),
         "aux": torch.empty((1,), dtype=torch.float32, device=dev)}
    layer.handle.forward_residual(x.data_ptr(), T, out.data_ptr(), r["logits"].data_ptr(),
                                  r["idx"].data_ptr(), r["w"].data_ptr(), r["counts"].data_ptr(),
                                  r["aux"].data_ptr(), ws.data_ptr(), ws.numel(), s.cuda_stream)
    s.synchronize()
    assert layer.handle.device_status(s.cuda_stream) == 0
    res = {k: v.cpu().numpy() for k, v in r.items()}
    res["out"] = out.float().cpu().numpy()
    res["idx"] = res["idx"].astype(np.int64)
    res["aux"] = float(res["aux"][0])
    lay = layer.handle.workspace_layout(T)
    stats_off = lay.slot_of + ((4 * T * c.top_k + 255) // 256) * 256
    res["stats"] = ws[stats_off:stats_off + 8 * T].view(torch.float32).cpu().numpy().reshape(T, 2)
    return res


@pytest.mark.parametrize("name", ln_golden_names())
def test_fp32_prenorm_matches_reference_goldens(name):
    case, g = load_golden(name)
    p = make_inputs(case)
    ni = make_norm_inputs(case)
    layer = AbiLayer(case, p, "f32")
    res = run_residual(layer, ni["x"], ni["ln_w"], ni["ln_b"], ni["eps"])
    assert O.norm_rel_err(res["logits"], g["logits"]) < 1e-5
    assert O.norm_rel_err(res["out"], g["out"]) < 1e-5
    assert abs(res["aux"] - float(g["aux"])) <= 1e-5 * abs(float(g["aux"]))
    # the statistics pass: mean and 1/sqrt(var + eps) of every residual row
    x64 = ni["x"].astype(np.float64)
    mu, var = x64.mean(-1), x64.var(-1)
    assert np.allclose(res["stats"][:, 0], mu, rtol=1e-5, atol=1e-5)
    assert np.allclose(res["stats"][:, 1], 1 / np.sqrt(var + float(ni["eps"])), rtol=1e-5)
    layer.close()


BF16_CASES = {
    # tensor-core router (E <= 64): statistics from the MMAs, folded router weights
    "tc_e16k4_ragged": MoECase(tokens=1000, hidden=256, inter=384, experts=16, top_k=4,
                               bias_std=0.02, seed=41),
    "tc_e64k2_lora": MoECase(tokens=700, hidden=512, inter=256, experts=64, top_k=2,
                             lora_on=True, seed=42),
    "tc_e8k2_h1024": MoECase(tokens=300, hidden=1024, inter=512, experts=8, top_k=2, seed=43),
    # decode-sized batches: routing blocks of 16 / 32 tokens copied by all the router's threads
    "tc_e8k2_decode48": MoECase(tokens=48, hidden=512, inter=256, experts=8, top_k=2, seed=45),
    "tc_e16k4_decode200": MoECase(tokens=200, hidden=256, inter=384, experts=16, top_k=4,
                                  seed=46),
    # CUDA-core router (E > 64) on bf16 inputs
    "simt_e80k2": MoECase(tokens=333, hidden=256, inter=256, experts=80, top_k=2, seed=44),
}


@pytest.mark.parametrize("name", list(BF16_CASES))
def test_bf16_prenorm_against_oracle(name):
    case = BF16_CASES[name]
    p = bf16_inputs(make_inputs(case))
    ni = make_norm_inputs(case)
    x, ln_w, ln_b = round_bf16(ni["x"]), round_bf16(ni["ln_w"]), round_bf16(ni["ln_b"])
    layer = AbiLayer(case, p, "bf16")
    res = run_residual(layer, x, ln_w, ln_b, ni["eps"])
    q = dict(p)
    q["x"] = x
    ora = O.prenorm_moe_forward(q, case, ln_w, ln_b, ni["eps"])
    # statistics (the tensor-core router forms them from bf16 x on the tensor cores)
    x64 = x.astype(np.float64)
    assert np.allclose(res["stats"][:, 0], x64.mean(-1), rtol=1e-4, atol=1e-4)
    assert np.allclose(res["stats"][:, 1], 1 / np.sqrt(x64.var(-1) + float(ni["eps"])), rtol=1e-4)
    # routing of LayerNorm(x): logits within bf16 rounding of the normalised rows / weights
    assert O.norm_rel_err(res["logits"], ora["logits"]) < 1e-2
    tie = O.near_ties(ora["probs"], case.top_k, rel=2e-2)
    assert tie.mean() < 0.5
    assert O.same_expert_sets(res["idx"][~tie], ora["topk_idx"][~tie]).all()
    # outputs on the GPU's own routing
    forced = O.prenorm_moe_forward(q, case, ln_w, ln_b, ni["eps"], force_idx=res["idx"])
    assert O.norm_rel_err(res["out"], forced["out"]) < 2e-2
    # the FFN part: out = bf16(x + bf16(ffn)) as the reference's bf16 residual add rounds;
    # within one bf16 ulp of that plus the bf16 tolerance on the FFN output itself
    ffn = forced["out"] - x
    expect = round_bf16(x + round_bf16(ffn))
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(expect), 1e-30))) - 7)
    assert (np.abs(res["out"] - expect) <= ulp + 2e-2 * np.abs(ffn).max()).all()
    # in place (out == x) gives the same bits, and reruns are deterministic
    res2 = run_residual(layer, x, ln_w, ln_b, ni["eps"], inplace=True)
    assert np.array_equal(res2["out"], res["out"]) and np.array_equal(res2["idx"], res["idx"])
    layer.close()


@torch.no_grad()
def test_module_forward_residual_matches_unfused():
    from velvetoptimizer_b200 import MoEConfig, MoELayer
    cfg = MoEConfig(hidden_size=256, intermediate_size=384, moe_num_experts=8, moe_top_k=2)
    torch.manual_seed(3)
    dev = torch.device("cuda", 0)
    layer = MoELayer(cfg).to(dev)
    norm = torch.nn.LayerNorm(256, eps=1e-6).to(dev)
    with torch.no_grad():
        norm.weight.normal_(1.0, 0.1)
        norm.bias.normal_(0.0, 0.1)
    x = (2 * torch.randn(2, 300, 256, device=dev) + torch.randn(2, 300, 1, device=dev))
    out_f, aux_f = layer.forward_residual(x, norm)
    out_u, aux_u = layer(norm(x))
    out_u = x + out_u
    assert (out_f - out_u).abs().max().item() <= 1e-5 * out_u.abs().max().item()
    assert abs(aux_f.item() - aux_u.item()) <= 1e-5 * abs(aux_u.item())
    # a changed norm is picked up
    with torch.no_grad():
        norm.bias.add_(0.5)
    out_f2, _ = layer.forward_residual(x, norm)
    out_u2 = x + layer(norm(x))[0]
    assert (out_f2 - out_u2).abs().max().item() <= 1e-5 * out_u2.abs().max().item()
    # bf16: fused vs unfused (torch LayerNorm, the module, torch add) on the tokens whose
    # expert sets agree -- bf16 rounding of the normalised rows vs of the folded router
    # weights may flip near-tied tokens, whose outputs then differ by a whole expert
    lb, nb = layer.to(torch.bfloat16), norm.to(torch.bfloat16)
    xb = x.to(torch.bfloat16)
    ob, _, lg_f = lb.forward_residual(xb, nb, return_router_logits=True)
    ou, _, lg_u = lb(nb(xb), return_router_logits=True)
    ou = xb + ou
    k = cfg.moe_top_k
    same = (lg_f.topk(k, -1).indices.sort(-1).values == lg_u.topk(k, -1).indices.sort(-1).values).all(-1)
    assert same.float().mean().item() > 0.95
    diff = (ob.float() - ou.float())[same]
    err = diff.abs().max().item() / ou.float().abs().max().item()
    assert err < 2e-2, err
