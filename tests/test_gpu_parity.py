"""GPU parity: the CUDA path through the C ABI against the reference goldens and the oracle.

Tolerances (from the path's specification):
  * expert indices, per-expert counts and the dispatch permutation: bit-exact, except on
    tokens whose K-th and (K+1)-th router probabilities are a near-tie (counted, reported);
  * fp32: out, router logits and aux loss within 1e-5 norm-relative error
    (max|got - ref| / max|ref|) of the reference;
  * bf16: out within 2e-2 norm-relative of the fp32 oracle on the same bf16-rounded inputs.
"""
import dataclasses

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, bf16_inputs, make_inputs
from tests.abi_runner import AbiLayer
from tests.golden_io import ffn_golden_names, golden_names, load_golden

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-5
BF16_TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def permutation_from_slots(layer, T, res):
    """Read slot_of / expert offsets from the workspace; rebuild the token order per expert."""
    lay = layer.handle.workspace_layout(T)
    K, E = layer.case.top_k, layer.case.experts
    ws = layer.ws
    slot = ws[lay.slot_of:lay.slot_of + 4 * T * K].view(torch.int32).cpu().numpy().reshape(T, K)
    offs = ws[lay.expert_offsets:lay.expert_offsets + 4 * (E + 1)].view(torch.int32).cpu().numpy()
    return slot, offs


def check_dispatch(layer, T, res, oracle_idx):
    """Slots are expert-major, padded to the forward's segment alignment (whole GEMM tiles,
    or 16 rows for a decode-sized bf16 batch), token-ascending within each expert."""
    slot, offs = permutation_from_slots(layer, T, res)
    E = layer.case.experts
    counts, perm_tok, _ = O.dispatch(oracle_idx, E)
    assert np.array_equal(res["counts"], counts)
    align = layer.handle.lib.vmoe_segment_align(layer.handle.ptr, T)
    assert align in (16, 128, 256)
    assert (offs[1:] - offs[:-1] >= 0).all() and (offs % align == 0).all()
    got = []
    for e in range(E):
        rows = []
        for t in range(T):
            for k in range(layer.case.top_k):
                if oracle_idx[t, k] == e:
                    rows.append((slot[t, k], t))
        rows.sort()
        assert [r for r, _ in rows] == list(range(offs[e], offs[e] + counts[e]))
        got.extend(t for _, t in rows)
    assert np.array_equal(np.asarray(got), perm_tok)


# ----------------------------------------------------------------------------------------
# fp32 path against the reference's own outputs
# ----------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", golden_names())
def test_fp32_matches_reference_goldens(name):
    case, g = load_golden(name)
    inp = make_inputs(case)
    layer = AbiLayer(case, inp, "f32")
    res = layer.run(inp["x"])
    T, K = case.tokens, case.top_k

    assert O.norm_rel_err(res["logits"], g["logits"]) < FP32_TOL
    tie = O.near_ties(g["probs"], K, rel=1e-5)
    assert np.array_equal(res["topk_idx"][~tie], g["topk_idx"][~tie])
    # the GPU's own routing vs the oracle (lowest-index ties) on the same logits
    ora = O.moe_forward(inp, case)
    tie_o = O.near_ties(ora["probs"], K, rel=1e-5)
    assert np.array_equal(res["topk_idx"][~tie_o], ora["topk_idx"][~tie_o])
    check_dispatch(layer, T, res, res["topk_idx"])

    if not tie.any():
        assert O.norm_rel_err(res["out"], g["out"]) < FP32_TOL
        assert np.array_equal(res["counts"], g["counts"])
        assert abs(float(res["aux"]) - float(g["aux"])) <= FP32_TOL * abs(float(g["aux"]))
        assert O.norm_rel_err(res["topk_w"], g["topk_w"]) < FP32_TOL
    # downstream of routing, on the routing the GPU chose
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"])
    assert O.norm_rel_err(res["out"], forced["out"]) < FP32_TOL
    assert abs(float(res["aux"]) - float(forced["aux"])) <= FP32_TOL * abs(float(forced["aux"]))
    layer.close()


def test_fp32_tied_router_picks_lowest_index():
    case, g = load_golden("t64_tied_router")
    inp = make_inputs(case)
    layer = AbiLayer(case, inp, "f32")
    res = layer.run(inp["x"])
    assert (res["topk_idx"] == np.arange(case.top_k)).all()
    assert float(res["aux"]) == pytest.approx(1.0, abs=1e-6)
    layer.close()


def test_fp32_deterministic():
    case, _ = load_golden("t256_lora_zipf")
    inp = make_inputs(case)
    layer = AbiLayer(case, inp, "f32")
    a = layer.run(inp["x"])
    b = layer.run(inp["x"])
    for k in ("out", "topk_idx", "topk_w", "counts", "aux", "logits"):
        assert np.array_equal(a[k], b[k]), k
    layer.close()


# ----------------------------------------------------------------------------------------
# bf16 tensor-core path against the fp32 oracle on bf16-rounded inputs
# ----------------------------------------------------------------------------------------
BF16_CASES = {
    "small_e8k2": MoECase(tokens=256, hidden=256, inter=256, experts=8, top_k=2, seed=11),
    "ragged_bias": MoECase(tokens=1000, hidden=512, inter=384, experts=16, top_k=4,
                           bias_std=0.05, seed=12),
    "lora_zipf_e32k8": MoECase(tokens=512, hidden=256, inter=512, experts=32, top_k=8,
                               lora_on=True, zipf_alpha=1.2, seed=13),
    "odd_dims": MoECase(tokens=130, hidden=200, inter=136, experts=4, top_k=2, seed=14),
    "single_token_k_eq_e": MoECase(tokens=1, hidden=128, inter=256, experts=4, top_k=4, seed=15),
    "era_tails": MoECase(tokens=300, hidden=256, inter=256, experts=4, top_k=2, weight_std=0.3,
                         bias_std=2.0, seed=16),
}


@pytest.mark.parametrize("name", list(BF16_CASES))
def test_bf16_matches_oracle(name):
    case = BF16_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, inp, "bf16")
    res = layer.run(inp["x"])
    ora = O.moe_forward(inp, case)
    tie = O.near_ties(ora["probs"], case.top_k, rel=1e-4)
    assert O.norm_rel_err(res["logits"], ora["logits"]) < 1e-4
    assert O.same_expert_sets(res["topk_idx"][~tie], ora["topk_idx"][~tie]).all()
    assert O.order_follows_probs(res["topk_idx"], O.softmax(res["logits"]), rel=1e-5).all()
    check_dispatch(layer, case.tokens, res, res["topk_idx"])
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"])
    err = O.norm_rel_err(res["out"], forced["out"])
    assert err < BF16_TOL, err
    assert abs(float(res["aux"]) - float(forced["aux"])) <= 1e-4 * abs(float(forced["aux"]))
    layer.close()


@pytest.mark.parametrize("name", ["ragged_bias", "odd_dims"])
def test_bf16_single_cta_gemms_match_oracle(name, monkeypatch):
    # VMOE_PAIR_GEMM=0 selects the single-CTA tcgen05 GEMMs (128-row tiles) at handle creation
    monkeypatch.setenv("VMOE_PAIR_GEMM", "0")
    case = BF16_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, inp, "bf16")
    assert layer.handle.lib.vmoe_gemm_tile_rows(layer.handle.ptr) == 128
    res = layer.run(inp["x"])
    check_dispatch(layer, case.tokens, res, res["topk_idx"])
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"])
    err = O.norm_rel_err(res["out"], forced["out"])
    assert err < BF16_TOL, err
    assert abs(float(res["aux"]) - float(forced["aux"])) <= 1e-4 * abs(float(forced["aux"]))
    layer.close()


def test_bf16_deterministic():
    case = BF16_CASES["ragged_bias"]
    inp = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, inp, "bf16")
    a = layer.run(inp["x"])
    b = layer.run(inp["x"])
    for k in ("out", "topk_idx", "topk_w", "counts", "aux"):
        assert np.array_equal(a[k], b[k]), k
    layer.close()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_capacity_drops_late_tokens(dtype):
    case = MoECase(tokens=384, hidden=256, inter=256, experts=4, top_k=2, zipf_alpha=1.2, seed=21)
    inp = make_inputs(case)
    if dtype == "bf16":
        inp = bf16_inputs(inp)
    cap = 100
    layer = AbiLayer(case, inp, dtype, capacity=cap)
    res = layer.run(inp["x"])
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"], capacity=cap)
    tol = FP32_TOL if dtype == "f32" else BF16_TOL
    assert O.norm_rel_err(res["out"], forced["out"]) < tol
    # counts are reported before the capacity cut, as the reference's aux loss uses them
    assert res["counts"].sum() == case.tokens * case.top_k
    layer.close()


def test_empty_batch():
    case = BF16_CASES["small_e8k2"]
    layer = AbiLayer(case, bf16_inputs(make_inputs(case)), "bf16")
    res = layer.run(np.zeros((0, case.hidden), dtype=np.float32))
    assert res["out"].shape == (0, case.hidden)
    assert np.isnan(res["aux"])          # mean over zero tokens, as in the reference
    assert (res["counts"] == 0).all()
    layer.close()


def test_workspace_too_small_is_reported():
    from velvetoptimizer_b200 import _lib
    case = BF16_CASES["small_e8k2"]
    layer = AbiLayer(case, bf16_inputs(make_inputs(case)), "bf16")
    dev = torch.device("cuda", 0)
    x = torch.zeros(case.tokens, case.hidden, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    ws = torch.empty(1024, dtype=torch.uint8, device=dev)
    with pytest.raises(_lib.VmoeError) as ei:
        layer.handle.forward(x.data_ptr(), case.tokens, out.data_ptr(), None, None, None, None,
                             None, ws.data_ptr(), ws.numel(), 0)
    assert ei.value.code == _lib.VMOE_ERR_WORKSPACE
    layer.close()


# ----------------------------------------------------------------------------------------
# the drop-in module
# ----------------------------------------------------------------------------------------
def _module_state(case, inp, sd):
    """The reference state_dict keys of ``sd`` filled with the case's weights."""
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    new = dict(sd)
    new["router.weight"], new["router.bias"] = t(inp["w_r"]), t(inp["b_r"])
    for e in range(case.experts):
        for p, nm in (("g", "gate_proj"), ("u", "up_proj")):
            pre = f"experts.{e}.{nm}"
            new[f"{pre}.base.weight"], new[f"{pre}.base.bias"] = t(inp[f"w_{p}"][e]), t(inp[f"b_{p}"][e])
            new[f"{pre}.lora_down.weight"] = t(inp[f"a_{p}"][e])
            new[f"{pre}.lora_down.bias"] = t(inp[f"ba_{p}"][e])
            new[f"{pre}.lora_up.weight"] = t(inp[f"l_{p}"][e])
            new[f"{pre}.lora_up.bias"] = t(inp[f"bl_{p}"][e])
        new[f"experts.{e}.down_proj.weight"] = t(inp["w_d"][e])
        new[f"experts.{e}.down_proj.bias"] = t(inp["b_d"][e])
    return new


def _load_module(case, inp, dtype):
    from velvetoptimizer_b200 import MoEConfig, MoELayer
    cfg = MoEConfig(hidden_size=case.hidden, intermediate_size=case.inter,
                    moe_num_experts=case.experts, moe_top_k=case.top_k,
                    flylora_rank=case.lora_rank, flylora_alpha=case.lora_alpha,
                    era_gamma=case.era_gamma)
    m = MoELayer(cfg)
    m.load_state_dict(_module_state(case, inp, m.state_dict()))
    return m.cuda()


@torch.no_grad()
def test_module_fp32_matches_reference_c1():
    case, g = load_golden("c1_fp32")
    inp = make_inputs(case)
    m = _load_module(case, inp, torch.float32)
    x = torch.from_numpy(inp["x"]).reshape(case.batch, case.seq, case.hidden).cuda()
    out, aux = m(x)
    assert out.shape == (case.batch, case.seq, case.hidden) and out.dtype == torch.float32
    assert O.norm_rel_err(out.reshape(-1, case.hidden).cpu().numpy(), g["out"]) < FP32_TOL
    assert abs(aux.item() - float(g["aux"])) <= FP32_TOL * abs(float(g["aux"]))
    out2, aux2, logits = m(x, return_router_logits=True)
    assert torch.equal(out, out2)
    assert O.norm_rel_err(logits.reshape(-1, case.experts).cpu().numpy(), g["logits"]) < FP32_TOL
    # parameters changed after the first call are repacked on the next one
    with torch.no_grad():
        m.experts[0].down_proj.bias.add_(1.0)
    out3, _ = m(x)
    assert not torch.equal(out, out3)
    m.close()


@torch.no_grad()
def test_module_eager_call_equals_registered_op():
    """In eager mode the module runs the custom op's body directly; calling the registered op
    (the path a tracer takes) gives the same bits."""
    case = BF16_CASES["lora_zipf_e32k8"]
    inp = make_inputs(case)
    m = _load_module(case, inp, torch.bfloat16)
    x = torch.from_numpy(inp["x"]).reshape(1, case.tokens, case.hidden).cuda().to(torch.bfloat16)
    out, aux, logits = m(x, return_router_logits=True)
    packed = m.packed_for(x.device, x.dtype)
    out2, logits2, aux2 = torch.ops.vesper_moe.forward(x.reshape(case.tokens, case.hidden),
                                                        packed.id, True)
    assert torch.equal(out.reshape(case.tokens, case.hidden), out2)
    assert torch.equal(logits.reshape(case.tokens, case.experts), logits2)
    assert torch.equal(aux, aux2)
    m.close()


@torch.no_grad()
def test_module_bf16_lora_matches_oracle():
    case = BF16_CASES["lora_zipf_e32k8"]
    inp = make_inputs(case)
    m = _load_module(case, inp, torch.bfloat16)
    x = torch.from_numpy(inp["x"]).reshape(1, case.tokens, case.hidden).cuda().to(torch.bfloat16)
    out, aux, logits = m(x, return_router_logits=True)
    ib = bf16_inputs(inp)
    probs = O.softmax(logits.reshape(-1, case.experts).cpu().numpy())
    _, idx = O.topk_lowest_index(probs, case.top_k)
    forced = O.moe_forward(ib, case, force_idx=idx)
    assert O.norm_rel_err(out.float().reshape(-1, case.hidden).cpu().numpy(), forced["out"]) < BF16_TOL
    m.close()


class _DataWriteOptimizer(torch.optim.Optimizer):
    """Writes new parameter values through ``p.data`` inside ``step``, as VelvetOptimizer
    does (python/vesper/optimizer.py:176,212): no parameter version changes."""

    def __init__(self, named_params, new_state):
        self.names = {id(p): n for n, p in named_params}
        self.new_state = new_state
        super().__init__([p for _, p in named_params], {})

    @torch.no_grad()
    def step(self, closure=None):
        for group in self.param_groups:
            for p in group["params"]:
                p.data.copy_(self.new_state[self.names[id(p)]].to(p.device, p.dtype))


@torch.no_grad()
def test_module_repacks_after_optimizer_writes_through_data():
    """A training loop's optimizer step between two forwards: the second forward runs on the
    new weights (checked against the oracle on them), not on the first packing."""
    case = BF16_CASES["lora_zipf_e32k8"]
    inp = make_inputs(case)
    inp2 = make_inputs(dataclasses.replace(case, seed=case.seed + 101))
    inp2["x"] = inp["x"]
    m = _load_module(case, inp, torch.bfloat16)
    x = torch.from_numpy(inp["x"]).reshape(1, case.tokens, case.hidden).cuda().to(torch.bfloat16)
    out1, _ = m(x)
    opt = _DataWriteOptimizer(list(m.named_parameters()), _module_state(case, inp2, m.state_dict()))
    opt.step()
    out2, aux2, logits = m(x, return_router_logits=True)
    assert not torch.equal(out1, out2)
    probs = O.softmax(logits.reshape(-1, case.experts).cpu().numpy())
    _, idx = O.topk_lowest_index(probs, case.top_k)
    forced = O.moe_forward(bf16_inputs(inp2), case, force_idx=idx)
    assert O.norm_rel_err(out2.float().reshape(-1, case.hidden).cpu().numpy(), forced["out"]) < BF16_TOL
    # a raw write outside any optimizer step needs mark_weights_dirty()
    m.router.weight.data.copy_(torch.from_numpy(inp["w_r"]))
    m.mark_weights_dirty()
    _, _, logits3 = m(x, return_router_logits=True)
    mixed = dict(inp2, w_r=inp["w_r"])  # only the router weight was written back
    ref3 = O.moe_forward(bf16_inputs(mixed), case)["logits"]
    assert O.norm_rel_err(logits3.reshape(-1, case.experts).cpu().numpy(), ref3) < 1e-4
    m.close()


# ----------------------------------------------------------------------------------------
# the dense FeedForward (non-MoE layers) on the same GEMMs
# ----------------------------------------------------------------------------------------
def _ffn_run(case, inp, dtype):
    import ctypes
    from tests.abi_runner import abi_config, _WEIGHT_KEYS
    from velvetoptimizer_b200 import _lib
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    h = _lib.Handle(abi_config(case, dtype), 0, dense=True)
    dev = torch.device("cuda", 0)
    w = {k: torch.from_numpy(np.ascontiguousarray(inp[v])).to(dev, tdt)
         for k, v in _WEIGHT_KEYS.items() if not k.startswith("router")}
    stream = torch.cuda.current_stream(dev).cuda_stream
    h.set_weights(_lib.VmoeWeights(**{k: ctypes.c_void_p(t.data_ptr()) for k, t in w.items()}),
                  stream)
    x = torch.from_numpy(inp["x"]).to(dev, tdt)
    out = torch.empty_like(x)
    n = ctypes.c_size_t()
    _lib.check(h.lib.vmoe_ffn_workspace_size(h.ptr, x.shape[0], ctypes.byref(n)), h.ptr)
    ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
    _lib.check(h.lib.vmoe_ffn_forward(h.ptr, ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                      ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                      ws.numel(), ctypes.c_void_p(stream)), h.ptr)
    torch.cuda.synchronize()
    assert h.device_status(stream) == 0
    h.close()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("name", ffn_golden_names())
def test_ffn_fp32_matches_reference_goldens(name):
    case, g = load_golden(name)
    got = _ffn_run(case, make_inputs(case), "f32")
    assert O.norm_rel_err(got, g["out"]) < FP32_TOL


@pytest.mark.parametrize("case", [
    MoECase(tokens=300, hidden=256, inter=512, experts=1, top_k=1, lora_on=True, bias_std=0.05, seed=41),
    MoECase(tokens=77, hidden=200, inter=136, experts=1, top_k=1, seed=42),
])
def test_ffn_bf16_matches_oracle(case):
    inp = bf16_inputs(make_inputs(case))
    got = _ffn_run(case, inp, "bf16")
    assert O.norm_rel_err(got, O.ffn_forward(inp, case)) < BF16_TOL


def test_ffn_module_matches_reference_golden():
    from velvetoptimizer_b200 import FeedForward, MoEConfig
    case, g = load_golden("ffn_t64_lora_bias")
    inp = make_inputs(case)
    m = FeedForward(MoEConfig(hidden_size=case.hidden, intermediate_size=case.inter,
                              flylora_rank=case.lora_rank, flylora_alpha=case.lora_alpha,
                              era_gamma=case.era_gamma))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    sd = dict(m.state_dict())
    for p, nm in (("g", "gate_proj"), ("u", "up_proj")):
        sd[f"{nm}.base.weight"], sd[f"{nm}.base.bias"] = t(inp[f"w_{p}"][0]), t(inp[f"b_{p}"][0])
        sd[f"{nm}.lora_down.weight"], sd[f"{nm}.lora_down.bias"] = t(inp[f"a_{p}"][0]), t(inp[f"ba_{p}"][0])
        sd[f"{nm}.lora_up.weight"], sd[f"{nm}.lora_up.bias"] = t(inp[f"l_{p}"][0]), t(inp[f"bl_{p}"][0])
    sd["down_proj.weight"], sd["down_proj.bias"] = t(inp["w_d"][0]), t(inp["b_d"][0])
    m.load_state_dict(sd)
    m = m.cuda()
    x = torch.from_numpy(inp["x"]).reshape(case.batch, case.seq, case.hidden).cuda()
    out = m(x)
    assert out.shape == x.shape
    assert O.norm_rel_err(out.reshape(-1, case.hidden).cpu().numpy(), g["out"]) < FP32_TOL
    m.close()



def test_ffn_bf16_writes_only_its_rows():
    """The dense FFN reads x and writes out in place (no padded copies): rows past T of the
    caller's buffer are untouched and the result matches the oracle."""
    import ctypes
    from tests.abi_runner import abi_config, _WEIGHT_KEYS
    from velvetoptimizer_b200 import _lib
    case = MoECase(tokens=1000, hidden=512, inter=1024, experts=1, top_k=1, lora_on=True,
                   bias_std=0.05, seed=43)
    inp = bf16_inputs(make_inputs(case))
    dev = torch.device("cuda", 0)
    h = _lib.Handle(abi_config(case, "bf16"), 0, dense=True)
    w = {k: torch.from_numpy(np.ascontiguousarray(inp[v])).to(dev, torch.bfloat16)
         for k, v in _WEIGHT_KEYS.items() if not k.startswith("router")}
    stream = torch.cuda.current_stream(dev).cuda_stream
    h.set_weights(_lib.VmoeWeights(**{k: ctypes.c_void_p(t.data_ptr()) for k, t in w.items()}),
                  stream)
    T = case.tokens
    x = torch.from_numpy(inp["x"]).to(dev, torch.bfloat16)
    out = torch.full((T + 24, case.hidden), 7.0, dtype=torch.bfloat16, device=dev)
    n = ctypes.c_size_t()
    _lib.check(h.lib.vmoe_ffn_workspace_size(h.ptr, T, ctypes.byref(n)), h.ptr)
    ws = torch.empty(n.value, dtype=torch.uint8, device=dev)
    _lib.check(h.lib.vmoe_ffn_forward(h.ptr, ctypes.c_void_p(x.data_ptr()), T,
                                      ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                      ws.numel(), ctypes.c_void_p(stream)), h.ptr)
    torch.cuda.synchronize()
    assert h.device_status(stream) == 0
    assert bool((out[T:] == 7.0).all())
    got = out[:T].float().cpu().numpy()
    assert O.norm_rel_err(got, O.ffn_forward(inp, case)) < BF16_TOL
    h.close()


def test_banded_tile_order_is_bit_identical(monkeypatch):
    """The pair GEMMs may take each expert's output tiles in bands of n tiles (every m tile
    of the expert per band) instead of row-major; each tile is computed the same way in
    either order, so the outputs are the same to the bit.  Bands of 3 of the gate|up GEMM's
    8 n tiles leave a narrower last band; Zipf routing gives the experts runs of different
    lengths."""
    case = MoECase(tokens=2048, hidden=512, inter=1024, experts=4, top_k=2, zipf_alpha=1.2,
                   seed=61)
    inp = bf16_inputs(make_inputs(case))
    monkeypatch.setenv("VMOE_GEMM1_BAND", "0")
    monkeypatch.setenv("VMOE_GEMM2_BAND", "0")
    rowmajor = AbiLayer(case, inp, "bf16")
    monkeypatch.setenv("VMOE_GEMM1_BAND", "3")
    monkeypatch.setenv("VMOE_GEMM2_BAND", "1")
    banded = AbiLayer(case, inp, "bf16")
    monkeypatch.delenv("VMOE_GEMM1_BAND")
    monkeypatch.delenv("VMOE_GEMM2_BAND")
    assert rowmajor.handle.lib.vmoe_segment_align(rowmajor.handle.ptr, case.tokens) == 256
    a, b = rowmajor.run(inp["x"]), banded.run(inp["x"])
    assert np.array_equal(a["out"], b["out"])
    assert a["aux"] == b["aux"]
    forced = O.moe_forward(inp, case, force_idx=a["topk_idx"])
    assert O.norm_rel_err(b["out"], forced["out"]) < 2e-2
    rowmajor.close()
    banded.close()
