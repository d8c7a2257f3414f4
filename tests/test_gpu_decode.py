"""GPU parity of the decode-sized forward (at most 256 tokens, bf16) through the C ABI.

Such a batch runs the swapped-operand GEMMs: the packed weights are the MMA's M operand
and each expert's rows, padded to 16, its N operand.  Checked here against the oracle (the
fp32 numpy restatement of python/vesper/model.py:317-385 on the same bf16-rounded inputs,
within the bf16 tolerance 2e-2 norm-relative, on the GPU's own routing), against the
row-tiled GEMMs on the same inputs, and for the cases the kernel has to get right: a
single token, every expert full (N = 256), many empty experts, widths off the tile grid,
ERA tails, a token capacity, and the dense segments' padding rows never reaching the output.
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, bf16_inputs, make_inputs
from tests.abi_runner import AbiLayer
from tests.test_gpu_parity import check_dispatch

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2

DECODE_CASES = {
    "t64_e8k2_bias": MoECase(tokens=64, hidden=512, inter=1024, experts=8, top_k=2,
                             bias_std=0.05, seed=41),
    "t1_k1": MoECase(tokens=1, hidden=256, inter=384, experts=8, top_k=1, seed=42),
    # both experts take every token: two segments of 256 rows, the largest N
    "t256_all_rows": MoECase(tokens=256, hidden=256, inter=256, experts=2, top_k=2, seed=43),
    # 64 experts, top-8, Zipf router bias and FlyLoRA: many experts empty, small segments
    "t64_e64k8_lora_zipf": MoECase(tokens=64, hidden=256, inter=256, experts=64, top_k=8,
                                   lora_on=True, zipf_alpha=1.2, seed=44),
    "t17_odd_dims": MoECase(tokens=17, hidden=200, inter=136, experts=4, top_k=3, seed=45),
    "t100_era_tails": MoECase(tokens=100, hidden=256, inter=256, experts=4, top_k=2,
                              weight_std=0.3, bias_std=2.0, seed=46),
}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


@pytest.mark.parametrize("name", list(DECODE_CASES))
def test_decode_matches_oracle(name):
    case = DECODE_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, inp, "bf16")
    assert layer.handle.lib.vmoe_segment_align(layer.handle.ptr, case.tokens) == 16
    res = layer.run(inp["x"])
    ora = O.moe_forward(inp, case)
    tie = O.near_ties(ora["probs"], case.top_k, rel=1e-4)
    assert O.norm_rel_err(res["logits"], ora["logits"]) < 1e-4
    assert O.same_expert_sets(res["topk_idx"][~tie], ora["topk_idx"][~tie]).all()
    check_dispatch(layer, case.tokens, res, res["topk_idx"])
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"])
    err = O.norm_rel_err(res["out"], forced["out"])
    assert err < BF16_TOL, err
    assert abs(float(res["aux"]) - float(forced["aux"])) <= 1e-4 * abs(float(forced["aux"]))
    # bit-identical reruns
    again = layer.run(inp["x"])
    assert np.array_equal(again["out"], res["out"])
    layer.close()


@pytest.mark.parametrize("name", ["t64_e8k2_bias", "t64_e64k8_lora_zipf", "t256_all_rows"])
def test_decode_agrees_with_row_tiled_gemms(name, monkeypatch):
    """The same inputs through the row-tiled GEMMs and 128-token routing blocks (decode
    path switched off at handle creation): bit-identical router logits, routing and
    dispatch order (a token's logits do not depend on its routing block), outputs within
    the bf16 tolerance, and the aux loss within float rounding of the per-block sums."""
    case = DECODE_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    dec = AbiLayer(case, inp, "bf16")
    monkeypatch.setenv("VMOE_DECODE_MAX_TOKENS", "0")
    tiled = AbiLayer(case, inp, "bf16")
    monkeypatch.delenv("VMOE_DECODE_MAX_TOKENS")
    assert tiled.handle.lib.vmoe_segment_align(tiled.handle.ptr, case.tokens) in (128, 256)
    a, b = dec.run(inp["x"]), tiled.run(inp["x"])
    assert np.array_equal(a["logits"], b["logits"])
    assert np.array_equal(a["topk_idx"], b["topk_idx"])
    assert np.array_equal(a["topk_w"], b["topk_w"])
    assert np.array_equal(a["counts"], b["counts"])
    assert abs(float(a["aux"]) - float(b["aux"])) <= 1e-6 * abs(float(b["aux"]))
    assert O.norm_rel_err(a["out"], b["out"]) < BF16_TOL
    dec.close()
    tiled.close()


def test_decode_capacity_drops_late_tokens():
    case = MoECase(tokens=200, hidden=256, inter=256, experts=4, top_k=2, zipf_alpha=1.2, seed=47)
    inp = bf16_inputs(make_inputs(case))
    cap = 37  # not a multiple of 16: the last kept rows share a 16-row group with padding
    layer = AbiLayer(case, inp, "bf16", capacity=cap)
    assert layer.handle.lib.vmoe_segment_align(layer.handle.ptr, case.tokens) == 16
    res = layer.run(inp["x"])
    forced = O.moe_forward(inp, case, force_idx=res["topk_idx"], capacity=cap)
    assert O.norm_rel_err(res["out"], forced["out"]) < BF16_TOL
    assert res["counts"].sum() == case.tokens * case.top_k
    layer.close()


def test_decode_threshold_selects_the_path(monkeypatch):
    """At most 256 tokens take the decode GEMMs; more, or VMOE_DECODE_MAX_TOKENS below the
    batch, take the row-tiled ones; fp32 never does."""
    case = DECODE_CASES["t64_e8k2_bias"]
    inp = bf16_inputs(make_inputs(case))
    layer = AbiLayer(case, inp, "bf16")
    lib, hp = layer.handle.lib, layer.handle.ptr
    tile = lib.vmoe_gemm_tile_rows(hp)
    assert [lib.vmoe_segment_align(hp, t) for t in (0, 1, 256, 257)] == [tile, 16, 16, tile]
    layer.close()
    monkeypatch.setenv("VMOE_DECODE_MAX_TOKENS", "32")
    small = AbiLayer(case, inp, "bf16")
    assert small.handle.lib.vmoe_segment_align(small.handle.ptr, 32) == 16
    assert small.handle.lib.vmoe_segment_align(small.handle.ptr, 33) == tile
    small.close()
    monkeypatch.delenv("VMOE_DECODE_MAX_TOKENS")
    f32 = AbiLayer(case, make_inputs(case), "f32")
    assert f32.handle.lib.vmoe_segment_align(f32.handle.ptr, 64) == 128
    f32.close()


@pytest.mark.parametrize("name", ["t64_e8k2_bias", "t64_e64k8_lora_zipf", "t17_odd_dims"])
def test_decode_one_launch_equals_two(name, monkeypatch):
    """Both decode GEMMs in one launch (the down GEMM's work items wait on per-expert counts
    of stored gate|up blocks) give the same bits as the two GEMMs launched one after the
    other (VMOE_DECODE_FUSED=0)."""
    case = DECODE_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    fused = AbiLayer(case, inp, "bf16")
    monkeypatch.setenv("VMOE_DECODE_FUSED", "0")
    split = AbiLayer(case, inp, "bf16")
    monkeypatch.delenv("VMOE_DECODE_FUSED")
    ipad = -(-case.inter // 128) * 128
    one_launch = ipad // 64 <= -(-case.hidden // 64)  # down items no larger than gate|up ones
    for _ in range(2):  # the counters start from zero every forward
        a, b = fused.run(inp["x"]), split.run(inp["x"])
        assert np.array_equal(a["out"], b["out"])
        assert a["aux"] == b["aux"]
        n_fused, n_split = fused.handle.last_launch_count(), split.handle.last_launch_count()
        assert n_fused == n_split - (1 if one_launch else 0), (n_fused, n_split)
    fused.close()
    split.close()


@pytest.mark.parametrize("name", ["t64_e8k2_bias", "t64_e64k8_lora_zipf", "t256_all_rows"])
def test_decode_folded_plan_equals_plan_kernels(name, monkeypatch):
    """The decode forward derives the expert offsets, counts and aux loss inside its
    dispatch from the router's histograms; with the scan and plan kernels instead
    (VMOE_FOLD_PLAN=0) every output is the same to the bit and two more kernels launch."""
    case = DECODE_CASES[name]
    inp = bf16_inputs(make_inputs(case))
    folded = AbiLayer(case, inp, "bf16")
    monkeypatch.setenv("VMOE_FOLD_PLAN", "0")
    kernels = AbiLayer(case, inp, "bf16")
    monkeypatch.delenv("VMOE_FOLD_PLAN")
    for _ in range(2):
        a, b = folded.run(inp["x"]), kernels.run(inp["x"])
        for key in ("out", "logits", "topk_idx", "topk_w", "counts", "aux"):
            assert np.array_equal(a[key], b[key]), key
        check_dispatch(folded, case.tokens, a, a["topk_idx"])
        n_a, n_b = folded.handle.last_launch_count(), kernels.handle.last_launch_count()
        assert n_a == n_b - 2, (n_a, n_b)
    folded.close()
    kernels.close()


def test_decode_without_programmatic_dependent_launch(monkeypatch):
    """A decode forward launches its kernels with programmatic dependent launch (each waits
    for its predecessor before touching memory); without it (VMOE_PDL=0) the outputs are the
    same to the bit."""
    case = DECODE_CASES["t64_e8k2_bias"]
    inp = bf16_inputs(make_inputs(case))
    pdl = AbiLayer(case, inp, "bf16")
    monkeypatch.setenv("VMOE_PDL", "0")
    plain = AbiLayer(case, inp, "bf16")
    monkeypatch.delenv("VMOE_PDL")
    for _ in range(2):
        a, b = pdl.run(inp["x"]), plain.run(inp["x"])
        for key in ("out", "logits", "topk_idx", "topk_w", "counts", "aux"):
            assert np.array_equal(a[key], b[key]), key
    pdl.close()
    plain.close()
