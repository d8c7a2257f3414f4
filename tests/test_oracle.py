"""Pin the CPU oracle against the reference's own outputs (golden vectors).

The reference ships no golden vectors or value-level tests for this path (its Rust tests
use all-zero weights and check shapes and ``aux >= 0``), so the goldens here were made by
executing the reference ``MoELayer`` (tests/golden/make_golden.py).  These tests run on
CPU only.
"""
import numpy as np
import pytest

from oracle import moe_oracle as O
from oracle.inputs import make_inputs, round_bf16
from tests.golden_io import (bw_golden_names, ffn_golden_names, golden_names, ln_golden_names,
                              load_golden)

NAMES = golden_names()


def test_goldens_present():
    assert "c1_fp32" in NAMES and len(NAMES) >= 8
    assert len(ffn_golden_names()) >= 2
    assert len(ln_golden_names()) >= 2
    assert len(bw_golden_names()) >= 3


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference(name):
    case, g = load_golden(name)
    inp = make_inputs(case)
    res = O.moe_forward(inp, case)
    T, K = case.tokens, case.top_k

    # router logits / probabilities: fp32, different summation order only
    assert O.norm_rel_err(res["logits"], g["logits"]) < 1e-5
    assert O.norm_rel_err(res["probs"], g["probs"]) < 1e-5

    # routing: bit-exact on every token without a (near-)tie at the K boundary
    tie = O.near_ties(g["probs"], K, rel=1e-6)
    ok = ~tie
    assert np.array_equal(res["topk_idx"][ok], g["topk_idx"][ok])
    if not tie.any():
        assert np.array_equal(res["counts"], g["counts"])
        assert np.array_equal(res["perm_tok"], g["perm_tok"])

    # everything downstream of routing, on the reference's own routing
    forced = O.moe_forward(inp, case, force_idx=g["topk_idx"])
    assert np.array_equal(forced["counts"], g["counts"])
    assert np.array_equal(forced["perm_tok"], g["perm_tok"])
    assert O.norm_rel_err(forced["topk_w"], g["topk_w"]) < 1e-6
    assert O.norm_rel_err(forced["out"], g["out"]) < 1e-5
    assert abs(float(forced["aux"]) - float(g["aux"])) <= 1e-5 * abs(float(g["aux"]))
    if not tie.any():
        assert O.norm_rel_err(res["out"], g["out"]) < 1e-5


@pytest.mark.parametrize("name", ffn_golden_names())
def test_oracle_ffn_matches_reference(name):
    # the reference's dense FeedForward (python/vesper/model.py:249-270)
    case, g = load_golden(name)
    out = O.ffn_forward(make_inputs(case), case)
    assert O.norm_rel_err(out, g["out"]) < 1e-5


@pytest.mark.parametrize("name", ln_golden_names())
def test_oracle_prenorm_matches_reference(name):
    # ffn_norm + MoELayer + residual as TransformerLayer.forward (python/vesper/model.py:418-425)
    from oracle.inputs import make_norm_inputs
    case, g = load_golden(name)
    ni = make_norm_inputs(case)
    p = make_inputs(case)
    p["x"] = ni["x"]
    res = O.prenorm_moe_forward(p, case, ni["ln_w"], ni["ln_b"], ni["eps"])
    assert O.norm_rel_err(res["normed"], g["normed"]) < 1e-5
    assert O.norm_rel_err(res["logits"], g["logits"]) < 1e-5
    assert not O.near_ties(g["probs"], case.top_k, rel=1e-5).any()
    assert O.norm_rel_err(res["out"], g["out"]) < 1e-5
    assert abs(float(res["aux"]) - float(g["aux"])) <= 1e-5 * abs(float(g["aux"]))


BW_KEYS = ("dx", "dw_r", "db_r", "dw_g", "db_g", "dw_u", "db_u", "dw_d", "db_d", "da_g", "dba_g",
           "dl_g", "dbl_g", "da_u", "dba_u", "dl_u", "dbl_u")


@pytest.mark.parametrize("name", bw_golden_names())
def test_oracle_backward_matches_reference_autograd(name):
    # autograd through the reference MoELayer for L = <out, dout> + daux * aux
    from oracle.inputs import backward_inputs
    case, g = load_golden(name)
    assert not O.near_ties(g["probs"], case.top_k, rel=1e-5).any()
    dout, daux = backward_inputs(case)
    res = O.moe_backward(make_inputs(case), case, dout, daux)
    for k in BW_KEYS:
        err = O.norm_rel_err(res[k], g[k])
        assert err < 1e-5, (k, err)


def test_tied_router_case_is_all_ties():
    # All-zero router weights: every probability is 1/E, torch.topk picks an
    # implementation-defined pair, the oracle picks experts 0..K-1.
    case, g = load_golden("t64_tied_router")
    assert O.near_ties(g["probs"], case.top_k).all()
    res = O.moe_forward(make_inputs(case), case)
    assert (res["topk_idx"] == np.arange(case.top_k)).all()
    # aux = E * sum_e f_e / E = 1 exactly, whichever experts are picked
    assert float(res["aux"]) == pytest.approx(1.0, abs=1e-6)
    assert float(g["aux"]) == pytest.approx(1.0, abs=1e-6)


def test_c1_no_ties_and_counts():
    case, g = load_golden("c1_fp32")
    assert not O.near_ties(g["probs"], case.top_k, rel=1e-4).any()
    assert g["counts"].sum() == case.tokens * case.top_k
    assert g["out"].shape == (512, 768)


@pytest.mark.parametrize("x", [-30.0, -20.0, -5.0, -1.0, 0.0, 1.0, 5.0, 19.999, 20.0, 20.001, 30.0])
def test_era_known_answers(x):
    # ERA(x) = F.gelu(x, approximate="tanh") + 0.1 * F.softplus(x)  (model.py:72-75)
    import torch
    import torch.nn.functional as F
    t = torch.tensor([x], dtype=torch.float32)
    ref = (F.gelu(t, approximate="tanh") + 0.1 * F.softplus(t)).item()
    got = float(O.era(np.array([x], dtype=np.float32), 0.1)[0])
    assert got == pytest.approx(ref, rel=1e-6, abs=1e-7)


def test_era_greater_than_gelu():
    # the one value-level property in the reference's tests (crates/vesper-core/src/era.rs:100-114)
    xs = np.array([1.0, 2.0, 3.0], dtype=np.float32)
    assert (O.era(xs, 0.1) > O.gelu_tanh(xs)).all()


def test_topk_lowest_index_tie_break():
    p = np.array([[0.125] * 8, [0.1, 0.3, 0.3, 0.3, 0, 0, 0, 0]], dtype=np.float32)
    _, idx = O.topk_lowest_index(p, 2)
    assert idx.tolist() == [[0, 1], [1, 2]]


def test_expert_set_and_order_helpers():
    a = np.array([[3, 1], [0, 2]])
    b = np.array([[1, 3], [0, 1]])
    assert O.same_expert_sets(a, b).tolist() == [True, False]
    p = np.array([[0.1, 0.4, 0.1, 0.4]])
    assert O.order_follows_probs(np.array([[1, 3]]), p).all()      # tie -> lowest index first
    assert not O.order_follows_probs(np.array([[3, 1]]), p).all()
    assert not O.order_follows_probs(np.array([[0, 1]]), p).all()


def test_dispatch_is_stable_expert_major():
    idx = np.array([[2, 0], [0, 1], [2, 1], [0, 2]])
    counts, tok, slot = O.dispatch(idx, 3)
    assert counts.tolist() == [3, 2, 3]
    assert tok.tolist() == [0, 1, 3, 1, 2, 0, 2, 3]
    assert slot.tolist() == [1, 0, 0, 1, 1, 0, 0, 1]


def test_token_subset_matches_full():
    case, _ = load_golden("t127_bias")
    inp = make_inputs(case)
    full = O.moe_forward(inp, case)
    sub = np.array([0, 5, 77, 126])
    part = O.moe_forward(inp, case, token_subset=sub)
    # per-token math; BLAS blocking differs with the row count, so ulp-level only
    assert O.norm_rel_err(part["out"], full["out"][sub]) < 1e-6


def test_round_bf16():
    a = np.array([1.0, 1.00390625, 1.0078125, -2.5, 3.0e-3, 65504.0], dtype=np.float32)
    import torch
    ref = torch.from_numpy(a).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(round_bf16(a), ref)
    r = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    assert np.array_equal(round_bf16(r), torch.from_numpy(r).to(torch.bfloat16).float().numpy())
