"""Full-size parity through the C ABI at the benchmark workloads' shapes (bf16).

The oracle cannot run these sizes end to end in seconds, so the tests check what holds at
any size, and the oracle on what it can do quickly:
  * routing: counts equal the histogram of the indices and sum to T*K, every token's K
    experts are distinct, the renormalised weights are positive and sum to 1;
  * dispatch: the slots form a bijection onto the expert segments, tokens ascending inside
    each expert (the reference's nonzero() order), segments padded to whole GEMM tiles;
  * router logits and the aux loss of ALL tokens against the oracle (numpy fp32 on the same
    bf16-rounded inputs), expert indices equal except near-ties;
  * the outputs against the oracle on the GPU's own routing, within the bf16 tolerance
    (2e-2 norm-relative): every token of the decode-sized batch, a sample of the others;
  * determinism: a second forward is bit-identical.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase
from velvetoptimizer_b200 import _lib

pytestmark = pytest.mark.gpu

# shapes of the benchmark workloads (tokens per GPU)
SHAPES = {
    "c2_decode": dict(tokens=64, hidden=2048, inter=8192, experts=8, top_k=2),
    "c3_prefill": dict(tokens=32768, hidden=2048, inter=8192, experts=8, top_k=2),
    "c4_skewed": dict(tokens=32768, hidden=2048, inter=1024, experts=64, top_k=8, lora_on=True,
                      zipf_alpha=1.2),
    "c5_ep": dict(tokens=65536, hidden=4096, inter=2048, experts=64, top_k=4),
}
KEYS = {"router_w": "w_r", "router_b": "b_r", "gate_w": "w_g", "gate_b": "b_g", "up_w": "w_u",
        "up_b": "b_u", "down_w": "w_d", "down_b": "b_d", "gate_lora_down_w": "a_g",
        "gate_lora_down_b": "ba_g", "gate_lora_up_w": "l_g", "gate_lora_up_b": "bl_g",
        "up_lora_down_w": "a_u", "up_lora_down_b": "ba_u", "up_lora_up_w": "l_u",
        "up_lora_up_b": "bl_u"}


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def device_weights(s, dev, seed=0):
    """All weights in bf16 on the device: N(0, 0.02), biases N(0, 0.01), Zipf router bias."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    E, H, I, r = s["experts"], s["hidden"], s["inter"], 16
    n = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    b = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.01).to(torch.bfloat16)  # noqa: E731
    z = lambda *sh: torch.zeros(*sh, dtype=torch.bfloat16, device=dev)  # noqa: E731
    w = {"router_w": n(E, H), "router_b": b(E), "down_w": n(E, H, I), "down_b": b(E, H)}
    for p in ("gate", "up"):
        w[f"{p}_w"], w[f"{p}_b"] = n(E, I, H), b(E, I)
        w[f"{p}_lora_down_w"], w[f"{p}_lora_down_b"] = n(E, r, H), b(E, r)
        w[f"{p}_lora_up_w"] = n(E, I, r) if s.get("lora_on") else z(E, I, r)
        w[f"{p}_lora_up_b"] = b(E, I) if s.get("lora_on") else z(E, I)
    if s.get("zipf_alpha"):
        ranks = torch.arange(1, E + 1, dtype=torch.float64)
        pmf = ranks ** (-s["zipf_alpha"])
        w["router_b"] = torch.log(pmf / pmf.sum()).to(device=dev, dtype=torch.bfloat16)
    return w


class LazyExperts:
    """Expert weights copied to the host (fp32 numpy) only when the oracle touches them."""

    def __init__(self, t):
        self.t = t
        self.cache = {}

    def __getitem__(self, e):
        if e not in self.cache:
            self.cache[e] = self.t[e].float().cpu().numpy()
        return self.cache[e]


@pytest.mark.parametrize("name", list(SHAPES))
def test_full_size_parity_and_invariants(name):
    s = SHAPES[name]
    T, H, I, E, K = s["tokens"], s["hidden"], s["inter"], s["experts"], s["top_k"]
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    w = device_weights(s, dev)
    cfg = _lib.VmoeConfig(hidden=H, inter=I, num_experts=E, top_k=K, lora_rank=16,
                          lora_scaling=2.0, era_gamma=0.1, dtype=_lib.VMOE_BF16, capacity=0)
    h = _lib.Handle(cfg, 0)
    h.set_weights(_lib.VmoeWeights(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in w.items()}),
                  stream)
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    ws = torch.empty(h.workspace_size(T), dtype=torch.uint8, device=dev)

    def run():
        r = {"out": torch.empty_like(x),
             "logits": torch.empty((T, E), dtype=torch.float32, device=dev),
             "idx": torch.empty((T, K), dtype=torch.int32, device=dev),
             "w": torch.empty((T, K), dtype=torch.float32, device=dev),
             "counts": torch.empty((E,), dtype=torch.int32, device=dev),
             "aux": torch.empty((1,), dtype=torch.float32, device=dev)}
        h.forward(x.data_ptr(), T, r["out"].data_ptr(), r["logits"].data_ptr(), r["idx"].data_ptr(),
                  r["w"].data_ptr(), r["counts"].data_ptr(), r["aux"].data_ptr(), ws.data_ptr(),
                  ws.numel(), stream)
        torch.cuda.synchronize()
        assert h.device_status(stream) == 0
        return r

    r1 = run()
    lay = h.workspace_layout(T)
    slot = ws[lay.slot_of:lay.slot_of + 4 * T * K].view(torch.int32).cpu().numpy().reshape(T, K)
    offs = ws[lay.expert_offsets:lay.expert_offsets + 4 * (E + 1)].view(torch.int32).cpu().numpy()
    r2 = run()
    for k in r1:  # determinism
        assert torch.equal(r1[k], r2[k]), k

    idx = r1["idx"].cpu().numpy().astype(np.int64)
    tw = r1["w"].cpu().numpy()
    counts = r1["counts"].cpu().numpy()
    # routing invariants
    assert ((idx >= 0) & (idx < E)).all()
    assert (np.sort(idx, axis=1)[:, 1:] != np.sort(idx, axis=1)[:, :-1]).all()
    assert np.array_equal(counts, np.bincount(idx.reshape(-1), minlength=E))
    assert counts.sum() == T * K
    assert (tw > 0).all() and np.allclose(tw.sum(axis=1), 1.0, atol=1e-5)
    # dispatch: stable expert-major bijection onto padded segments (16 rows for the decode
    # GEMMs of a batch of at most 256 tokens, whole GEMM tiles otherwise)
    align = h.lib.vmoe_segment_align(h.ptr, T)
    assert align == (16 if T <= 256 else h.lib.vmoe_gemm_tile_rows(h.ptr))
    assert (offs % align == 0).all() and (np.diff(offs) >= counts).all()
    flat_e, flat_s = idx.reshape(-1), slot.reshape(-1)
    flat_t = np.repeat(np.arange(T), K)
    order = np.lexsort((flat_t, flat_e))
    expect = np.concatenate([offs[e] + np.arange(counts[e]) for e in range(E)])
    assert np.array_equal(flat_s[order], expect)

    # the oracle on the same bf16-rounded inputs
    p = {"x": x.float().cpu().numpy(), "w_r": w["router_w"].float().cpu().numpy(),
         "b_r": w["router_b"].float().cpu().numpy()}
    for k, v in KEYS.items():
        if v not in p:
            p[v] = LazyExperts(w[k])
    logits = O.router_logits(p["x"], p["w_r"], p["b_r"])
    assert O.norm_rel_err(r1["logits"].cpu().numpy(), logits) < 1e-4
    probs = O.softmax(logits)
    _, oidx = O.topk_lowest_index(probs, K)
    tie = O.near_ties(probs, K, rel=1e-4)
    assert O.same_expert_sets(idx[~tie], oidx[~tie]).all()
    # the GPU lists each token's experts by its own probabilities, lowest index on ties
    assert O.order_follows_probs(idx, O.softmax(r1["logits"].cpu().numpy()), rel=1e-5).all()
    aux = float(O.load_balancing_loss(O.softmax(r1["logits"].cpu().numpy()), idx, E))
    assert abs(float(r1["aux"].item()) - aux) <= 1e-4 * abs(aux)

    case = MoECase(tokens=T, hidden=H, inter=I, experts=E, top_k=K, lora_on=bool(s.get("lora_on")))
    # every token of a decode-sized batch, a sample of the large ones
    sample = np.arange(T) if T <= 256 else np.unique(
        np.concatenate([np.arange(4), np.linspace(0, T - 1, 28).astype(np.int64)]))
    ref = O.moe_forward(p, case, force_idx=idx, token_subset=sample)
    got = r1["out"][torch.from_numpy(sample).to(dev)].float().cpu().numpy()
    err = O.norm_rel_err(got, ref["out"])
    assert err < 2e-2, err
    h.close()
