"""Generate golden vectors by executing the reference MoELayer on CPU.

Run where a VelvetOptimizer checkout is available (read-only is enough)::

    python tests/golden/make_golden.py [--reference DIR] [names...]   # writes tests/golden/*.npz

``DIR`` is the checkout's ``python/`` directory; without ``--reference`` it is
``$VESPER_REFERENCE_PYTHON``, else ``reference/python`` beside this repository.

The reference's Python package is imported in place (``sys.path``), never copied.
Inputs come from ``oracle.inputs.make_inputs`` (seeded numpy), are loaded into the
reference module through its own state_dict keys, and the forward runs exactly as
``MoELayer.forward`` (python/vesper/model.py:317-364).  The router logits are captured
with a forward hook on ``moe.router``; softmax / top-K are recomputed from them with the
same torch calls as model.py:323-329 to record the reference's routing.

Each ``<name>.npz`` stores only the case description (JSON) and the outputs, not the
inputs: tests rebuild the inputs from the seed.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.inputs import MoECase, backward_inputs, make_inputs  # noqa: E402
from tests.golden_io import reference_python_dir  # noqa: E402

REFERENCE_PY = ""  # set by main()

# name -> case.  Small enough to commit; together they cover the reference's own edge
# cases (K == E, E == 2, a single token, empty experts, K = 1) and the option set
# (biases, FlyLoRA on, Zipf router bias, an all-tied router).
CASES = {
    "c1_fp32": MoECase(tokens=512, batch=2, hidden=768, inter=3072, experts=8, top_k=2),
    "t1_single_token": MoECase(tokens=1, batch=1, hidden=64, inter=128, experts=4, top_k=2, seed=1),
    "t3_k_eq_e": MoECase(tokens=3, batch=1, hidden=32, inter=64, experts=2, top_k=2, seed=2),
    "t127_bias": MoECase(tokens=127, batch=1, hidden=96, inter=160, experts=8, top_k=3,
                         bias_std=0.05, seed=3),
    "t5_empty_experts": MoECase(tokens=5, batch=1, hidden=48, inter=80, experts=16, top_k=1, seed=4),
    "t256_lora_zipf": MoECase(tokens=256, batch=2, hidden=128, inter=256, experts=16, top_k=4,
                              lora_on=True, zipf_alpha=1.2, seed=5),
    "t64_tied_router": MoECase(tokens=64, batch=4, hidden=64, inter=96, experts=8, top_k=2,
                               router_std=0.0, seed=6),
    "t200_era_tails": MoECase(tokens=200, batch=2, hidden=64, inter=128, experts=4, top_k=2,
                              weight_std=0.5, bias_std=2.0, seed=7),
}


def reference_layer(case: MoECase, inp: dict[str, np.ndarray]):
    import torch
    sys.path.insert(0, REFERENCE_PY)
    from vesper.config import VesperConfig  # noqa: E402
    from vesper.model import MoELayer  # noqa: E402

    cfg = VesperConfig(hidden_size=case.hidden, intermediate_size=case.inter,
                       num_heads=1, era_gamma=case.era_gamma,
                       flylora_rank=case.lora_rank, flylora_alpha=case.lora_alpha)
    cfg.with_moe(num_experts=case.experts, top_k=case.top_k)
    cfg.validate()
    torch.manual_seed(case.seed)
    moe = MoELayer(cfg)
    sd = moe.state_dict()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    new = {"router.weight": t(inp["w_r"]), "router.bias": t(inp["b_r"])}
    for e in range(case.experts):
        for p, name in (("g", "gate_proj"), ("u", "up_proj")):
            pre = f"experts.{e}.{name}"
            new[f"{pre}.base.weight"] = t(inp[f"w_{p}"][e])
            new[f"{pre}.base.bias"] = t(inp[f"b_{p}"][e])
            new[f"{pre}.lora_down.weight"] = t(inp[f"a_{p}"][e])
            new[f"{pre}.lora_down.bias"] = t(inp[f"ba_{p}"][e])
            new[f"{pre}.lora_up.weight"] = t(inp[f"l_{p}"][e])
            new[f"{pre}.lora_up.bias"] = t(inp[f"bl_{p}"][e])
            new[f"{pre}.proj_a"] = sd[f"{pre}.proj_a"]
        new[f"experts.{e}.down_proj.weight"] = t(inp["w_d"][e])
        new[f"experts.{e}.down_proj.bias"] = t(inp["b_d"][e])
    assert set(new) == set(sd), set(sd) ^ set(new)
    moe.load_state_dict(new)
    moe.eval()
    return moe


def run_reference(case: MoECase):
    import torch
    import torch.nn.functional as F

    inp = make_inputs(case)
    moe = reference_layer(case, inp)
    captured = {}
    moe.router.register_forward_hook(lambda m, i, o: captured.__setitem__("logits", o.detach().clone()))
    x = torch.from_numpy(inp["x"]).reshape(case.batch, case.seq, case.hidden)
    with torch.no_grad():
        out, aux = moe(x)
    logits = captured["logits"]
    probs = F.softmax(logits, dim=-1)                       # model.py:323
    topv, topi = torch.topk(probs, case.top_k, dim=-1)      # model.py:326
    topw = topv / topv.sum(dim=-1, keepdim=True)            # model.py:329
    T = case.tokens
    idx = topi.reshape(T, case.top_k).numpy().astype(np.int64)
    counts = np.bincount(idx.reshape(-1), minlength=case.experts)
    perm = [np.nonzero((idx == e).any(-1))[0] for e in range(case.experts)]  # model.py:346-347
    return {
        "logits": logits.reshape(T, case.experts).numpy(),
        "probs": probs.reshape(T, case.experts).numpy(),
        "topk_idx": idx,
        "topk_w": topw.reshape(T, case.top_k).numpy(),
        "counts": counts.astype(np.int64),
        "perm_tok": np.concatenate(perm).astype(np.int64) if perm else np.zeros(0, np.int64),
        "out": out.reshape(T, case.hidden).numpy(),
        "aux": np.asarray(aux.item(), dtype=np.float32),
    }


# dense FeedForward cases (python/vesper/model.py:249-270): the non-MoE layers' FFN
FFN_CASES = {
    "ffn_t64_lora_bias": MoECase(tokens=64, batch=2, hidden=128, inter=256, experts=1, top_k=1,
                                 lora_on=True, bias_std=0.05, seed=21),
    "ffn_t3_small": MoECase(tokens=3, batch=1, hidden=32, inter=48, experts=1, top_k=1, seed=22),
}


def run_reference_ffn(case: MoECase):
    import torch
    sys.path.insert(0, REFERENCE_PY)
    from vesper.config import VesperConfig  # noqa: E402
    from vesper.model import FeedForward  # noqa: E402

    inp = make_inputs(case)
    cfg = VesperConfig(hidden_size=case.hidden, intermediate_size=case.inter, num_heads=1,
                       era_gamma=case.era_gamma, flylora_rank=case.lora_rank,
                       flylora_alpha=case.lora_alpha)
    torch.manual_seed(case.seed)
    ffn = FeedForward(cfg)
    sd = ffn.state_dict()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    new = {}
    for p, name in (("g", "gate_proj"), ("u", "up_proj")):
        new[f"{name}.base.weight"] = t(inp[f"w_{p}"][0])
        new[f"{name}.base.bias"] = t(inp[f"b_{p}"][0])
        new[f"{name}.lora_down.weight"] = t(inp[f"a_{p}"][0])
        new[f"{name}.lora_down.bias"] = t(inp[f"ba_{p}"][0])
        new[f"{name}.lora_up.weight"] = t(inp[f"l_{p}"][0])
        new[f"{name}.lora_up.bias"] = t(inp[f"bl_{p}"][0])
        new[f"{name}.proj_a"] = sd[f"{name}.proj_a"]
    new["down_proj.weight"] = t(inp["w_d"][0])
    new["down_proj.bias"] = t(inp["b_d"][0])
    assert set(new) == set(sd), set(sd) ^ set(new)
    ffn.load_state_dict(new)
    x = torch.from_numpy(inp["x"]).reshape(case.batch, case.seq, case.hidden)
    with torch.no_grad():
        out = ffn(x)
    return {"out": out.reshape(case.tokens, case.hidden).numpy()}


# fused pre-norm block cases (python/vesper/model.py:418-425): residual stream x with
# per-token and per-channel offsets, LayerNorm with random affine parameters
LN_CASES = {
    "ln_t96_bias": MoECase(tokens=96, batch=2, hidden=128, inter=192, experts=8, top_k=2,
                           bias_std=0.05, seed=31),
    "ln_t40_lora_e16k4": MoECase(tokens=40, batch=1, hidden=64, inter=96, experts=16, top_k=4,
                                 lora_on=True, seed=32),
}


def run_reference_prenorm(case: MoECase):
    """ffn_norm + MoELayer + residual exactly as TransformerLayer.forward (model.py:418-425)."""
    import torch
    from oracle.inputs import make_norm_inputs

    inp = make_inputs(case)
    ni = make_norm_inputs(case)
    moe = reference_layer(case, inp)
    norm = torch.nn.LayerNorm(case.hidden, eps=float(ni["eps"]))   # model.py:399
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(ni["ln_w"]))
        norm.bias.copy_(torch.from_numpy(ni["ln_b"]))
    captured = {}
    moe.router.register_forward_hook(lambda m, i, o: captured.__setitem__("logits", o.detach().clone()))
    hidden = torch.from_numpy(ni["x"]).reshape(case.batch, case.seq, case.hidden)
    with torch.no_grad():
        normed = norm(hidden)                 # model.py:418
        ffn_out, aux = moe(normed)            # model.py:420
        out = hidden + ffn_out                # model.py:425
    T = case.tokens
    probs = torch.softmax(captured["logits"], dim=-1)
    return {"normed": normed.reshape(T, case.hidden).numpy(),
            "logits": captured["logits"].reshape(T, case.experts).numpy(),
            "probs": probs.reshape(T, case.experts).numpy(),
            "out": out.reshape(T, case.hidden).numpy(),
            "aux": np.asarray(aux.item(), dtype=np.float32)}


# backward cases: autograd through the reference MoELayer for
# L = sum(out * dout) + daux * aux (python/train.py:95-96: the aux weight scales the loss)
BW_CASES = {
    "bw_t64_lora_bias": MoECase(tokens=64, batch=2, hidden=64, inter=96, experts=4, top_k=2,
                                lora_on=True, bias_std=0.05, seed=51),
    "bw_t37_k1": MoECase(tokens=37, batch=1, hidden=48, inter=64, experts=8, top_k=1, seed=52),
    "bw_t20_k_eq_e": MoECase(tokens=20, batch=1, hidden=32, inter=48, experts=2, top_k=2,
                             bias_std=0.05, seed=53),
}


def run_reference_backward(case: MoECase):
    import torch

    inp = make_inputs(case)
    moe = reference_layer(case, inp)
    dout, daux = backward_inputs(case)
    x = torch.from_numpy(inp["x"]).reshape(case.batch, case.seq, case.hidden).requires_grad_(True)
    out, aux = moe(x)
    loss = (out * torch.from_numpy(dout).reshape(out.shape)).sum() + float(daux) * aux
    loss.backward()
    E = case.experts
    st = lambda f: np.stack([f(e).grad.numpy() for e in moe.experts])  # noqa: E731
    res = {"dx": x.grad.reshape(case.tokens, case.hidden).numpy(),
           "dw_r": moe.router.weight.grad.numpy(), "db_r": moe.router.bias.grad.numpy(),
           "dw_d": st(lambda e: e.down_proj.weight), "db_d": st(lambda e: e.down_proj.bias)}
    for q, name in (("g", "gate_proj"), ("u", "up_proj")):
        res[f"dw_{q}"] = st(lambda e: getattr(e, name).base.weight)
        res[f"db_{q}"] = st(lambda e: getattr(e, name).base.bias)
        res[f"da_{q}"] = st(lambda e: getattr(e, name).lora_down.weight)
        res[f"dba_{q}"] = st(lambda e: getattr(e, name).lora_down.bias)
        res[f"dl_{q}"] = st(lambda e: getattr(e, name).lora_up.weight)
        res[f"dbl_{q}"] = st(lambda e: getattr(e, name).lora_up.bias)
    with torch.no_grad():
        probs = torch.softmax(moe.router(x.reshape(-1, case.hidden)), dim=-1)
    res["probs"] = probs.numpy()
    res["out"] = out.detach().reshape(case.tokens, case.hidden).numpy()
    res["aux"] = np.asarray(aux.item(), dtype=np.float32)
    assert E == res["dw_g"].shape[0]
    return res


def dump_state_dict_keys():
    """Record the reference MoELayer's state_dict keys and shapes for a small config."""
    sys.path.insert(0, REFERENCE_PY)
    from vesper.config import VesperConfig  # noqa: E402
    from vesper.model import MoELayer  # noqa: E402
    conf = dict(hidden_size=64, intermediate_size=96, moe_num_experts=3, moe_top_k=2,
                flylora_rank=8, flylora_alpha=16.0, era_gamma=0.1)
    cfg = VesperConfig(hidden_size=64, intermediate_size=96, num_heads=1, flylora_rank=8,
                       flylora_alpha=16.0).with_moe(num_experts=3, top_k=2)
    keys = {k: list(v.shape) for k, v in MoELayer(cfg).state_dict().items()}
    from vesper.model import FeedForward  # noqa: E402
    ffn_keys = {k: list(v.shape) for k, v in FeedForward(cfg).state_dict().items()}
    path = os.path.join(HERE, "state_dict_keys.json")
    with open(path, "w") as f:
        json.dump({"config": conf, "keys": keys, "ffn_keys": ffn_keys}, f, indent=1)
    print(f"state_dict keys: {len(keys)} -> {path}")


def main(names=None, reference=None):
    global REFERENCE_PY
    REFERENCE_PY = reference or reference_python_dir() or ""
    if not os.path.isfile(os.path.join(REFERENCE_PY, "vesper", "model.py")):
        raise SystemExit("no reference checkout found: pass --reference DIR (the checkout's "
                         "python/ directory) or set VESPER_REFERENCE_PYTHON")
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    if not names:
        dump_state_dict_keys()
    for name, case in FFN_CASES.items():
        if names and name not in names:
            continue
        res = run_reference_ffn(case)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, case=np.asarray(json.dumps(case.to_dict())),
                            torch_version=np.asarray(torch.__version__), **res)
        print(f"{name}: out {res['out'].shape} -> {path}")
    for name, case in BW_CASES.items():
        if names and name not in names:
            continue
        res = run_reference_backward(case)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, case=np.asarray(json.dumps(case.to_dict())),
                            torch_version=np.asarray(torch.__version__), **res)
        print(f"{name}: |dx|={np.abs(res['dx']).max():.4f} -> {path}")
    for name, case in LN_CASES.items():
        if names and name not in names:
            continue
        res = run_reference_prenorm(case)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, case=np.asarray(json.dumps(case.to_dict())),
                            torch_version=np.asarray(torch.__version__), **res)
        print(f"{name}: aux={float(res['aux']):.6f} -> {path}")
    for name, case in CASES.items():
        if names and name not in names:
            continue
        res = run_reference(case)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, case=np.asarray(json.dumps(case.to_dict())),
                            torch_version=np.asarray(torch.__version__), **res)
        print(f"{name}: aux={float(res['aux']):.6f} counts={res['counts'].tolist()} -> {path}")


if __name__ == "__main__":
    argv = sys.argv[1:]
    ref = None
    if "--reference" in argv:
        i = argv.index("--reference")
        ref = argv[i + 1]
        del argv[i:i + 2]
    main(argv or None, ref)
