"""CPU restatement of VelvetOptimizer's MoE FFN forward (TEST INFRASTRUCTURE ONLY).

This is the oracle.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference leg may import it, and only as the checker or as the timed
CPU baseline -- never as the product path.  The product path (``velvetoptimizer_b200``)
runs CUDA kernels and fails loudly if they are missing.

Every function follows a specific piece of the reference (paths relative to the
VelvetOptimizer project root):

* router GEMM            python/vesper/model.py:314,322
* softmax                python/vesper/model.py:323
* top-K + renormalise    python/vesper/model.py:326,329
* dispatch order         python/vesper/model.py:339-349  (expert-major, tokens ascending)
* FlyLoRA linear         python/vesper/model.py:123-126
* ERA activation         python/vesper/model.py:69-76    (CPU form: F.gelu tanh + softplus)
* expert FFN             python/vesper/model.py:295-298
* combine                python/vesper/model.py:337,354-357 (index_add_ in expert order)
* load-balancing loss    python/vesper/model.py:366-385
* pre-norm block         python/vesper/model.py:418-425 (ffn_norm LayerNorm, residual add)
* backward               autograd of all of the above for loss = <out, dout> + daux * aux
                         (python/train.py:95-96,465 trains through it; ERA derivative as
                         python/vesper/kernels/era_triton.py:57-84)

Pinning: ``tests/golden/make_golden.py`` executes the reference ``MoELayer`` itself (in
the container where the reference is mounted) and commits its outputs as fixtures;
``tests/test_oracle.py`` checks this restatement against every one of them.

Top-K tie rule.  ``torch.topk`` on CPU does not break exact ties by lowest index (its
order on equal values is implementation-defined).  This restatement breaks ties by
lowest index, as the CUDA router does.  The two agree on every token whose K-th and
(K+1)-th probabilities differ; ``near_ties`` lists the tokens where they may not.
"""
from __future__ import annotations

import numpy as np

GELU_C = np.float32(0.7978845608028654)   # sqrt(2/pi)
GELU_A = np.float32(0.044715)
SOFTPLUS_THRESHOLD = np.float32(20.0)     # torch F.softplus default threshold


def _mm(a: np.ndarray, b_t: np.ndarray, dtype) -> np.ndarray:
    """y = a @ b_t.T in ``dtype`` (nn.Linear without bias)."""
    return a.astype(dtype, copy=False) @ b_t.astype(dtype, copy=False).T


def router_logits(x, w_r, b_r, dtype=np.float32):
    """logits = x W_r^T + b_r  (model.py:314,322)."""
    return (_mm(x, w_r, dtype) + b_r.astype(dtype)).astype(dtype)


def softmax(logits):
    """Row softmax with max subtraction (model.py:323, F.softmax(dim=-1))."""
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m)
    return e / e.sum(axis=-1, keepdims=True)


def topk_lowest_index(probs, k):
    """Top-k by (probability descending, expert index ascending) (model.py:326).

    Returns (values [T,k], indices [T,k] int64) sorted like torch.topk(sorted=True).
    """
    t, e = probs.shape
    # lexsort sorts by the last key first: primary -prob, secondary index
    idx_grid = np.broadcast_to(np.arange(e), (t, e))
    order = np.lexsort((idx_grid, -probs), axis=-1)
    top = order[:, :k].astype(np.int64)
    vals = np.take_along_axis(probs, top, axis=-1)
    return vals, top


def renormalise(vals):
    """w = p_k / sum_k p_k  (model.py:329)."""
    return vals / vals.sum(axis=-1, keepdims=True)


def near_ties(probs, k, rel=1e-4):
    """Tokens whose K-th and (K+1)-th probabilities are within ``rel`` (relative).

    On those tokens the chosen expert set may legitimately differ between two correct
    implementations (different accumulation order in the router GEMM, or torch's own
    tie order).  Returns a boolean mask [T].  With k == E there is no boundary.
    """
    t, e = probs.shape
    if k >= e:
        return np.zeros(t, dtype=bool)
    s = -np.sort(-probs, axis=-1)
    gap = s[:, k - 1] - s[:, k]
    return gap <= rel * s[:, k - 1]


def same_expert_sets(a, b):
    """Row-wise equality of the chosen expert SETS of two [T, K] index arrays.

    The order inside a token's K choices follows the probabilities; where two chosen
    experts are a near-tie, two correct implementations may order them differently, which
    changes nothing downstream except the fp add order of the combine.
    """
    return np.all(np.sort(a, axis=-1) == np.sort(b, axis=-1), axis=-1)


def order_follows_probs(idx, probs, rel=0.0):
    """True per token when idx lists experts by (probability desc, index asc).

    With ``rel`` > 0 (``probs`` recomputed elsewhere, last-ulp differences possible) only
    clear inversions count: a later choice more than ``rel`` above an earlier one.
    """
    p = np.take_along_axis(probs, idx, axis=-1)
    dp = p[:, :-1] - p[:, 1:]
    di = idx[:, :-1] - idx[:, 1:]
    if rel > 0:
        return np.all(dp >= -rel * p[:, :-1], axis=-1)
    return np.all((dp > 0) | ((dp == 0) & (di < 0)), axis=-1)


def dispatch(topk_idx, experts):
    """Per-expert counts and the stable expert-major permutation (model.py:339-349).

    For each expert e in ascending order the reference takes ``token_mask.nonzero()``,
    i.e. the tokens that chose e in ascending token order.  Returns

    * counts   [E] int64
    * perm_tok [T*K] int64 : token index of each dispatched row, expert-major
    * perm_k   [T*K] int64 : which of the token's K slots the row came from
    """
    t, k = topk_idx.shape
    flat = topk_idx.reshape(-1)
    counts = np.bincount(flat, minlength=experts).astype(np.int64)
    tok = np.repeat(np.arange(t), k)
    slot = np.tile(np.arange(k), t)
    order = np.lexsort((tok, flat))  # expert primary, token secondary
    return counts, tok[order].astype(np.int64), slot[order].astype(np.int64)


def gelu_tanh(g):
    """F.gelu(approximate='tanh') (model.py:72)."""
    return np.float32(0.5) * g * (np.float32(1.0) + np.tanh(GELU_C * (g + GELU_A * g * g * g)))


def softplus(g):
    """F.softplus(beta=1, threshold=20): x if x > 20 else log1p(exp(x)) (model.py:74)."""
    with np.errstate(over="ignore"):
        sp = np.log1p(np.exp(np.minimum(g, SOFTPLUS_THRESHOLD)))
    return np.where(g > SOFTPLUS_THRESHOLD, g, sp).astype(g.dtype)


def era(g, gamma):
    """ERA(x) = GELU_tanh(x) + gamma * softplus(x)  (model.py:62-76)."""
    out = gelu_tanh(g)
    if gamma > 0.0:
        out = out + g.dtype.type(gamma) * softplus(g)
    return out


def flylora_linear(x, w, b, a, ba, l, bl, scaling, dtype):
    """base(x) + scaling * lora_up(lora_down(x))  (model.py:123-126)."""
    base = _mm(x, w, dtype) + b.astype(dtype)
    down = _mm(x, a, dtype) + ba.astype(dtype)
    up = _mm(down, l, dtype) + bl.astype(dtype)
    return base + dtype(scaling) * up


def expert_ffn(x_e, p, e, gamma, scaling, dtype):
    """down(ERA(gate(x)) * up(x)) for expert e  (model.py:295-298)."""
    gate = flylora_linear(x_e, p["w_g"][e], p["b_g"][e], p["a_g"][e], p["ba_g"][e],
                          p["l_g"][e], p["bl_g"][e], scaling, dtype)
    up = flylora_linear(x_e, p["w_u"][e], p["b_u"][e], p["a_u"][e], p["ba_u"][e],
                        p["l_u"][e], p["bl_u"][e], scaling, dtype)
    h = era(gate, gamma) * up
    return _mm(h, p["w_d"][e], dtype) + p["b_d"][e].astype(dtype)


def ffn_forward(p, case, dtype=np.float32):
    """Dense FeedForward: down(ERA(gate(x)) * up(x)) with FlyLoRA (model.py:249-270).

    ``p`` holds one expert's weights at index 0 (``make_inputs`` with experts=1)."""
    return expert_ffn(p["x"], p, 0, case.era_gamma, case.lora_scaling, dtype)


def load_balancing_loss(probs, topk_idx, experts):
    """Switch-Transformer aux loss E * sum_e f_e * P_e  (model.py:366-385)."""
    t, k = topk_idx.shape
    p_mean = probs.mean(axis=0)
    counts = np.bincount(topk_idx.reshape(-1), minlength=experts).astype(probs.dtype)
    f = counts / probs.dtype.type(t * k)
    return probs.dtype.type(experts) * (f * p_mean).sum()


def moe_forward(p, case, *, dtype=np.float32, force_idx=None, token_subset=None, capacity=0):
    """Full MoE layer forward (model.py:317-364).

    ``p`` is the dict of ``oracle.inputs.make_inputs``.  ``force_idx`` ([T,K]) replaces
    the top-K choice (used to compare outputs on identical routing when a near-tie was
    resolved differently).  ``token_subset`` computes outputs only for those tokens
    (the forward is per-token once routing is fixed), while router, routing and aux
    loss still cover all T tokens.  ``capacity`` > 0 keeps only the first ``capacity``
    tokens (ascending token order) of each expert -- an extension: the reference has no
    capacity limit, which is ``capacity=0``.

    Returns a dict with logits, probs, topk_idx, topk_w, counts, perm_tok, perm_k,
    out ([T,H], or [len(subset),H]) and aux (0-d).
    """
    x = p["x"]
    t, h = x.shape
    E, K = case.experts, case.top_k
    logits = router_logits(x, p["w_r"], p["b_r"], dtype)
    probs = softmax(logits)
    vals, idx = topk_lowest_index(probs, K)
    if force_idx is not None:
        idx = np.asarray(force_idx, dtype=np.int64).reshape(t, K)
        vals = np.take_along_axis(probs, idx, axis=-1)
    w = renormalise(vals)
    counts, perm_tok, perm_k = dispatch(idx, E)
    aux = load_balancing_loss(probs, idx, E)

    if token_subset is None:
        rows = np.arange(t)
    else:
        rows = np.asarray(token_subset, dtype=np.int64)
    kept = np.ones_like(idx, dtype=bool)
    if capacity > 0:
        for e in range(E):
            tok = np.nonzero((idx == e).any(axis=-1))[0]
            for t in tok[capacity:]:
                kept[t] &= idx[t] != e
    sub_idx, sub_w, xs = idx[rows], w[rows], x[rows]
    sub_kept = kept[rows]
    out = np.zeros((len(rows), h), dtype=dtype)
    for e in range(E):  # ascending expert order, like the reference's index_add_ loop
        mask = (sub_idx == e) & sub_kept
        sel = np.nonzero(mask.any(axis=-1))[0]
        if sel.size == 0:
            continue
        y = expert_ffn(xs[sel], p, e, case.era_gamma, case.lora_scaling, dtype)
        we = (mask[sel].astype(dtype) * sub_w[sel].astype(dtype)).sum(axis=-1)
        out[sel] += (y * we[:, None]).astype(dtype)
    return {
        "logits": logits, "probs": probs, "topk_idx": idx, "topk_w": w,
        "counts": counts, "perm_tok": perm_tok, "perm_k": perm_k,
        "out": out, "aux": np.asarray(aux, dtype=dtype),
    }


def era_grad(g, gamma):
    """d ERA / dg: GELU-tanh derivative + gamma * softplus derivative (sigmoid; 1 above the
    threshold 20, as torch's softplus backward)  (model.py:62-76, era_triton.py:57-84)."""
    g = np.asarray(g, dtype=np.float32)
    k = GELU_C * (g + GELU_A * g * g * g)
    t = np.tanh(k)
    d = np.float32(0.5) * (np.float32(1.0) + t) + np.float32(0.5) * g * (np.float32(1.0) - t * t) \
        * GELU_C * (np.float32(1.0) + np.float32(3.0) * GELU_A * g * g)
    if gamma > 0.0:
        with np.errstate(over="ignore"):
            sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-np.minimum(g, SOFTPLUS_THRESHOLD)))
        d = d + np.float32(gamma) * np.where(g > SOFTPLUS_THRESHOLD, np.float32(1.0), sig)
    return d.astype(np.float32)


def moe_backward(p, case, dout, daux, *, force_idx=None):
    """Gradients of L = sum(out * dout) + daux * aux through ``moe_forward`` (fp32).

    Restates autograd of MoELayer.forward (model.py:317-385) on the forward's routing:
    the combine (out += y_e * w_e) gives dy = w * dout and dw = <dout, y>; the top-K
    renormalisation w = p_k / S (S = sum_k p_k, :329) gives dp_k = (dw_k - sum_j w_j dw_j) / S;
    the aux loss (:366-385) adds daux * E * f_e / T to every p[t, e] (counts carry no
    gradient); softmax backward dl = p * (dp - sum_e p dp); the expert chain
    down(ERA(gate) * up) (:295-298) and FlyLoRA's effective weight W + s U D (:123-126).

    Returns dx [T,H]; router dw_r [E,H], db_r [E]; per expert (stacked over E) dw_g / dw_u
    [E,I,H] and db_g / db_u [E,I] (base weights), dw_d [E,H,I], db_d [E,H]; FlyLoRA factors
    da_g / da_u (lora_down.weight) [E,r,H], dba_* [E,r], dl_g / dl_u (lora_up.weight) [E,I,r],
    dbl_* [E,I]; and the forward's routing (topk_idx).
    """
    f32 = np.float32
    x = p["x"].astype(f32)
    t, h = x.shape
    E, K, s = case.experts, case.top_k, f32(case.lora_scaling)
    dout = np.asarray(dout, dtype=f32)
    logits = router_logits(x, p["w_r"], p["b_r"])
    probs = softmax(logits)
    _, idx = topk_lowest_index(probs, K)
    if force_idx is not None:
        idx = np.asarray(force_idx, dtype=np.int64).reshape(t, K)
    vals = np.take_along_axis(probs, idx, axis=-1)
    ssum = vals.sum(axis=-1, keepdims=True)
    w = vals / ssum
    counts = np.bincount(idx.reshape(-1), minlength=E).astype(f32)

    g = {k: np.zeros_like(p[k], dtype=f32) for k in
         ("w_g", "b_g", "w_u", "b_u", "w_d", "b_d", "a_g", "ba_g", "l_g", "bl_g",
          "a_u", "ba_u", "l_u", "bl_u")}
    dx = np.zeros((t, h), dtype=f32)
    dw = np.zeros((t, K), dtype=f32)
    for e in range(E):
        mask = idx == e
        rows = np.nonzero(mask.any(axis=-1))[0]
        if rows.size == 0:
            continue
        kk = np.argmax(mask[rows], axis=-1)
        xe = x[rows]
        pre = {}
        for q in ("g", "u"):
            pre[q] = flylora_linear(xe, p[f"w_{q}"][e], p[f"b_{q}"][e], p[f"a_{q}"][e],
                                    p[f"ba_{q}"][e], p[f"l_{q}"][e], p[f"bl_{q}"][e], s, f32)
        a = era(pre["g"], case.era_gamma)
        hid = a * pre["u"]
        y = _mm(hid, p["w_d"][e], f32) + p["b_d"][e].astype(f32)
        we = w[rows, kk]
        dw[rows, kk] = (dout[rows] * y).sum(axis=-1)
        dy = dout[rows] * we[:, None]
        g["w_d"][e] = dy.T @ hid
        g["b_d"][e] = dy.sum(axis=0)
        dh = dy @ p["w_d"][e].astype(f32)
        dpre = {"g": dh * pre["u"] * era_grad(pre["g"], case.era_gamma), "u": dh * a}
        for q in ("g", "u"):
            dq = dpre[q]
            dW = dq.T @ xe                       # effective weight gradient
            db = dq.sum(axis=0)
            down = p[f"a_{q}"][e].astype(f32)    # D [r, H]
            up = p[f"l_{q}"][e].astype(f32)      # U [I, r]
            g[f"w_{q}"][e] = dW
            g[f"b_{q}"][e] = db
            g[f"l_{q}"][e] = s * (dW @ down.T + np.outer(db, p[f"ba_{q}"][e]))
            g[f"bl_{q}"][e] = s * db
            g[f"a_{q}"][e] = s * (up.T @ dW)
            g[f"ba_{q}"][e] = s * (up.T @ db)
            # x through base + s * lora_up(lora_down(x)) = x W_eff^T
            dx[rows] += dq @ (p[f"w_{q}"][e].astype(f32) + s * (up @ down))
    # router: top-K renormalisation, aux loss, softmax
    dvals = (dw - (dw * w).sum(axis=-1, keepdims=True)) / ssum
    dp = np.zeros_like(probs)
    np.put_along_axis(dp, idx, dvals, axis=-1)
    dp += f32(daux) * f32(E) * (counts / f32(t * K))[None, :] / f32(t)
    dl = probs * (dp - (probs * dp).sum(axis=-1, keepdims=True))
    out = {f"d{k}": v for k, v in g.items()}
    out["dw_r"] = dl.T @ x
    out["db_r"] = dl.sum(axis=0)
    out["dx"] = dx + dl @ p["w_r"].astype(f32)
    out["dlogits"] = dl
    out["topk_idx"] = idx
    return out


def layer_norm(x, w, b, eps):
    """nn.LayerNorm over the last axis (model.py:398-399): biased variance, affine."""
    x64 = np.asarray(x, dtype=np.float64)
    mu = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(axis=-1, keepdims=True)
    y = (x64 - mu) / np.sqrt(var + float(eps)) * np.asarray(w, np.float64) + np.asarray(b, np.float64)
    return y.astype(np.float32)


def prenorm_moe_forward(p, case, ln_w, ln_b, eps, **kw):
    """The FFN half of TransformerLayer.forward for a MoE layer (model.py:418-425):
    normed = ffn_norm(x); ffn_out, aux = ffn(normed); out = x + ffn_out.

    ``p["x"]`` is the residual stream; keyword arguments go to ``moe_forward`` (whose
    ``token_subset`` also selects the residual rows).
    """
    q = dict(p)
    q["x"] = layer_norm(p["x"], ln_w, ln_b, eps)
    r = moe_forward(q, case, **kw)
    sub = kw.get("token_subset")
    xr = p["x"] if sub is None else p["x"][np.asarray(sub, dtype=np.int64)]
    r["normed"] = q["x"]
    r["out"] = (xr.astype(np.float32) + r["out"]).astype(np.float32)
    return r


def norm_rel_err(got, ref):
    """max|got - ref| / max|ref|  (the tolerance metric of the parity tests)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.max(np.abs(ref)) if ref.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(got - ref))) if ref.size else 0.0
    return float(np.max(np.abs(got - ref)) / denom)
