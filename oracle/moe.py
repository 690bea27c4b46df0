"""Numpy restatement of the routed expert FFN (test infrastructure only).

Each function cites the reference code it restates (paths relative to the
seruva19/mirai tree).  Activations are held as float32 arrays; ``bf16=True``
rounds at the points where the reference's bf16 tensors round.
"""

from __future__ import annotations

import numpy as np

from .quant import bf16_round


def _r(x, bf16: bool):
    return bf16_round(x) if bf16 else np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------- a1 router

def softmax_f32(logits: np.ndarray) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp((x - m).astype(np.float32)).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def sigmoid_f32(logits: np.ndarray) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def route_topk(logits: np.ndarray, k: int, *, score_func: str = "softmax",
               bias: np.ndarray | None = None, norm: str = "clamp",
               route_scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    """Top-k routing on fp32 logits.

    ``norm="clamp"`` is ``TokenChoiceRouter`` (routers.py:241-249):
    softmax, top-k, ``w / clamp_min(sum w, 1e-20)``.
    ``norm="eps"`` is the LingBot router (transformer_lingbot_video.py:1002-1033):
    softmax or sigmoid scores, choice on ``scores + bias``, weights gathered
    from the unbiased scores, ``w / (sum w + 1e-20)`` when k > 1, times
    ``route_scale``.  ``norm="none"`` skips the renormalisation.

    The reference calls ``torch.topk(sorted=False)``, whose slot order is
    implementation-defined; this restatement returns the canonical order
    (descending choice score, equal scores by ascending expert id) and is
    compared with the reference by per-token index *sets*.  Selection ranks
    the choice scores; for softmax without bias it ranks the logits, which
    orders the same experts whenever the fp32 scores are distinct.
    """
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    scores = softmax_f32(logits) if score_func == "softmax" else sigmoid_f32(logits)
    if bias is not None:
        choice = (scores + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    elif score_func == "softmax":
        choice = logits
    else:
        choice = scores
    # stable descending sort: negate and use lexsort on (expert id, -choice)
    order = np.argsort(-choice, axis=1, kind="stable")[:, :k]
    w = np.take_along_axis(scores, order, axis=1).astype(np.float32)
    if norm == "clamp":
        s = np.maximum(w.sum(axis=1, keepdims=True, dtype=np.float32), np.float32(1e-20))
        w = (w / s).astype(np.float32)
    elif norm == "eps":
        if k > 1:
            s = (w.sum(axis=1, keepdims=True, dtype=np.float32) + np.float32(1e-20)).astype(np.float32)
            w = (w / s).astype(np.float32)
        w = (w * np.float32(route_scale)).astype(np.float32)
    return order.astype(np.int64), w


def canonical_slots(idx: np.ndarray, w: np.ndarray | None = None):
    """Sort each token's slots by expert id (for set comparison)."""
    order = np.argsort(idx, axis=1, kind="stable")
    ci = np.take_along_axis(idx, order, axis=1)
    if w is None:
        return ci
    return ci, np.take_along_axis(w, order, axis=1)


# ----------------------------------------------------------------------------- a2 dispatch plan

def dispatch_plan(top_idx: np.ndarray, num_experts: int) -> dict:
    """``build_dispatch_plan`` (dispatch_preprocess.py:128-179)."""
    top_idx = np.asarray(top_idx, dtype=np.int64)
    T, k = top_idx.shape
    flat = top_idx.reshape(-1)
    sort_positions = np.argsort(flat, kind="stable").astype(np.int64)
    counts = np.bincount(flat, minlength=num_experts).astype(np.int64)
    cumsum = np.cumsum(counts)
    inverse = np.empty_like(sort_positions)
    inverse[sort_positions] = np.arange(flat.size, dtype=np.int64)
    return {
        "counts": counts,
        "starts": (cumsum - counts).astype(np.int64),
        "offsets": cumsum.astype(np.int32),
        "sort_positions": sort_positions,
        "sorted_token_indices": (sort_positions // k).astype(np.int64),
        "inverse_order": inverse,
    }


# ----------------------------------------------------------------------------- a3 / a8 permute, combine

def permute(tokens: np.ndarray, sorted_token_indices: np.ndarray) -> np.ndarray:
    """``permute_routed_tokens`` forward (dispatch_ops.py:8-20)."""
    return np.asarray(tokens)[np.asarray(sorted_token_indices)]


def combine(expert_out_sorted: np.ndarray, top_w: np.ndarray, plan: dict, T: int) -> np.ndarray:
    """fp32 weighted un-permute: ``out.index_add_(0, tok, y.float() * w)`` in sorted order
    (experts.py:2433-2437, dispatch_ops.py:23-44).  Returns fp32 [T, H]."""
    k = top_w.shape[1]
    sp = plan["sort_positions"]
    tok = sp // k
    w_sorted = np.asarray(top_w, dtype=np.float32).reshape(-1)[sp]
    contrib = (np.asarray(expert_out_sorted, dtype=np.float32) * w_sorted[:, None]).astype(np.float32)
    out = np.zeros((T, expert_out_sorted.shape[1]), dtype=np.float32)
    np.add.at(out, tok, contrib)  # sequential in sorted order, like CPU index_add_
    return out


# ----------------------------------------------------------------------------- a6-a8 forward

def silu_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def expert_ffn_forward(x_sorted: np.ndarray, offsets: np.ndarray, w1: np.ndarray, w3: np.ndarray,
                       w2: np.ndarray, *, bf16: bool = True, lora: dict | None = None,
                       keep: bool = False):
    """Per-expert SwiGLU MLP over expert-contiguous rows.

    ``w1``/``w3`` are [E, I, H], ``w2`` is [E, H, I] (dequantised values, as
    produced by the reference's dequant-then-bmm path, linear.py:166-203 and
    experts.py:301-317).  ``lora`` (optional) is ``{"a": [E, r, I], "b": [E, H, r],
    "scale": float}`` on the down projection (active_expert_lora.py:434-478).
    Returns y [S, H] (and the gate/up/h intermediates when ``keep``).
    """
    S, H = x_sorted.shape
    E, I, _ = w1.shape
    y = np.zeros((S, H), dtype=np.float32)
    gate_all = np.zeros((S, I), dtype=np.float32)
    up_all = np.zeros((S, I), dtype=np.float32)
    h_all = np.zeros((S, I), dtype=np.float32)
    start = 0
    for e in range(E):
        end = int(offsets[e])
        if end > start:
            xe = x_sorted[start:end].astype(np.float32)
            gate = _r(xe @ w1[e].T, bf16)
            up = _r(xe @ w3[e].T, bf16)
            h = _r(_r(silu_f32(gate), bf16) * up, bf16)
            ye = _r(h @ w2[e].T, bf16)
            if lora is not None:
                low = _r(h @ lora["a"][e].T, bf16)
                delta = _r(_r(low @ lora["b"][e].T, bf16) * np.float32(lora["scale"]), bf16)
                ye = _r(ye + delta, bf16)
            y[start:end] = ye
            gate_all[start:end] = gate
            up_all[start:end] = up
            h_all[start:end] = h
        start = end
    if keep:
        return y, {"gate": gate_all, "up": up_all, "h": h_all}
    return y


def moe_forward(x: np.ndarray, top_idx: np.ndarray, top_w: np.ndarray, w1, w3, w2, *,
                bf16: bool = True, lora: dict | None = None) -> np.ndarray:
    """``run_direct_routed`` semantics (experts.py:1749-1912, vectorized runner
    experts.py:2329-2438): plan, permute, expert MLPs, fp32 combine, cast."""
    E = w1.shape[0]
    T = x.shape[0]
    plan = dispatch_plan(top_idx, E)
    xs = permute(x, plan["sorted_token_indices"])
    y = expert_ffn_forward(xs, plan["offsets"], w1, w3, w2, bf16=bf16, lora=lora)
    out = combine(y, top_w, plan, T)
    return _r(out, bf16)


# ----------------------------------------------------------------------------- a9 dX

def silu_backward_f32(grad: np.ndarray, x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)
    return (grad * sig * (np.float32(1.0) + x * (np.float32(1.0) - sig))).astype(np.float32)


def expert_ffn_backward(grad_y: np.ndarray, offsets: np.ndarray, w1, w3, w2, inter: dict, *, bf16: bool = True,
                        lora: dict | None = None) -> np.ndarray:
    """Per-expert input gradient of the SwiGLU MLP over expert-contiguous rows
    (linear.py:116-125, 191-203 and autograd of experts.py:301-317), given the
    forward's ``gate`` / ``up`` intermediates (``expert_ffn_forward(keep=True)``)."""
    E = w1.shape[0]
    dxs = np.zeros((grad_y.shape[0], w1.shape[2]), dtype=np.float32)
    start = 0
    for e in range(E):
        end = int(offsets[e])
        if end > start:
            gy = grad_y[start:end]
            gate = inter["gate"][start:end]
            up = inter["up"][start:end]
            dh = _r(gy @ w2[e], bf16)
            if lora is not None:
                dlow_out = _r(gy * np.float32(lora["scale"]), bf16)
                dlow = _r(dlow_out @ lora["b"][e], bf16)
                dh = _r(dh + _r(dlow @ lora["a"][e], bf16), bf16)
            act = _r(silu_f32(gate), bf16)
            d_act = _r(dh * up, bf16)
            d_up = _r(dh * act, bf16)
            d_gate = _r(silu_backward_f32(d_act, gate), bf16)
            dxs[start:end] = _r(_r(d_gate @ w1[e], bf16) + _r(d_up @ w3[e], bf16), bf16)
        start = end
    return dxs


def moe_backward_dx(x: np.ndarray, top_idx: np.ndarray, top_w: np.ndarray, w1, w3, w2,
                    grad_out: np.ndarray, *, bf16: bool = True, lora: dict | None = None):
    """Input gradient through frozen experts (linear.py:116-125, 191-203;
    dispatch_ops.py:15-20, 36-44).  Returns (dx [T,H], d_top_w [T,k])."""
    E = w1.shape[0]
    T, k = top_idx.shape
    plan = dispatch_plan(top_idx, E)
    xs = permute(x, plan["sorted_token_indices"])
    y, inter = expert_ffn_forward(xs, plan["offsets"], w1, w3, w2, bf16=bf16, lora=lora, keep=True)
    sp = plan["sort_positions"]
    tok = sp // k
    w_sorted = np.asarray(top_w, dtype=np.float32).reshape(-1)[sp]
    g = np.asarray(grad_out, dtype=np.float32)[tok]
    grad_y = _r(g * w_sorted[:, None], bf16)
    grad_w_sorted = (g * y).sum(axis=1, dtype=np.float32)
    grad_w = np.zeros(T * k, dtype=np.float32)
    grad_w[sp] = grad_w_sorted
    dxs = expert_ffn_backward(grad_y, plan["offsets"], w1, w3, w2, inter, bf16=bf16, lora=lora)
    dx = np.zeros((T, x.shape[1]), dtype=np.float32)
    if bf16:
        # permute backward accumulates in the activation dtype, sequentially in
        # sorted order: per token, add its slots by ascending sorted position
        pos_by_token = np.sort(plan["inverse_order"].reshape(T, k), axis=1)
        for r in range(k):
            dx = bf16_round(dx + dxs[pos_by_token[:, r]])
    else:
        np.add.at(dx, tok, dxs)
    return dx, grad_w.reshape(T, k)


def rel_max_err(a: np.ndarray, r: np.ndarray) -> float:
    """max|a - r| / max|r| -- the north-star tolerance metric."""
    a = np.asarray(a, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    den = np.abs(r).max()
    return float(np.abs(a - r).max() / den) if den > 0 else float(np.abs(a - r).max())


# ----------------------------------------------------------------------------- f4: MAGI-2 multi-head grouped MoE

def magi2_route(x_heads: np.ndarray, gate: np.ndarray, expert_bias: np.ndarray | None, *, experts: int,
                top_k: int, score_func: str = "sigmoid", route_norm: bool = True, route_scale: float = 1.0):
    """MAGI-2 router (magi2_preview.py:2727-2744; flash_mh_moe/route.py:28-154,
    torch path without virtual groups): per head h, logits = x_heads[:, h] @
    gate[h]^T in fp32, sigmoid / softmax scores, top-k of score +
    expert_bias[h] (descending, ties to the lower id), weights gathered from
    the unbiased scores, F.normalize(p=1, eps=1e-12) when route_norm, times
    route_scale.  Returns (probs [H, S, k], indices [H, S, k])."""
    S, H, d = x_heads.shape
    g = np.asarray(gate, dtype=np.float32).reshape(H, experts, d)
    logits = np.einsum("shd,hed->hse", np.asarray(x_heads, dtype=np.float32), g).astype(np.float32)
    scores = sigmoid_f32(logits) if score_func == "sigmoid" else softmax_f32(logits)
    choice = scores if expert_bias is None else (scores + np.asarray(expert_bias, np.float32).reshape(H, 1, experts))
    order = np.argsort(-choice, axis=-1, kind="stable")[..., :top_k]
    w = np.take_along_axis(scores, order, axis=-1).astype(np.float32)
    if route_norm:
        w = (w / np.maximum(np.abs(w).sum(-1, keepdims=True, dtype=np.float32), np.float32(1e-12))).astype(np.float32)
    return (w * np.float32(route_scale)).astype(np.float32), order.astype(np.int64)


def swiglu7_f32(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """grouped_moe.py:287-306 on fp32 copies of bf16 gate / up."""
    g = np.minimum(np.asarray(gate, np.float32), np.float32(7.0))
    u = np.clip(np.asarray(up, np.float32), np.float32(-7.0), np.float32(7.0))
    return (g * sigmoid_f32(np.float32(1.702) * g) * (u + np.float32(1.0))).astype(np.float32)


def swiglu7_backward_f32(grad: np.ndarray, gate: np.ndarray, up: np.ndarray):
    """grouped_moe.py:309-335 (the same as autograd of the clamps and products)."""
    gr = np.asarray(gate, np.float32)
    ur = np.asarray(up, np.float32)
    g = np.minimum(gr, np.float32(7.0))
    u = np.clip(ur, np.float32(-7.0), np.float32(7.0))
    s = sigmoid_f32(np.float32(1.702) * g)
    dgate = (s + np.float32(1.702) * g * s * (np.float32(1.0) - s)) * (gr <= 7.0)
    d_g = (grad * dgate * (u + np.float32(1.0))).astype(np.float32)
    d_u = (grad * (g * s) * ((ur >= -7.0) & (ur <= 7.0))).astype(np.float32)
    return d_g, d_u


def magi2_experts(x_heads: np.ndarray, probs: np.ndarray, idx: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray,
                  w_down: np.ndarray, grad_out: np.ndarray | None = None):
    """``CoreMultiHeadMoE._torch_forward`` (magi2_preview.py:2770-2793) in bf16,
    and, with ``grad_out``, its autograd: per head, per expert (ascending), the
    selected tokens' gate = bf16(x W_gate[g]), up = bf16(x W_up[g]), h =
    bf16(swiglu7), y = bf16(h W_down[g]), added as bf16(y * bf16(w)) into a bf16
    output.  Weights are [G, in, out] with G = heads * experts.
    Returns out [S, H, d] (and dx [S, H, d], dprobs [H, S, k])."""
    S, H, d = x_heads.shape
    E = w_gate.shape[0] // H
    x = bf16_round(np.asarray(x_heads, np.float32))
    out = np.zeros((S, H, d), np.float32)
    dx = np.zeros((S, H, d), np.float32)
    dprobs = np.zeros(idx.shape, np.float32)
    for h in range(H):
        for e in range(E):
            tok, slot = np.nonzero(idx[h] == e)
            if tok.size == 0:
                continue
            gidx = h * E + e
            xs = x[tok, h]
            gate = bf16_round(xs @ w_gate[gidx])
            up = bf16_round(xs @ w_up[gidx])
            hid = bf16_round(swiglu7_f32(gate, up))
            y = bf16_round(hid @ w_down[gidx])
            wb = bf16_round(probs[h, tok, slot])
            contrib = bf16_round(y * wb[:, None])
            for r, t in enumerate(tok):  # index_add_: rows in order, bf16 running sum
                out[t, h] = bf16_round(out[t, h] + contrib[r])
            if grad_out is None:
                continue
            g = bf16_round(np.asarray(grad_out, np.float32)[tok, h])
            dy = bf16_round(g * wb[:, None])
            dprobs[h, tok, slot] = bf16_round((g * y).sum(axis=1, dtype=np.float32))
            dh = bf16_round(dy @ w_down[gidx].T)
            d_g, d_u = swiglu7_backward_f32(dh, gate, up)
            d_g, d_u = bf16_round(d_g), bf16_round(d_u)
            dxs = bf16_round(bf16_round(d_g @ w_gate[gidx].T) + bf16_round(d_u @ w_up[gidx].T))
            for r, t in enumerate(tok):
                dx[t, h] = bf16_round(dx[t, h] + dxs[r])
    if grad_out is None:
        return out
    return out, dx, dprobs
