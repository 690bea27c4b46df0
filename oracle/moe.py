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
    dxs = np.zeros_like(xs, dtype=np.float32)
    start = 0
    for e in range(E):
        end = int(plan["offsets"][e])
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
