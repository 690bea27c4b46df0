"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py``, which imports and runs
the seruva19/mirai reference on the CPU.  These tests need no GPU.
"""

import numpy as np
import pytest

from oracle import moe as om
from oracle import quant as oq


@pytest.mark.parametrize("name", ["router_e8_k2", "router_e64_k4", "router_e128_k8"])
def test_router_topk_sets_match_reference(golden, name):
    g = golden(name)
    k = int(g["k"])
    idx, w = om.route_topk(g["logits"], k, norm="clamp")
    ci, cw = om.canonical_slots(idx, w)
    ri, rw = om.canonical_slots(g["top_indices"], g["top_weights"])
    np.testing.assert_array_equal(ci, ri)  # bit-exact index sets
    np.testing.assert_allclose(cw, rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("name", ["plan_uniform", "plan_dups_empty", "plan_single", "plan_skew"])
def test_dispatch_plan_matches_reference(golden, name):
    g = golden(name)
    plan = om.dispatch_plan(g["top_indices"], int(g["num_experts"]))
    for field in ("counts", "starts", "offsets", "sort_positions", "sorted_token_indices", "inverse_order"):
        np.testing.assert_array_equal(plan[field], g[field], err_msg=field)


def test_permute_combine_forward_backward(golden):
    g = golden("permute_combine")
    tokens, idx, scores = g["tokens"], g["indices"], g["scores"]
    routed = om.permute(tokens, idx)
    expert_out = (routed * np.float32(1.5) - np.float32(0.25)).astype(np.float32)
    out = np.zeros_like(tokens)
    np.add.at(out, idx, expert_out * scores[:, None])
    np.testing.assert_allclose(out, g["out"], rtol=1e-6, atol=1e-6)
    gathered = g["grad"][idx]
    grad_tokens = np.zeros_like(tokens)
    np.add.at(grad_tokens, idx, gathered * scores[:, None] * np.float32(1.5))
    np.testing.assert_allclose(grad_tokens, g["grad_tokens"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose((gathered * expert_out).sum(1), g["grad_scores"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("gsz", [0, 16, 64, 256])
def test_int8_quantizer_matches_reference(golden, gsz):
    g = golden("int8_quant")
    q, s, gres = oq.int8_quantize(g["weight"], gsz)
    assert gres == int(g[f"gres_g{gsz}"])
    np.testing.assert_array_equal(s, g[f"s_g{gsz}"]) if gsz == 0 else \
        np.testing.assert_allclose(s, g[f"s_g{gsz}"], rtol=1e-6)
    diff = q.astype(np.int32) - g[f"q_g{gsz}"].astype(np.int32)
    if gsz == 0:
        assert not diff.any()
    else:  # rotation matmul order differs from torch's; only rounding ties may move by one step
        assert np.abs(diff).max() <= 1 and (diff != 0).mean() < 1e-3
    deq = oq.int8_dequantize(g[f"q_g{gsz}"], g[f"s_g{gsz}"], gres)
    np.testing.assert_allclose(deq, g[f"deq_g{gsz}"], rtol=1e-5, atol=1e-6)


def _routed_weights(g):
    if "w1_int8" in g:
        gsz = int(g["group_size"])
        ws = [oq.int8_dequantize(g[f"{k}_int8"], g[f"{k}_scale"], gsz) for k in ("w1", "w3", "w2")]
    else:
        ws = [oq.bf16_bits_to_f32(g[k]) for k in ("w1", "w3", "w2")]
    if bool(g["bf16"]):
        ws = [oq.bf16_round(w) for w in ws]
    return ws


def _act(g, key):
    v = g[key]
    return oq.bf16_bits_to_f32(v) if v.dtype == np.uint16 else v.astype(np.float32)


@pytest.mark.parametrize("name", ["routed_int8_fp32", "routed_int8_g16_fp32", "routed_int8_bf16",
                                  "routed_dense_bf16", "routed_dense_bf16_lora"])
def test_routed_forward_and_dx_match_reference(golden, name):
    g = golden(name)
    bf16 = bool(g["bf16"])
    w1, w3, w2 = _routed_weights(g)
    x = _act(g, "tokens")
    tw = _act(g, "top_scores")
    lora = None
    if "lora_a" in g:
        lora = {"a": oq.bf16_round(g["lora_a"]) if bf16 else g["lora_a"],
                "b": oq.bf16_round(g["lora_b"]) if bf16 else g["lora_b"],
                "scale": float(g["lora_scale"])}
    out = om.moe_forward(x, g["top_indices"], tw, w1, w3, w2, bf16=bf16, lora=lora)
    ref = _act(g, "out")
    tol = 2e-2 if bf16 else 1e-5
    assert om.rel_max_err(out, ref) < tol
    dx, dw = om.moe_backward_dx(x, g["top_indices"], tw, w1, w3, w2, _act(g, "grad"), bf16=bf16, lora=lora)
    assert om.rel_max_err(dx, _act(g, "grad_tokens")) < (3e-2 if bf16 else 1e-5)
    assert om.rel_max_err(dw, _act(g, "grad_scores")) < (3e-2 if bf16 else 1e-5)


def test_nf4_roundtrip_properties():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((2, 64, 128)) * 0.05).astype(np.float32)
    g = oq.nf4_quantize_grouped(w)
    assert g["nf4"].shape == (2, 64 * 128 // 2, 1) and g["nf4"].dtype == np.uint8
    assert g["absmax"].shape == (2, 64 * 128 // 64) and g["absmax"].dtype == np.uint8
    assert g["nabsmax"].shape == (2, -(-(64 * 128 // 64) // 256))
    d = oq.nf4_dequantize_grouped(g)
    # re-quantising the dequantised weight is idempotent on the codes
    g2 = oq.nf4_quantize_grouped(d)
    assert (g2["nf4"] == g["nf4"]).mean() > 0.99
    err = np.abs(d - w).mean() / np.abs(w).mean()
    assert err < 0.12
    code = oq.nf4_code_table()
    assert code[0] == -1.0 and code[-1] == 1.0 and code[7] == 0.0 and np.all(np.diff(code) > 0)
    ncode = oq.dynamic_tree_map()
    assert ncode.shape == (256,) and ncode[-1] == 1.0 and np.all(np.diff(ncode) >= 0)


def test_magi2_oracle_matches_the_reference_layer(golden):
    """The numpy restatement of MAGI-2's multi-head MoE (oracle.moe.magi2_*)
    against the reference's CoreMultiHeadMoE (fixture recorded from it):
    routes bit-exact as index sets, forward and autograd within bf16
    matmul-ordering differences."""
    g = golden("magi2_moe")
    b = lambda k: oq.bf16_bits_to_f32(g[k])
    H, E, k = int(g["heads"]), int(g["experts"]), int(g["top_k"])
    x = b("x")
    S = x.shape[0]
    xh = x.reshape(S, H, -1)
    p, i = om.magi2_route(xh, g["gate"], g["expert_bias"], experts=E, top_k=k, route_scale=float(g["route_scale"]))
    ci, cw = om.canonical_slots(i.reshape(-1, k), p.reshape(-1, k))
    ri, rw = om.canonical_slots(g["topk_indices"].reshape(-1, k), g["topk_probs"].reshape(-1, k))
    np.testing.assert_array_equal(ci, ri)
    np.testing.assert_allclose(cw, rw, rtol=1e-5, atol=1e-6)
    out, dx, dp = om.magi2_experts(xh, g["topk_probs"], g["topk_indices"], b("W_gate"), b("W_up"), b("W_down"),
                                   b("grad").reshape(xh.shape))
    assert om.rel_max_err(out.reshape(S, -1), b("out")) < 2e-3
    assert om.rel_max_err(dx, b("grad_x_heads")) < 5e-3
    assert om.rel_max_err(dp, g["grad_probs"]) < 1e-2


def test_magi2_flat_routes_follow_the_reference_order():
    """(token, head) rows with flat group ids head * E + expert: a stable sort
    of them lists each group's tokens in ascending order, the order of the
    reference's argsort over (head, token, k) (grouped_moe.py:660-666)."""
    import torch
    from mirai_b200.magi2 import _flat_routes
    rng = np.random.default_rng(0)
    H, S, k, E = 3, 7, 2, 5
    idx = np.stack([np.stack([rng.permutation(E)[:k] for _ in range(S)]) for _ in range(H)])
    probs = rng.random((H, S, k)).astype(np.float32)
    flat, pr = _flat_routes(torch.from_numpy(probs), torch.from_numpy(idx), E)
    assert flat.shape == (S * H, k) and torch.equal(flat[1 * H + 2], torch.from_numpy(idx[2, 1] + 2 * E))
    assert torch.equal(pr[1 * H + 2], torch.from_numpy(probs[2, 1]))
    ours = np.argsort(flat.numpy().reshape(-1), kind="stable")
    rows_ours = ours // k  # row = token * H + head
    ref_flat = (idx + (np.arange(H) * E)[:, None, None]).reshape(-1)
    ref_order = np.argsort(ref_flat, kind="stable")
    ref_rows = ((ref_order % (S * k)) // k) * H + ref_order // (S * k)
    np.testing.assert_array_equal(rows_ours, ref_rows)
