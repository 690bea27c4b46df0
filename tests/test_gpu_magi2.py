"""MAGI-2's multi-head grouped MoE (f4) on the GPU: the [G, in, out] weight
layout read as stored, the swiglu7 epilogue and its backward, more than 1024
(head, expert) groups, the per-head router bias and the bf16-accumulating
combine -- against the reference's own layer (fixture) and the oracle."""

import numpy as np
import pytest
import torch

from oracle import moe as om
from oracle import quant as oq

pytestmark = pytest.mark.gpu
TOL, TOL_DX = 2e-2, 3e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mirai_b200.build import build
    build()
    return torch.device("cuda:0")


def _np(t):
    return t.detach().float().cpu().numpy()


def test_magi2_layer_against_the_reference(golden):
    dev = _dev()
    from mirai_b200 import ops
    from mirai_b200.magi2 import Magi2ExpertWeights, route, run_experts
    g = golden("magi2_moe")
    bits = lambda k: torch.from_numpy(oq.bf16_bits_to_f32(g[k])).to(torch.bfloat16).to(dev)
    H, E, k = int(g["heads"]), int(g["experts"]), int(g["top_k"])
    x = bits("x")
    S = x.shape[0]
    d = x.shape[1] // H
    xh = x.view(S, H, d)
    ws = Magi2ExpertWeights(bits("W_gate"), bits("W_up"), bits("W_down"), heads=H, experts=E, d_head=d,
                            d_expert=g["W_gate"].shape[2])
    probs, idx = route(xh, torch.from_numpy(g["gate"]).to(dev), torch.from_numpy(g["expert_bias"]).to(dev),
                       experts=E, top_k=k, route_scale=float(g["route_scale"]))
    ci, cw = om.canonical_slots(idx.cpu().numpy().reshape(-1, k), probs.cpu().numpy().reshape(-1, k))
    ri, rw = om.canonical_slots(g["topk_indices"].reshape(-1, k), g["topk_probs"].reshape(-1, k))
    np.testing.assert_array_equal(ci, ri)
    np.testing.assert_allclose(cw, rw, rtol=1e-5, atol=1e-6)
    with torch.no_grad():
        out = run_experts(xh, probs, idx, ws)
    assert om.rel_max_err(_np(out).reshape(S, -1), oq.bf16_bits_to_f32(g["out"])) < TOL
    # the experts' autograd given the reference's routes
    xg = xh.clone().requires_grad_(True)
    pg = torch.from_numpy(g["topk_probs"]).to(dev).requires_grad_(True)
    eo = run_experts(xg, pg, torch.from_numpy(g["topk_indices"]).to(dev), ws)
    eo.backward(bits("grad").view(S, H, d))
    ops.check_device()
    assert om.rel_max_err(_np(eo).reshape(S, -1), oq.bf16_bits_to_f32(g["experts_out"]).reshape(S, -1)) < TOL
    assert om.rel_max_err(_np(xg.grad), oq.bf16_bits_to_f32(g["grad_x_heads"])) < TOL_DX
    assert om.rel_max_err(_np(pg.grad), g["grad_probs"]) < TOL_DX


def _magi2_case(dev, *, S, H, E, k, d, I, fmt, seed):
    from mirai_b200 import ops, tables
    from mirai_b200.magi2 import Magi2ExpertWeights, route
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(S, H, d, generator=gen, device=dev).to(torch.bfloat16)
    gate = torch.randn(H * E, d, generator=gen, device=dev) * 0.05
    bias = torch.randn(H * E, generator=gen, device=dev) * 0.05
    raw = [(torch.randn(s, generator=gen, device=dev) * 0.05).to(torch.bfloat16)
           for s in ((H * E, d, I), (H * E, d, I), (H * E, I, d))]
    if fmt == "nf4":  # the NF4 store quantises each group's stored [in, out] matrix row-major
        ws_t = [ops.nf4_quantize(w, tables.nf4_code(dev), tables.dynamic_map(dev)) for w in raw]
    else:
        ws_t = raw
    ws = Magi2ExpertWeights(*ws_t, heads=H, experts=E, d_head=d, d_expert=I)
    probs, idx = route(x, gate, bias, experts=E, top_k=k, route_scale=4.9)
    return x, probs, idx, raw, ws_t, ws


def _oracle_weights(fmt, ws_t, raw, groups):
    out = []
    for w, r in zip(ws_t, raw):
        if fmt == "nf4":
            _, o, i = w.shape
            dense = np.stack([oq.nf4_dequantize_2d({
                "packed": w.packed[gi].cpu().numpy(), "absmax": w.absmax[gi].cpu().numpy(),
                "nested_absmax": w.nested_absmax[gi].cpu().numpy(), "offset": w.offset[gi].cpu().numpy(),
                "code": w.code.cpu().numpy(), "nested_code": w.nested_code.cpu().numpy()}, (o, i)) for gi in groups])
        else:
            dense = r[groups].float().cpu().numpy()
        out.append(dense)
    return out


@pytest.mark.parametrize("fmt,S,H,E,k,d,I", [
    ("bf16", 1024, 12, 128, 6, 128, 256),      # 1536 groups: two GEMM launches, a 1536-group plan
    ("nf4", 1024, 12, 128, 6, 128, 256),
    ("nf4", 512, 12, 256, 6, 256, 1280),       # MAGI-2's own sizes: 3072 groups, d_head 256, d_expert 1280
])
def test_magi2_many_groups_against_the_oracle(fmt, S, H, E, k, d, I):
    """More than 1024 (head, expert) groups, forward and dX, on a seeded subset
    of tokens recomputed by the oracle (each token's rows depend on its own
    routes only; the subset's groups are renumbered in ascending order)."""
    dev = _dev()
    from mirai_b200 import ops
    from mirai_b200.magi2 import run_experts
    x, probs, idx, raw, ws_t, ws = _magi2_case(dev, S=S, H=H, E=E, k=k, d=d, I=I, fmt=fmt, seed=S + E)
    xg = x.clone().requires_grad_(True)
    pg = probs.clone().requires_grad_(True)
    out = run_experts(xg, pg, idx, ws)
    grad = torch.randn(out.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(3)).to(torch.bfloat16)
    out.backward(grad)
    ops.check_device()
    tokens = np.sort(np.random.default_rng(S).choice(S, 6, replace=False))
    gi = idx.cpu().numpy()[:, tokens]                                  # [H, t, k] expert ids per head
    xs, gs, ps = _np(x)[tokens], _np(grad)[tokens], probs.cpu().numpy()[:, tokens]
    ref, rdx, rdp = np.zeros_like(xs), np.zeros_like(xs), np.zeros_like(ps)
    for h in range(H):  # heads are independent: one single-head oracle call per head, its used experts only
        used = np.unique(gi[h])
        w_h = _oracle_weights(fmt, ws_t, raw, h * E + used)
        o, dxh, dph = om.magi2_experts(xs[:, h:h + 1], ps[h:h + 1], np.searchsorted(used, gi[h:h + 1]), *w_h,
                                       grad_out=gs[:, h:h + 1])
        ref[:, h:h + 1], rdx[:, h:h + 1], rdp[h:h + 1] = o, dxh, dph
    assert om.rel_max_err(_np(out)[tokens], ref) < TOL
    assert om.rel_max_err(_np(xg.grad)[tokens], rdx) < TOL_DX
    assert om.rel_max_err(_np(pg.grad)[:, tokens], rdp) < TOL_DX


def test_magi2_backend_seam_and_token_chunks():
    """B200Magi2MoEBackend.execute(module, x_heads, topk_probs, topk_indices)
    on a module shaped like CoreMultiHeadMoE (bf16 W_gate / W_up / W_down), and
    the same with token chunks: identical results."""
    dev = _dev()
    import types
    from mirai_b200.magi2 import B200Magi2MoEBackend, attach
    x, probs, idx, raw, ws_t, ws = _magi2_case(dev, S=300, H=4, E=16, k=2, d=128, I=128, fmt="bf16", seed=5)
    mod = types.SimpleNamespace(num_heads=4, num_experts=16, d_head=128, d_expert=128, W_gate=raw[0], W_up=raw[1],
                                W_down=raw[2], _mirai_moe_kernel_backend=None, _parameters={}, _buffers={})
    model = types.SimpleNamespace(modules=lambda: [mod])
    assert attach(model) == 1 and isinstance(mod._mirai_moe_kernel_backend, B200Magi2MoEBackend)
    a = mod._mirai_moe_kernel_backend.execute(mod, x, probs, idx)
    b = B200Magi2MoEBackend(token_chunk_size=64).execute(mod, x, probs, idx)
    assert torch.equal(a, b)
