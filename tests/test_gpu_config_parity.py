"""Parity at the benchmarked configurations' own shapes.

``bench.py`` times c2 (T=32768, H=2048, E=32, k=2, I=1408, NF4, forward + dX
with a rank-16 LoRA on w2), c3 (T=8192, H=3072, E=64, k=4, I=1024, INT8,
Zipf-skewed load with many segments under 64 rows) and the c4 layer shape
(H=4096 -- the largest reduction the quantised GEMMs accept -- E=128, k=8,
I=1536, NF4).  Each test runs the whole layer on the GPU at that shape and
checks it against the CPU oracle:

* routing index sets over every token and every field of the dispatch plan
  over every route: bit-exact;
* outputs, dX and top-score gradients of a seeded subset of tokens: the
  oracle recomputes only those tokens' routes (a token's result depends on
  its own routed rows alone; expert ids are renumbered monotonically so the
  per-token order of the fp32 combine is unchanged), max|a - r| / max|r|
  <= 2e-2 forward and 3e-2 for the gradients.

The expert weights are quantised on the GPU and their buffers copied to the
host: the oracle dequantises those exact buffers (the GPU quantiser is
compared bit-exact with the oracle's separately, here on one expert).
"""

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest
import torch

from oracle import moe as om
from oracle import quant as oq

pytestmark = pytest.mark.gpu

TOL, TOL_DX = 2e-2, 3e-2
THREADS = max(1, min(32, os.cpu_count() or 1))


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mirai_b200.build import build
    build()
    return torch.device("cuda:0")


def _np(t):
    return t.detach().float().cpu().numpy()


def _workload(T, H, E, I, fmt, seed, dev, zipf=None, rotated=False):
    """Seeded tokens, router logits and GPU-quantised experts (bench.py's recipe)."""
    from mirai_b200 import ops, tables
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(E, H, generator=g, device=dev) * 0.02
    logits = x.float() @ gate.T
    if zipf:
        perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
        p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** zipf
        p = (p / p.sum())[perm.argsort()].to(torch.float32).to(dev)
        logits = logits + 2.0 * torch.log(p)[None, :]
    raw = [(torch.randn(s, generator=g, device=dev) * 0.02).to(torch.bfloat16) for s in ((E, I, H), (E, I, H), (E, H, I))]
    if fmt == "nf4":
        ws = [ops.nf4_quantize(w, tables.nf4_code(dev), tables.dynamic_map(dev)) for w in raw]
    else:
        groups = (oq.best_group_size(H), oq.best_group_size(H), oq.best_group_size(I)) if rotated else (0, 0, 0)
        ws = [ops.int8_quantize(w.float(), group_size=gs) for w, gs in zip(raw, groups)]
    torch.cuda.synchronize()
    return x, logits, raw, ws


def _dense_experts(fmt, ws, experts):
    """Oracle dequantisation of the given experts of each key, from the GPU's buffers."""
    def one(args):
        key, e = args
        w = ws[key]
        if fmt == "nf4":
            _, o, i = w.shape
            return oq.nf4_dequantize_2d({"packed": w.packed[e].cpu().numpy(), "absmax": w.absmax[e].cpu().numpy(),
                                         "nested_absmax": w.nested_absmax[e].cpu().numpy(),
                                         "offset": w.offset[e].cpu().numpy(), "code": w.code.cpu().numpy(),
                                         "nested_code": w.nested_code.cpu().numpy()}, (o, i))
        return oq.bf16_round(oq.int8_dequantize(w.q[e].cpu().numpy(), w.scale[e].cpu().numpy(), w.group_size))

    jobs = [(key, int(e)) for key in range(3) for e in experts]
    with ThreadPoolExecutor(THREADS) as pool:
        flat = list(pool.map(one, jobs))
    n = len(experts)
    return [np.stack(flat[key * n:(key + 1) * n]) for key in range(3)]


def _subset_oracle(fmt, ws, x, idx, tw, g_out, tokens, lora=None):
    """Oracle forward and dX for the chosen tokens, with only their experts
    dequantised (ids renumbered in ascending order)."""
    sub_idx = idx[tokens]
    experts = np.unique(sub_idx)
    remap = np.searchsorted(experts, sub_idx)
    w1, w3, w2 = _dense_experts(fmt, ws, experts)
    ol = None
    if lora is not None:
        ol = {"a": lora["a"][experts], "b": lora["b"][experts], "scale": lora["scale"]}
    xs = x[tokens]
    ref = om.moe_forward(xs, remap, tw[tokens], w1, w3, w2, bf16=True, lora=ol)
    rdx, rdw = om.moe_backward_dx(xs, remap, tw[tokens], w1, w3, w2, g_out[tokens], bf16=True, lora=ol)
    return ref, rdx, rdw


def _check_routing_and_plan(ops, logits, idx, tw, plan, k, E):
    lg = logits.cpu().numpy()
    ridx, rw = om.route_topk(lg, k)
    gi = idx.cpu().numpy()
    np.testing.assert_array_equal(gi, ridx)  # canonical slot order: descending score, ties to the lower id
    np.testing.assert_allclose(tw.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
    ref = om.dispatch_plan(gi, E)
    for f in ("counts", "starts", "offsets", "sort_positions", "sorted_token_indices", "inverse_order"):
        np.testing.assert_array_equal(getattr(plan, f).cpu().numpy(), ref[f], err_msg=f)
    return gi, ref


def _run_layer(ops, x, logits, ws, k, E, I, g_out, lora=None):
    idx, tw = ops.route_topk(logits, k)
    out, st = ops.moe_forward_train(x, idx, tw, *ws, num_experts=E, inter=I, lora=lora)
    dx, dw = ops.moe_backward_dx(g_out, st, *ws, inter=I, lora=lora)
    ops.check_device()
    return idx, tw, st.plan, out, dx, dw


def test_c2_full_shape_nf4_forward_dx_lora():
    """c2 exactly as bench.py times it: 32768 tokens, NF4, forward + dX + rank-16 LoRA on w2."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I, r = 32768, 2048, 32, 2, 1408, 16
    x, logits, raw, ws = _workload(T, H, E, I, "nf4", 1234, dev)
    gen = torch.Generator(device=dev).manual_seed(99)
    la = (torch.randn(E, r, I, device=dev, generator=gen) * (1.0 / I ** 0.5)).to(torch.bfloat16)
    lb = (torch.randn(E, H, r, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
    g_out = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16)
    lora = ops.DownLoRA(la, lb, 16.0 / r)
    idx, tw, plan, out, dx, dw = _run_layer(ops, x, logits, ws, k, E, I, g_out, lora)
    gi, _ = _check_routing_and_plan(ops, logits, idx, tw, plan, k, E)
    # the GPU quantiser against the oracle's on one expert of w1 at this shape (bit-exact buffers)
    q = oq.nf4_quantize_2d(raw[0][5].float().cpu().numpy())
    assert np.array_equal(ws[0].packed[5].cpu().numpy().reshape(-1), q["packed"].reshape(-1))
    assert np.array_equal(ws[0].absmax[5].cpu().numpy(), q["absmax"])
    assert np.array_equal(ws[0].nested_absmax[5].cpu().numpy(), q["nested_absmax"])
    tokens = np.sort(np.random.default_rng(0).choice(T, 256, replace=False))
    lo = {"a": _np(la), "b": _np(lb), "scale": 16.0 / r}
    ref, rdx, rdw = _subset_oracle("nf4", ws, oq.bf16_round(_np(x)), gi, tw.cpu().numpy(), _np(g_out), tokens, lo)
    assert om.rel_max_err(_np(out)[tokens], ref) < TOL
    assert om.rel_max_err(_np(dx)[tokens], rdx) < TOL_DX
    assert om.rel_max_err(_np(dw)[tokens], rdw) < TOL_DX


@pytest.mark.parametrize("rotated", [False, True], ids=["g0", "hadamard"])
def test_c3_full_shape_int8_zipf_small_segments(rotated):
    """c3: 8192 tokens, INT8, H=3072, E=64, k=4, Zipf(1.2) load with dozens of
    segments under 64 rows (the HBM-bound weight-streaming tail); plain
    per-channel INT8 and the reference's default block-Hadamard format
    (g = 256 on both input dimensions)."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 8192, 3072, 64, 4, 1024
    x, logits, raw, ws = _workload(T, H, E, I, "int8", 1234, dev, zipf=1.2, rotated=rotated)
    if rotated:
        assert [w.group_size for w in ws] == [256, 256, 256]
    g_out = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).to(torch.bfloat16)
    idx, tw, plan, out, dx, dw = _run_layer(ops, x, logits, ws, k, E, I, g_out)
    gi, rplan = _check_routing_and_plan(ops, logits, idx, tw, plan, k, E)
    counts = rplan["counts"]
    assert counts.max() > 0.2 * T * k and (counts < 64).sum() >= 8, counts  # the skew the config asks for
    rng = np.random.default_rng(1)
    # the subset covers the small segments: tokens routed to the rarest experts, plus random ones
    rare = np.argsort(counts)[:12]
    pick = np.concatenate([np.nonzero(np.isin(gi, rare).any(axis=1))[0][:96], rng.choice(T, 160, replace=False)])
    tokens = np.unique(pick)
    ref, rdx, rdw = _subset_oracle("int8", ws, oq.bf16_round(_np(x)), gi, tw.cpu().numpy(), _np(g_out), tokens)
    assert om.rel_max_err(_np(out)[tokens], ref) < TOL
    assert om.rel_max_err(_np(dx)[tokens], rdx) < TOL_DX
    assert om.rel_max_err(_np(dw)[tokens], rdw) < TOL_DX


def test_c4_layer_shape_nf4_at_the_largest_reduction():
    """c4's layer: H=4096 (the quantised GEMMs' largest reduction, which fills
    the absmax prefetch buffer exactly), E=128, k=8, I=1536, NF4, on 4096
    tokens (32768 routed rows; the bench runs 65536 tokens over the stack)."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 4096, 4096, 128, 8, 1536
    x, logits, raw, ws = _workload(T, H, E, I, "nf4", 4321, dev)
    g_out = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(8)).to(torch.bfloat16)
    idx, tw, plan, out, dx, dw = _run_layer(ops, x, logits, ws, k, E, I, g_out)
    gi, _ = _check_routing_and_plan(ops, logits, idx, tw, plan, k, E)
    tokens = np.sort(np.random.default_rng(2).choice(T, 8, replace=False))
    ref, rdx, rdw = _subset_oracle("nf4", ws, oq.bf16_round(_np(x)), gi, tw.cpu().numpy(), _np(g_out), tokens)
    assert om.rel_max_err(_np(out)[tokens], ref) < TOL
    assert om.rel_max_err(_np(dx)[tokens], rdx) < TOL_DX
    assert om.rel_max_err(_np(dw)[tokens], rdw) < TOL_DX


def test_c4_checksum_over_every_token():
    """Size-independent check over all 4096 tokens of the c4 layer: the combine
    is linear in the routing weights, so doubling every weight doubles the
    output exactly (a power-of-two scale commutes with every fp32 rounding),
    and with all weights zero the output is exactly zero."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 4096, 4096, 128, 8, 1536
    x, logits, raw, ws = _workload(T, H, E, I, "nf4", 4321, dev)
    idx, tw = ops.route_topk(logits, k)
    out = ops.moe_forward(x, idx, tw, *ws, num_experts=E, inter=I, out_dtype=torch.float32)
    out2 = ops.moe_forward(x, idx, tw * 2, *ws, num_experts=E, inter=I, out_dtype=torch.float32)
    out0 = ops.moe_forward(x, idx, tw * 0, *ws, num_experts=E, inter=I, out_dtype=torch.float32)
    ops.check_device()
    assert torch.equal(out2, out * 2)
    assert not out0.any()
    assert torch.isfinite(out).all() and out.abs().max() > 0
