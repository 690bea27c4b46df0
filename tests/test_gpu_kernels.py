"""Parity of the sm_100a kernels (called through the C ABI) against the CPU oracle.

Integer outputs (routing index sets, dispatch plan, permutation) must be
bit-exact; floating outputs are held to the north-star tolerance
max|a - r| / max|r| <= 2e-2 (3e-2 for dX), computed against the oracle's
restatement of the reference's dequantise-then-matmul path.
"""

import numpy as np
import pytest
import torch

from oracle import moe as om
from oracle import quant as oq

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mirai_b200.build import build
    build()
    return torch.device("cuda:0")


def _bf16(t_np):
    return torch.from_numpy(np.ascontiguousarray(t_np)).to(torch.bfloat16)


def _f32(t):
    return t.detach().float().cpu().numpy()


def _check(ops):
    ops.check_device()


# ----------------------------------------------------------------------------- a1

@pytest.mark.parametrize("E,k", [(8, 2), (32, 2), (64, 4), (128, 8), (200, 3), (1000, 16)])
@pytest.mark.parametrize("mode", ["softmax", "sigmoid_bias"])
def test_route_topk_matches_oracle(E, k, mode):
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(E * 7 + k)
    T = 777
    logits = (rng.standard_normal((T, E)) * 1.3).astype(np.float32)
    logits[5, :] = 0.25  # all-equal row: ties resolve to the lowest expert ids
    if mode == "softmax":
        kw = dict(score_func="softmax", norm="clamp")
        okw = dict(score_func="softmax", norm="clamp")
    else:
        bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
        kw = dict(score_func="sigmoid", choice_bias=torch.from_numpy(bias).to(dev), norm="eps", route_scale=2.5)
        okw = dict(score_func="sigmoid", bias=bias, norm="eps", route_scale=2.5)
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k, **kw)
    _check(ops)
    ridx, rw = om.route_topk(logits, k, **okw)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)  # same canonical slot order
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", ["router_e8_k2", "router_e64_k4", "router_e128_k8"])
def test_route_topk_matches_reference_golden(golden, name):
    dev = _dev()
    from mirai_b200 import ops
    g = golden(name)
    idx, w = ops.route_topk(torch.from_numpy(g["logits"]).to(dev), int(g["k"]))
    ci, cw = om.canonical_slots(idx.cpu().numpy(), w.cpu().numpy())
    ri, rw = om.canonical_slots(g["top_indices"], g["top_weights"])
    np.testing.assert_array_equal(ci, ri)
    np.testing.assert_allclose(cw, rw, rtol=1e-5, atol=1e-7)


# ----------------------------------------------------------------------------- a2

def _plan_cases():
    rng = np.random.default_rng(3)
    yield "uniform", rng.integers(0, 32, (5000, 2)), 32
    yield "dups_and_empty", rng.integers(0, 4, (3001, 4)) * 3, 16
    yield "single_expert", np.zeros((2049, 1), np.int64), 1
    zipf = np.minimum(rng.zipf(1.2, (9000, 4)) - 1, 63)
    yield "zipf", zipf, 64
    yield "e1000", rng.integers(0, 1000, (4000, 8)), 1000
    yield "tiny", np.array([[1, 0]]), 3


@pytest.mark.parametrize("case", list(_plan_cases()), ids=lambda c: c[0])
def test_dispatch_plan_bit_exact(case):
    dev = _dev()
    from mirai_b200 import ops
    _, idx, E = case
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    plan = ops.dispatch_plan(torch.from_numpy(idx).to(dev), E)
    _check(ops)
    ref = om.dispatch_plan(idx, E)
    for f in ("counts", "starts", "offsets", "sort_positions", "sorted_token_indices", "inverse_order"):
        np.testing.assert_array_equal(getattr(plan, f).cpu().numpy(), ref[f], err_msg=f)


@pytest.mark.parametrize("name", ["plan_uniform", "plan_dups_empty", "plan_single", "plan_skew"])
def test_dispatch_plan_matches_reference_golden(golden, name):
    dev = _dev()
    from mirai_b200 import ops
    g = golden(name)
    plan = ops.dispatch_plan(torch.from_numpy(g["top_indices"]).to(dev), int(g["num_experts"]))
    for f in ("counts", "starts", "offsets", "sort_positions", "sorted_token_indices", "inverse_order"):
        np.testing.assert_array_equal(getattr(plan, f).cpu().numpy(), g[f], err_msg=f)


def test_dispatch_plan_rejects_bad_expert_ids_on_device():
    dev = _dev()
    from mirai_b200 import ops
    idx = torch.tensor([[0, 1], [2, 7]], device=dev)  # 7 >= E
    ops.dispatch_plan(idx, 4)
    code, info = ops.device_status()
    assert code == 5 and info == 100


# ----------------------------------------------------------------------------- a3 / a8

def test_permute_and_combine_exact():
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(5)
    T, H, E, k = 301, 264, 16, 4
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    idx = rng.integers(0, E, (T, k))
    plan = ops.dispatch_plan(torch.from_numpy(idx).to(dev), E)
    xs = ops.permute_rows(_bf16(x).to(dev), plan.sorted_token_indices)
    ref_plan = om.dispatch_plan(idx, E)
    np.testing.assert_array_equal(_f32(xs), om.permute(x, ref_plan["sorted_token_indices"]))
    y = oq.bf16_round(rng.standard_normal((T * k, H)).astype(np.float32))
    w = rng.random((T, k)).astype(np.float32)
    out = ops.combine(_bf16(y).to(dev), plan.inverse_order, torch.from_numpy(w).to(dev), out_dtype=torch.float32)
    _check(ops)
    ref = om.combine(y, w, ref_plan, T)
    np.testing.assert_array_equal(_f32(out), ref)  # same fp32 order of additions
    outb = ops.combine(_bf16(y).to(dev), plan.inverse_order, torch.from_numpy(w).to(dev))
    np.testing.assert_array_equal(_f32(outb), oq.bf16_round(ref))


# ----------------------------------------------------------------------------- a6 / a7 bf16

def _segments(rng, E, total, skew=False):
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** 1.2
        p /= p.sum()
        counts = rng.multinomial(total, p)
    else:
        counts = rng.multinomial(total, np.ones(E) / E)
    if E > 1:
        counts[1] = 0  # an empty expert
    return counts


@pytest.mark.parametrize("E,H,I,S,skew", [(4, 256, 256, 700, False), (8, 512, 384, 3000, True),
                                          (3, 256, 128, 130, False), (16, 256, 512, 5000, True),
                                          (1, 768, 128, 64, False)])
def test_gateup_and_down_bf16_match_oracle(E, H, I, S, skew):
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(S)
    counts = _segments(rng, E, S, skew)
    S = int(counts.sum())
    offsets = np.cumsum(counts).astype(np.int32)
    x = oq.bf16_round(rng.standard_normal((S, H)).astype(np.float32))
    w1 = oq.bf16_round((rng.standard_normal((E, I, H)) * 0.05).astype(np.float32))
    w3 = oq.bf16_round((rng.standard_normal((E, I, H)) * 0.05).astype(np.float32))
    w2 = oq.bf16_round((rng.standard_normal((E, H, I)) * 0.05).astype(np.float32))
    off = torch.from_numpy(offsets).to(dev)
    h, gu = ops.gateup_swiglu(_bf16(x).to(dev), off, _bf16(w1).to(dev), _bf16(w3).to(dev), inter=I,
                              save_gate_up=True)
    y = ops.down(h, off, _bf16(w2).to(dev), hidden=H)
    _check(ops)
    ry, inter = om.expert_ffn_forward(x, offsets, w1, w3, w2, bf16=True, keep=True)
    assert om.rel_max_err(_f32(gu[:, :I]), inter["gate"]) < TOL
    assert om.rel_max_err(_f32(gu[:, I:]), inter["up"]) < TOL
    assert om.rel_max_err(_f32(h), inter["h"]) < TOL
    # the down GEMM checked on its own input
    ry2 = om.expert_ffn_forward(x, offsets, w1, w3, w2, bf16=True)
    assert om.rel_max_err(_f32(y), ry2) < TOL
    hy = _f32(h)
    ref_down = np.zeros((S, H), np.float32)
    start = 0
    for e in range(E):
        end = offsets[e]
        ref_down[start:end] = hy[start:end] @ w2[e].T
        start = end
    assert om.rel_max_err(_f32(y), ref_down) < 1e-2


def test_moe_forward_bf16_end_to_end():
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(11)
    T, H, E, k, I = 1024, 256, 8, 2, 512
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (x @ (rng.standard_normal((E, H)) * 0.02).T).astype(np.float32)
    w1 = oq.bf16_round((rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    w3 = oq.bf16_round((rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    w2 = oq.bf16_round((rng.standard_normal((E, H, I)) * 0.02).astype(np.float32))
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out = ops.moe_forward(_bf16(x).to(dev), idx, w, _bf16(w1).to(dev), _bf16(w3).to(dev), _bf16(w2).to(dev),
                          num_experts=E, inter=I)
    _check(ops)
    ridx, rw = om.route_topk(logits, k)
    ref = om.moe_forward(x, ridx, rw, w1, w3, w2, bf16=True)
    assert om.rel_max_err(_f32(out), ref) < TOL


# ----------------------------------------------------------------------------- a4 / a5: fused NF4 / INT8 dequant

def nf4_to_device(g, dev):
    from mirai_b200 import ops
    return ops.NF4Tensor(torch.from_numpy(g["nf4"]).to(dev), torch.from_numpy(g["absmax"]).to(dev),
                         torch.from_numpy(g["nabsmax"]).to(dev), torch.from_numpy(g["offset"]).to(dev),
                         torch.from_numpy(g["code"]).to(dev), torch.from_numpy(g["ncode"]).to(dev), g["shape"])


def int8_to_device(q, s, dev):
    from mirai_b200 import ops
    return ops.Int8Tensor(torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev))


@pytest.mark.parametrize("fmt", ["nf4", "int8"])
@pytest.mark.parametrize("E,H,I,S,skew", [(4, 256, 256, 700, False), (8, 512, 384, 3000, True),
                                          (2, 1024, 1408, 400, False), (3, 3072, 1024, 500, True),
                                          (3, 384, 256, 400, False)])
def test_quantized_gemms_match_dequant_then_matmul(fmt, E, H, I, S, skew):
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(S + len(fmt))
    counts = _segments(rng, E, S, skew)
    S = int(counts.sum())
    offsets = np.cumsum(counts).astype(np.int32)
    x = oq.bf16_round(rng.standard_normal((S, H)).astype(np.float32))
    raw = [(rng.standard_normal(shape) * 0.05).astype(np.float32) for shape in ((E, I, H), (E, I, H), (E, H, I))]
    if fmt == "nf4":
        gs = [oq.nf4_quantize_grouped(w) for w in raw]
        dense = [oq.nf4_dequantize_grouped(g) for g in gs]
        dw = [nf4_to_device(g, dev) for g in gs]
    else:
        qs = [oq.int8_quantize(w, 0) for w in raw]
        dense = [oq.bf16_round(oq.int8_dequantize(q, s, 0)) for q, s, _ in qs]
        dw = [int8_to_device(q, s, dev) for q, s, _ in qs]
    off = torch.from_numpy(offsets).to(dev)
    h, gu = ops.gateup_swiglu(_bf16(x).to(dev), off, dw[0], dw[1], inter=I, save_gate_up=True)
    y = ops.down(h, off, dw[2], hidden=H)
    _check(ops)
    _, inter = om.expert_ffn_forward(x, offsets, dense[0], dense[1], dense[2], bf16=True, keep=True)
    assert om.rel_max_err(_f32(gu[:, :I]), inter["gate"]) < 1e-2
    assert om.rel_max_err(_f32(gu[:, I:]), inter["up"]) < 1e-2
    assert om.rel_max_err(_f32(h), inter["h"]) < TOL
    hy = _f32(h)
    ref_down = np.zeros((S, H), np.float32)
    start = 0
    for e in range(E):
        end = offsets[e]
        ref_down[start:end] = hy[start:end] @ dense[2][e].T
        start = end
    assert om.rel_max_err(_f32(y), ref_down) < 1e-2


def test_nf4_moe_forward_end_to_end_config0_shape():
    """Config-0 shape (T=512, H=256, E=8, k=2, I=512) with NF4 experts."""
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(0)
    T, H, E, k, I = 512, 256, 8, 2, 512
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (x @ (rng.standard_normal((E, H)) * 0.02).T).astype(np.float32)
    raw = [(rng.standard_normal(shape) * 0.02).astype(np.float32) for shape in ((E, I, H), (E, I, H), (E, H, I))]
    gs = [oq.nf4_quantize_grouped(w) for w in raw]
    dense = [oq.nf4_dequantize_grouped(g) for g in gs]
    dw = [nf4_to_device(g, dev) for g in gs]
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out = ops.moe_forward(_bf16(x).to(dev), idx, w, dw[0], dw[1], dw[2], num_experts=E, inter=I)
    _check(ops)
    ridx, rw = om.route_topk(logits, k)
    ref = om.moe_forward(x, ridx, rw, dense[0], dense[1], dense[2], bf16=True)
    assert om.rel_max_err(_f32(out), ref) < TOL


# ----------------------------------------------------------------------------- weight ingest

@pytest.mark.parametrize("E,out_f,in_f", [(2, 128, 256), (3, 256, 1408), (1, 64, 64)])
def test_nf4_quantizer_matches_oracle(E, out_f, in_f):
    dev = _dev()
    from mirai_b200 import ops, tables
    rng = np.random.default_rng(out_f + in_f)
    w = oq.bf16_round((rng.standard_normal((E, out_f, in_f)) * 0.05).astype(np.float32))
    w[0, 3, :64] = 0.0  # an all-zero block
    got = ops.nf4_quantize(_bf16(w).to(dev), tables.nf4_code(dev), tables.dynamic_map(dev))
    _check(ops)
    ref = oq.nf4_quantize_grouped(w)
    np.testing.assert_array_equal(got.packed.cpu().numpy().reshape(E, -1), ref["nf4"].reshape(E, -1))
    np.testing.assert_array_equal(got.absmax.cpu().numpy(), ref["absmax"])
    np.testing.assert_array_equal(got.nested_absmax.cpu().numpy(), ref["nabsmax"])
    np.testing.assert_array_equal(got.offset.cpu().numpy(), ref["offset"])


@pytest.mark.parametrize("E,out_f,in_f", [(2, 128, 256), (3, 1408, 256), (1, 64, 64), (5, 192, 320)])
def test_nf4_dequantize_matches_oracle(E, out_f, in_f):
    """The standalone NF4 decode (the staging pass) equals the reference rule
    bf16(code[nibble] * (ncode[q] * nested_absmax + offset)) bit for bit."""
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(E * out_f + in_f)
    g = oq.nf4_quantize_grouped((rng.standard_normal((E, out_f, in_f)) * 0.05).astype(np.float32),
                                nested_blocksize=256 if out_f * in_f >= 64 * 256 else 16)
    w = ops.NF4Tensor(torch.from_numpy(g["nf4"]).to(dev), torch.from_numpy(g["absmax"]).to(dev),
                      torch.from_numpy(g["nabsmax"]).to(dev), torch.from_numpy(g["offset"]).to(dev),
                      torch.from_numpy(g["code"]).to(dev), torch.from_numpy(g["ncode"]).to(dev), g["shape"],
                      nested_blocksize=g["nested_blocksize"])
    got = ops.nf4_dequantize(w)
    _check(ops)
    assert got.dtype == torch.bfloat16 and tuple(got.shape) == (E, out_f, in_f)
    assert np.array_equal(_f32(got), oq.nf4_dequantize_grouped(g))


@pytest.mark.parametrize("lora_rank", [0, 16])
def test_nf4_staged_train_step_equals_in_loop_decode(lora_rank):
    """A training pass on bf16 copies of the NF4 keys (decoded once) gives the
    same bits as the GEMMs that decode inside their main loops: the decoded
    values, the tiles and the accumulation order are the same."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 2048, 512, 4, 2, 384
    rng = np.random.default_rng(21)
    _, dw = _weights("nf4", rng, E, H, I, dev)
    x = _bf16(rng.standard_normal((T, H)).astype(np.float32)).to(dev)
    g = _bf16(rng.standard_normal((T, H)).astype(np.float32)).to(dev)
    idx, w = ops.route_topk(torch.from_numpy((rng.standard_normal((T, E)) * 1.5).astype(np.float32)).to(dev), k)
    res = {}
    for mode in ("never", "always"):
        ops.set_nf4_staging(mode)
        try:
            lora = None
            if lora_rank:
                gen = torch.Generator(device=dev).manual_seed(3)
                lora = ops.DownLoRA(torch.randn(E, lora_rank, I, device=dev, generator=gen) * 0.05,
                                    torch.randn(E, H, lora_rank, device=dev, generator=gen) * 0.05, 2.0,
                                    compute_grads=True)
            out, st = ops.moe_forward_train(x, idx, w, *dw, num_experts=E, inter=I, lora=lora)
            dx, dwt = ops.moe_backward_dx(g, st, *dw, inter=I, lora=lora)
            res[mode] = (out, dx, dwt) + ((lora.grad_a, lora.grad_b) if lora else ())
        finally:
            ops.set_nf4_staging("auto")
    _check(ops)
    for a, b in zip(res["never"], res["always"]):
        assert torch.equal(a, b)


def test_nf4_staged_forward_equals_in_loop_decode_at_c4_width():
    """The forward on bf16 copies of NF4 keys (what "auto" runs from 4096 rows
    per expert) gives the in-loop decode's bits at c4's H=4096, I=1536."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 4096, 4096, 4, 4, 1536
    rng = np.random.default_rng(31)
    _, dw = _weights("nf4", rng, E, H, I, dev, std=0.02)
    x = _bf16(rng.standard_normal((T, H)).astype(np.float32)).to(dev)
    idx, w = ops.route_topk(torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(dev), k)
    res = {}
    for mode in ("never", "auto"):  # 4096 * 4 / 4 = 4096 rows per expert: "auto" stages
        ops.set_nf4_staging(mode)
        try:
            res[mode] = ops.moe_forward(x, idx, w, *dw, num_experts=E, inter=I)
        finally:
            ops.set_nf4_staging("auto")
    _check(ops)
    assert torch.equal(res["never"], res["auto"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_int8_quantizer_matches_reference_golden(golden, dtype):
    dev = _dev()
    from mirai_b200 import ops
    g = golden("int8_quant")
    w = torch.from_numpy(g["weight"]).to(dtype)
    got = ops.int8_quantize(w.to(dev))
    _check(ops)
    if dtype == torch.float32:
        np.testing.assert_array_equal(got.q.cpu().numpy(), g["q_g0"])
        np.testing.assert_array_equal(got.scale.cpu().numpy(), g["s_g0"])
    else:
        q, s, _ = oq.int8_quantize(w.float().numpy(), 0)
        np.testing.assert_array_equal(got.q.cpu().numpy(), q)
        np.testing.assert_array_equal(got.scale.cpu().numpy(), s)


# ----------------------------------------------------------------------------- a9: dX

def _weights(fmt, rng, E, H, I, dev, std=0.05):
    raw = [(rng.standard_normal(shape) * std).astype(np.float32) for shape in ((E, I, H), (E, I, H), (E, H, I))]
    if fmt == "nf4":
        gs = [oq.nf4_quantize_grouped(w) for w in raw]
        return [oq.nf4_dequantize_grouped(g) for g in gs], [nf4_to_device(g, dev) for g in gs]
    if fmt == "int8":
        qs = [oq.int8_quantize(w, 0) for w in raw]
        return ([oq.bf16_round(oq.int8_dequantize(q, s, 0)) for q, s, _ in qs],
                [int8_to_device(q, s, dev) for q, s, _ in qs])
    dense = [oq.bf16_round(w) for w in raw]
    return dense, [_bf16(w).to(dev) for w in dense]


@pytest.mark.parametrize("fmt", ["bf16", "nf4", "int8"])
@pytest.mark.parametrize("T,H,E,k,I", [(512, 256, 8, 2, 512), (300, 512, 6, 3, 1408), (700, 1024, 16, 4, 384)])
def test_moe_forward_and_dx_match_oracle(fmt, T, H, E, k, I):
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(T + H + I)
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    dense, dw = _weights(fmt, rng, E, H, I, dev)
    g = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, w, *dw, num_experts=E, inter=I)
    dx, dwts = ops.moe_backward_dx(_bf16(g).to(dev), st, *dw, inter=I)
    _check(ops)
    ridx, rw = om.route_topk(logits, k)
    ref = om.moe_forward(x, ridx, rw, *dense, bf16=True)
    rdx, rdw = om.moe_backward_dx(x, ridx, rw, *dense, g, bf16=True)
    assert om.rel_max_err(_f32(out), ref) < TOL
    assert om.rel_max_err(_f32(dx), rdx) < 3e-2
    assert om.rel_max_err(_f32(dwts), rdw) < 3e-2


def test_dx_matches_reference_golden(golden):
    """dX and top-score gradients against the reference's own autograd (bf16 experts)."""
    dev = _dev()
    from mirai_b200 import ops
    g = golden("routed_dense_bf16")
    x = oq.bf16_bits_to_f32(g["tokens"])
    w1, w3, w2 = (oq.bf16_bits_to_f32(g[k]) for k in ("w1", "w3", "w2"))
    scores = oq.bf16_bits_to_f32(g["top_scores"])
    idx = torch.from_numpy(g["top_indices"]).to(dev)
    E, I, H = w1.shape
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, torch.from_numpy(scores).to(dev),
                                    _bf16(w1).to(dev), _bf16(w3).to(dev), _bf16(w2).to(dev), num_experts=E, inter=I)
    dx, dws = ops.moe_backward_dx(_bf16(oq.bf16_bits_to_f32(g["grad"])).to(dev), st, _bf16(w1).to(dev),
                                  _bf16(w3).to(dev), _bf16(w2).to(dev), inter=I)
    _check(ops)
    assert om.rel_max_err(_f32(out), oq.bf16_bits_to_f32(g["out"])) < TOL
    assert om.rel_max_err(_f32(dx), oq.bf16_bits_to_f32(g["grad_tokens"])) < 3e-2
    assert om.rel_max_err(_f32(dws), oq.bf16_bits_to_f32(g["grad_scores"])) < 3e-2


# ----------------------------------------------------------------------------- a10: LoRA on the down projection

@pytest.mark.parametrize("fmt", ["bf16", "nf4"])
@pytest.mark.parametrize("rank", [16, 4])
def test_lora_on_down_forward_and_dx(fmt, rank):
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I = 400, 256, 6, 2, 384
    rng = np.random.default_rng(rank + len(fmt))
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    dense, dw = _weights(fmt, rng, E, H, I, dev)
    la = oq.bf16_round((rng.standard_normal((E, rank, I)) * 0.05).astype(np.float32))
    lb = oq.bf16_round((rng.standard_normal((E, H, rank)) * 0.05).astype(np.float32))
    scale = 16.0 / rank
    lora = ops.DownLoRA(_bf16(la).to(dev), _bf16(lb).to(dev), scale)
    g = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, w, *dw, num_experts=E, inter=I, lora=lora)
    dx, dwts = ops.moe_backward_dx(_bf16(g).to(dev), st, *dw, inter=I, lora=lora)
    _check(ops)
    ridx, rw = om.route_topk(logits, k)
    ol = {"a": la, "b": lb, "scale": scale}
    ref = om.moe_forward(x, ridx, rw, *dense, bf16=True, lora=ol)
    rdx, rdw = om.moe_backward_dx(x, ridx, rw, *dense, g, bf16=True, lora=ol)
    assert om.rel_max_err(_f32(out), ref) < TOL
    assert om.rel_max_err(_f32(dx), rdx) < 3e-2
    assert om.rel_max_err(_f32(dwts), rdw) < 3e-2
    # the adapter matters: without it the forward differs by far more than the tolerance
    ref0 = om.moe_forward(x, ridx, rw, *dense, bf16=True)
    assert om.rel_max_err(ref0, ref) > 5 * om.rel_max_err(_f32(out), ref)


def test_lora_factor_gradients():
    """dA / dB of the down-projection adapter against the bmm backward formulas."""
    dev = _dev()
    from mirai_b200 import ops
    T, H, E, k, I, r = 300, 256, 4, 2, 256, 8
    rng = np.random.default_rng(17)
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    dense, dw = _weights("bf16", rng, E, H, I, dev)
    la = oq.bf16_round((rng.standard_normal((E, r, I)) * 0.05).astype(np.float32))
    lb = oq.bf16_round((rng.standard_normal((E, H, r)) * 0.05).astype(np.float32))
    scale = 2.0
    g = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    lora = ops.DownLoRA(_bf16(la).to(dev), _bf16(lb).to(dev), scale, compute_grads=True)
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, w, *dw, num_experts=E, inter=I, lora=lora)
    ops.moe_backward_dx(_bf16(g).to(dev), st, *dw, inter=I, lora=lora)
    _check(ops)
    ridx, rw = om.route_topk(logits, k)
    plan = om.dispatch_plan(ridx, E)
    xs = om.permute(x, plan["sorted_token_indices"])
    _, inter = om.expert_ffn_forward(xs, plan["offsets"], *dense, bf16=True,
                                     lora={"a": la, "b": lb, "scale": scale}, keep=True)
    sp = plan["sort_positions"]
    gy = oq.bf16_round(g[sp // k] * rw.reshape(-1)[sp][:, None])
    ga = np.zeros((E, r, I), np.float32)
    gb = np.zeros((E, H, r), np.float32)
    start = 0
    for e in range(E):
        end = plan["offsets"][e]
        h_e, gy_e = inter["h"][start:end], gy[start:end]
        gb[e] = scale * gy_e.T @ (h_e @ la[e].T)
        ga[e] = scale * (gy_e @ lb[e]).T @ h_e
        start = end
    assert om.rel_max_err(lora.grad_a.cpu().numpy(), ga) < 3e-2
    assert om.rel_max_err(lora.grad_b.cpu().numpy(), gb) < 3e-2


@pytest.mark.parametrize("K", [256, 200, 1408])
@pytest.mark.parametrize("rank", [16, 5, 32])
def test_lora_project_and_grad_ragged_segments(K, rank):
    """The tensor-core rank-block kernels on ragged segments: an empty expert, a
    one-row expert, partial 64/128-row blocks and K not a multiple of 128."""
    dev = _dev()
    from mirai_b200 import ops
    counts = [0, 1, 130, 64, 300, 0]
    E, H = len(counts), 192
    offsets = np.cumsum(counts).astype(np.int32)
    S = int(offsets[-1])
    rng = np.random.default_rng(K + rank)
    x = oq.bf16_round(rng.standard_normal((S, K)).astype(np.float32))
    la = oq.bf16_round((rng.standard_normal((E, rank, K)) * 0.1).astype(np.float32))
    lb = oq.bf16_round((rng.standard_normal((E, K, rank)) * 0.1).astype(np.float32))
    g = np.zeros((S, 64), np.float32)
    g[:, :rank] = oq.bf16_round(rng.standard_normal((S, rank)).astype(np.float32))
    scale = 0.75
    lora = ops.DownLoRA(_bf16(la).to(dev), _bf16(lb).to(dev), scale)
    xd, od = _bf16(x).to(dev), torch.from_numpy(offsets).to(dev)
    fwd = ops.lora_project(xd, od, lora, forward=True)
    bwd = ops.lora_project(xd, od, lora, forward=False)
    ga = ops.lora_grad(xd, _bf16(g).to(dev), od, rank, torch.full((E, rank, K), 7.0, device=dev),
                       (rank * K, K, 1))
    gb = ops.lora_grad(xd, _bf16(g).to(dev), od, rank, torch.full((E, K, rank), 7.0, device=dev),
                       (K * rank, 1, rank))
    _check(ops)
    ref_f = np.zeros((S, 64), np.float32)
    ref_b = np.zeros((S, 64), np.float32)
    ref_ga = np.zeros((E, rank, K), np.float64)
    start = 0
    for e in range(E):
        end = int(offsets[e])
        xs = x[start:end].astype(np.float64)
        ref_f[start:end, :rank] = scale * xs @ la[e].T
        ref_b[start:end, :rank] = scale * xs @ lb[e]
        ref_ga[e] = g[start:end, :rank].T.astype(np.float64) @ xs
        start = end
    assert om.rel_max_err(_f32(fwd), oq.bf16_round(ref_f)) < 1e-2
    assert om.rel_max_err(_f32(bwd), oq.bf16_round(ref_b)) < 1e-2
    assert np.all(_f32(fwd)[:, rank:] == 0) and np.all(_f32(bwd)[:, rank:] == 0)
    assert om.rel_max_err(ga.cpu().numpy(), ref_ga) < 1e-4
    assert om.rel_max_err(gb.cpu().numpy(), ref_ga.transpose(0, 2, 1)) < 1e-4
    assert np.all(ga.cpu().numpy()[[0, 5]] == 0)


@pytest.mark.parametrize("fmt", ["nf4", "int8", "bf16"])
@pytest.mark.parametrize("H", [256, 320])
def test_grouped_gemms_on_tile_edge_segments(fmt, H):
    """All four grouped GEMMs on segments around the 256-row tile edges (empty,
    1, 255..257, 511..513 rows), and with H = 320 a last 256-column tile of the
    down GEMM that is three quarters empty (N % 256 == 64)."""
    dev = _dev()
    from mirai_b200 import ops
    counts = np.array([0, 1, 255, 256, 257, 511, 512, 513, 0, 130])
    E, I = len(counts), 384
    offsets = np.cumsum(counts).astype(np.int32)
    S = int(offsets[-1])
    rng = np.random.default_rng(7 + len(fmt))
    x = oq.bf16_round(rng.standard_normal((S, H)).astype(np.float32))
    gy = oq.bf16_round(rng.standard_normal((S, H)).astype(np.float32))
    dense, dw = _weights(fmt, rng, E, H, I, dev)
    off = torch.from_numpy(offsets).to(dev)
    h, gu = ops.gateup_swiglu(_bf16(x).to(dev), off, dw[0], dw[1], inter=I, save_gate_up=True)
    y = ops.down(h, off, dw[2], hidden=H)
    dgu = ops.down_dx(_bf16(gy).to(dev), off, dw[2], gu, inter=I)
    dxs = ops.gateup_dx(dgu, off, dw[0], dw[1], hidden=H)
    _check(ops)
    _, inter = om.expert_ffn_forward(x, offsets, dense[0], dense[1], dense[2], bf16=True, keep=True)
    assert om.rel_max_err(_f32(gu[:, :I]), inter["gate"]) < 1e-2
    assert om.rel_max_err(_f32(gu[:, I:]), inter["up"]) < 1e-2
    assert om.rel_max_err(_f32(h), inter["h"]) < TOL
    hk, guk, dguk = _f32(h), _f32(gu), _f32(dgu)
    ref_y = np.zeros((S, H), np.float32)
    ref_dgu = np.zeros((S, 2 * I), np.float32)
    ref_dx = np.zeros((S, H), np.float32)
    start = 0
    for e in range(E):
        end = int(offsets[e])
        if end > start:
            ref_y[start:end] = hk[start:end] @ dense[2][e].T
            gate, up = guk[start:end, :I], guk[start:end, I:]
            dh = oq.bf16_round(gy[start:end] @ dense[2][e])
            act = oq.bf16_round(om.silu_f32(gate))
            d_act = oq.bf16_round(dh * up)
            ref_dgu[start:end, I:] = dh * act
            ref_dgu[start:end, :I] = om.silu_backward_f32(d_act, gate)
            ref_dx[start:end] = dguk[start:end, :I] @ dense[0][e] + dguk[start:end, I:] @ dense[1][e]
        start = end
    assert om.rel_max_err(_f32(y), ref_y) < TOL
    assert om.rel_max_err(dguk, ref_dgu) < 3e-2
    assert om.rel_max_err(_f32(dxs), ref_dx) < TOL


def test_lora_dx_matches_reference_golden(golden):
    """Forward, dX and top-score gradients with a LoRA adapter on w2 against the
    reference's own autograd (bf16 experts, ActiveExpertLoRA)."""
    dev = _dev()
    from mirai_b200 import ops
    g = golden("routed_dense_bf16_lora")
    x = oq.bf16_bits_to_f32(g["tokens"])
    w1, w3, w2 = (oq.bf16_bits_to_f32(g[k]) for k in ("w1", "w3", "w2"))
    la, lb = oq.bf16_round(g["lora_a"]), oq.bf16_round(g["lora_b"])  # stored as fp32 values
    scores = oq.bf16_bits_to_f32(g["top_scores"])
    idx = torch.from_numpy(g["top_indices"]).to(dev)
    E, I, H = w1.shape
    dw = [_bf16(w).to(dev) for w in (w1, w3, w2)]
    lora = ops.DownLoRA(_bf16(la).to(dev), _bf16(lb).to(dev), float(g["lora_scale"]))
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, torch.from_numpy(scores).to(dev), *dw, num_experts=E,
                                    inter=I, lora=lora)
    dx, dws = ops.moe_backward_dx(_bf16(oq.bf16_bits_to_f32(g["grad"])).to(dev), st, *dw, inter=I, lora=lora)
    _check(ops)
    assert om.rel_max_err(_f32(out), oq.bf16_bits_to_f32(g["out"])) < TOL
    assert om.rel_max_err(_f32(dx), oq.bf16_bits_to_f32(g["grad_tokens"])) < 3e-2
    assert om.rel_max_err(_f32(dws), oq.bf16_bits_to_f32(g["grad_scores"])) < 3e-2


def test_router_nan_rows_select_valid_experts():
    """A row of NaN logits (a diverged activation upstream) must still yield k
    distinct in-range expert ids, so the dispatch plan downstream stays valid;
    NaN entries rank after every number."""
    dev = _dev()
    from mirai_b200 import ops
    E, k = 128, 8
    lg = torch.randn(6, E)
    lg[0] = float("nan")
    lg[1, ::2] = float("nan")
    lg[2] = float("-inf")
    idx, w = ops.route_topk(lg.to(dev), k)
    plan = ops.dispatch_plan(idx, E)
    _check(ops)
    idx = idx.cpu()
    assert int(idx.min()) >= 0 and int(idx.max()) < E
    for row in idx:
        assert len(set(row.tolist())) == k
    assert sorted(idx[0].tolist()) == list(range(k))           # all NaN: lowest ids
    assert all(e % 2 == 1 for e in idx[1].tolist())            # the numbers win over the NaNs
    assert int(plan.counts.sum()) == 6 * k


@pytest.mark.parametrize("fmt", ["nf4", "int8", "bf16"])
def test_source_major_segments_equal_expert_major(fmt):
    """The GEMMs over G x E source-major segments (an expert owner's receive
    buffer) give, row for row, exactly the results of the same rows grouped by
    expert (the expert-parallel layer relies on it for bit-exactness)."""
    dev = _dev()
    from mirai_b200 import ops
    G, E, H, I = 3, 5, 256, 384
    rng = np.random.default_rng(21 + len(fmt))
    counts = rng.integers(0, 300, size=(G, E))
    counts[1, 2] = 0
    counts[2, 4] = 513
    R = int(counts.sum())
    x = torch.randn(R, H).to(torch.bfloat16)
    _, dw = _weights(fmt, rng, E, H, I, dev)
    ends = np.cumsum(counts.reshape(-1)).astype(np.int32)
    starts = np.concatenate([[0], ends[:-1]])
    perm = np.concatenate([np.arange(starts[s * E + e], ends[s * E + e]) for e in range(E) for s in range(G)])
    off_src = torch.from_numpy(ends).to(dev)
    off_exp = torch.from_numpy(np.cumsum(counts.sum(0)).astype(np.int32)).to(dev)
    xd = x.to(dev)
    h_src = ops.gateup_swiglu(xd, off_src, dw[0], dw[1], inter=I, sources=G)
    y_src = ops.down(h_src, off_src, dw[2], hidden=H, sources=G)
    pd = torch.from_numpy(perm).to(dev)
    h_exp = ops.gateup_swiglu(xd[pd], off_exp, dw[0], dw[1], inter=I)
    y_exp = ops.down(h_exp, off_exp, dw[2], hidden=H)
    _check(ops)
    assert torch.equal(h_src[pd], h_exp)
    assert torch.equal(y_src[pd], y_exp)


@pytest.mark.parametrize("fmt", ["nf4", "bf16"])
def test_source_major_lora_equals_expert_major(fmt):
    """The LoRA kernels and the rank-block GEMMs over source-major segments
    (forward rank block, fused down, down dX with the SwiGLU backward, the
    factor gradients) against the same rows grouped by expert: row products
    exactly equal; factor gradients, which sum an expert's rows in 64-row
    blocks that start anew at each source, to fp32 rounding."""
    dev = _dev()
    from mirai_b200 import ops
    G, E, H, I, r = 3, 4, 256, 384, 16
    rng = np.random.default_rng(5 + len(fmt))
    counts = rng.integers(0, 260, size=(G, E))
    counts[0, 1] = 0
    counts[2, 3] = 300
    R = int(counts.sum())
    _, dw = _weights(fmt, rng, E, H, I, dev)
    x = torch.randn(R, H, device=dev).to(torch.bfloat16)
    gy = torch.randn(R, H, device=dev).to(torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(9)
    lora = ops.DownLoRA(torch.randn(E, r, I, device=dev, generator=gen) * 0.05,
                        torch.randn(E, H, r, device=dev, generator=gen) * 0.05, 2.0)
    ends = np.cumsum(counts.reshape(-1)).astype(np.int32)
    starts = np.concatenate([[0], ends[:-1]])
    perm = torch.from_numpy(np.concatenate([np.arange(starts[s * E + e], ends[s * E + e])
                                            for e in range(E) for s in range(G)])).to(dev)
    off_src = torch.from_numpy(ends).to(dev)
    off_exp = torch.from_numpy(np.cumsum(counts.sum(0)).astype(np.int32)).to(dev)

    def run(xx, gg, offs, sources):
        h, gu = ops.gateup_swiglu(xx, offs, dw[0], dw[1], inter=I, sources=sources, save_gate_up=True)
        low = ops.lora_project(h, offs, lora, forward=True, sources=sources)
        y = ops.down(h, offs, dw[2], hidden=H, lora=lora, rank_a=low, sources=sources)
        glow = ops.lora_project(gg, offs, lora, forward=False, sources=sources)
        dgu = ops.down_dx(gg, offs, dw[2], gu, inter=I, lora=lora, rank_a=glow, sources=sources)
        ga = ops.lora_grad(h, glow, offs, r, torch.empty((E, r, I), device=dev), (r * I, I, 1), sources=sources)
        gb = ops.lora_grad(gg, low, offs, r, torch.empty((E, H, r), device=dev), (H * r, 1, r), sources=sources)
        return low, y, glow, dgu, ga, gb

    src = run(x, gy, off_src, G)
    exp = run(x[perm], gy[perm], off_exp, 1)
    _check(ops)
    for a, b in zip(src[:4], exp[:4]):
        assert torch.equal(a[perm], b)
    for a, b in zip(src[4:], exp[4:]):
        assert float((a - b).abs().max() / b.abs().max()) < 1e-5


def test_exchange_wait_gives_up_and_reports_a_timeout():
    """A peer that never signals (a flag nothing sets): the exchange's arrival
    wait gives up after its 2 s limit, records MIRAI_ERR_DEVICE_TIMEOUT with the
    silent peer's slot (site 700 + slot) and returns, so the host learns of it
    and the context stays usable; a flag that has reached the epoch passes at once."""
    import time

    dev = _dev()
    from mirai_b200 import _lib, ops
    ops.device_status()  # start from a clear error word
    flags = torch.zeros(2, dtype=torch.int64, device=dev)
    stream = _lib.c_vp(torch.cuda.current_stream().cuda_stream)
    t0 = time.monotonic()
    _lib.call("mirai_ep_wait", _lib.c_vp(flags.data_ptr()), 2, 0, 1, stream)
    code, info = ops.device_status()
    waited = time.monotonic() - t0
    assert (code, info) == (4, 701)  # MIRAI_ERR_DEVICE_TIMEOUT, slot 1
    assert 1.5 < waited < 30
    idx, _ = ops.route_topk(torch.randn(64, 8, device=dev), 2)  # the context still runs kernels
    ops.check_device()
    assert idx.shape == (64, 2)
    flags[1] = 3
    t0 = time.monotonic()
    _lib.call("mirai_ep_wait", _lib.c_vp(flags.data_ptr()), 2, 0, 2, stream)
    assert ops.device_status() == (0, 0) and time.monotonic() - t0 < 1.0


# ----------------------------------------------------------------------------- a5: rotated INT8

@pytest.mark.parametrize("group", [4, 16, 64, 256, 1024, 4096])
@pytest.mark.parametrize("dtypes", [("bf16", "bf16"), ("f32", "f32"), ("f32", "bf16")])
def test_rotate_rows_matches_the_hadamard_product(group, dtypes):
    """Block-Hadamard rotation of rows (quant.py:150-182 restated in
    oracle.quant.rotate_last_dim) in fp32: within fp32 rounding of the product,
    and exactly its own inverse up to rounding."""
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(group)
    rows, cols = 37, max(group, 64) * 3
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    tin = {"bf16": torch.bfloat16, "f32": torch.float32}[dtypes[0]]
    tout = {"bf16": torch.bfloat16, "f32": torch.float32}[dtypes[1]]
    xt = torch.from_numpy(x).to(dev).to(tin)
    got = ops.rotate_rows(xt, group, out_dtype=tout)
    _check(ops)
    ref = oq.rotate_last_dim(_f32(xt), group, inverse=False)
    tol = 1e-5 if tout == torch.float32 else 8e-3
    assert np.abs(_f32(got) - ref).max() <= tol * np.abs(ref).max()
    back = ops.rotate_rows(got.float(), group, out_dtype=torch.float32)
    assert np.abs(_f32(back) - _f32(xt)).max() <= tol * 4 * np.abs(x).max()


def test_rotate_rows_in_place_and_rejects_bad_groups():
    dev = _dev()
    from mirai_b200 import ops
    from mirai_b200._lib import MiraiError
    x = torch.randn(64, 512, device=dev)
    ref = ops.rotate_rows(x, 64)
    ops.rotate_rows(x, 64, out=x)
    assert torch.equal(x, ref)
    for bad in (8, 32, 3, 0, 8192):
        with pytest.raises(MiraiError):
            ops.rotate_rows(x, bad)


@pytest.mark.parametrize("group", [16, 64, 256])
def test_gpu_rotated_int8_quantiser_matches_the_reference_rule(group):
    """Rotate in fp32, per-row amax/127, round half to even (quant.py:189-235):
    identical codes except, rarely, one step where the rotated value sits on a
    rounding boundary (the fast transform orders its fp32 sums differently)."""
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(group + 1)
    w = (rng.standard_normal((3, 96, 1024)) * 0.02).astype(np.float32)
    t = ops.int8_quantize(torch.from_numpy(w).to(dev), group_size=group)
    _check(ops)
    q, s, g = oq.int8_quantize(w, group)
    assert g == group and t.group_size == group
    gq = t.q.cpu().numpy().astype(np.int32)
    assert np.abs(gq - q).max() <= 1 and (gq != q).mean() < 1e-3
    np.testing.assert_allclose(t.scale.cpu().numpy(), s, rtol=4e-6)  # a few fp32 ulps of the rotated amax


def _rotated_int8_weights(rng, E, H, I, g_in, g_mid, dev):
    from mirai_b200 import ops
    raw = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in ((E, I, H), (E, I, H), (E, H, I))]
    groups = (g_in, g_in, g_mid)
    qs = [oq.int8_quantize(w, g) for w, g in zip(raw, groups)]
    dense = [oq.bf16_round(oq.int8_dequantize(q, s, g)) for q, s, g in qs]
    dw = [ops.Int8Tensor(torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev), group_size=g) for q, s, g in qs]
    return dense, dw


@pytest.mark.parametrize("T,H,E,k,I,lora_rank", [(600, 1024, 8, 2, 1024, 0), (333, 256, 6, 3, 384, 8),
                                                 (512, 3072, 4, 2, 1024, 16)])
def test_rotated_int8_layer_forward_and_dx_match_oracle(T, H, E, k, I, lora_rank):
    """The reference's default INT8 format (g = best of 256/64/16 per input
    dimension), run as rotated activations into the INT8 GEMMs, against the
    oracle's dequantise-then-matmul (weights de-rotated on the host)."""
    dev = _dev()
    from mirai_b200 import ops
    rng = np.random.default_rng(T + I)
    g_in, g_mid = oq.best_group_size(H), oq.best_group_size(I)
    assert g_in and g_mid
    dense, dw = _rotated_int8_weights(rng, E, H, I, g_in, g_mid, dev)
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    g = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    lora, ol = None, None
    if lora_rank:
        la = oq.bf16_round((rng.standard_normal((E, lora_rank, I)) * 0.05).astype(np.float32))
        lb = oq.bf16_round((rng.standard_normal((E, H, lora_rank)) * 0.05).astype(np.float32))
        lora = ops.DownLoRA(_bf16(la).to(dev), _bf16(lb).to(dev), 2.0, compute_grads=True)
        ol = {"a": la, "b": lb, "scale": 2.0}
    idx, w = ops.route_topk(torch.from_numpy(logits).to(dev), k)
    out, st = ops.moe_forward_train(_bf16(x).to(dev), idx, w, *dw, num_experts=E, inter=I, lora=lora)
    dx, dwts = ops.moe_backward_dx(_bf16(g).to(dev), st, *dw, inter=I, lora=lora)
    fwd = ops.moe_forward(_bf16(x).to(dev), idx, w, *dw, num_experts=E, inter=I, lora=lora)
    _check(ops)
    assert torch.equal(fwd, out)
    ridx, rw = om.route_topk(logits, k)
    ref = om.moe_forward(x, ridx, rw, *dense, bf16=True, lora=ol)
    rdx, rdw = om.moe_backward_dx(x, ridx, rw, *dense, g, bf16=True, lora=ol)
    assert om.rel_max_err(_f32(out), ref) < TOL
    assert om.rel_max_err(_f32(dx), rdx) < 3e-2
    assert om.rel_max_err(_f32(dwts), rdw) < 3e-2
