"""The drop-in layer on the GPU: the reference-compatible module, the
``execute_direct`` backend and autograd, checked against the oracle."""

import os
import types

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


def _np(t):
    return t.detach().float().cpu().numpy()


def _nf4_dense_from_module(m, key):
    E, out_f, in_f = m._nf4_shapes[key]
    g = {"nf4": _np(getattr(m, f"{key}_nf4")).astype(np.uint8).reshape(E, -1),
         "absmax": getattr(m, f"{key}_nf4_absmax").cpu().numpy(),
         "nabsmax": getattr(m, f"{key}_nf4_nabsmax").cpu().numpy(),
         "offset": getattr(m, f"{key}_nf4_offset").cpu().numpy(),
         "code": getattr(m, f"{key}_nf4_code").cpu().numpy(),
         "ncode": getattr(m, f"{key}_nf4_ncode").cpu().numpy(),
         "shape": (E, out_f, in_f), "blocksize": 64, "nested_blocksize": 256}
    g["nf4"] = getattr(m, f"{key}_nf4").cpu().numpy().reshape(E, -1)
    return oq.nf4_dequantize_grouped(g)


@pytest.mark.parametrize("token_dtype", [torch.bfloat16, torch.float32])
def test_module_nf4_forward_and_autograd(token_dtype):
    dev = _dev()
    from mirai_b200.experts import B200GroupedExperts
    T, H, E, k, I = 384, 256, 8, 2, 512
    torch.manual_seed(0)
    m = B200GroupedExperts.from_empty(num_experts=E, quant_format="nf4")
    raw = {"w1": torch.randn(E, I, H) * 0.05, "w3": torch.randn(E, I, H) * 0.05, "w2": torch.randn(E, H, I) * 0.05}
    for key, w in raw.items():
        m.load_dense_weight(key, w.to(dev))
    dense = [_nf4_dense_from_module(m, key) for key in ("w1", "w3", "w2")]
    x = torch.randn(T, H).to(torch.bfloat16).to(token_dtype)
    logits = torch.randn(T, E) * 1.5
    sc, idx = torch.topk(torch.softmax(logits, -1), k)
    sc = (sc / sc.sum(-1, keepdim=True)).to(token_dtype)
    xt = x.to(dev).requires_grad_(True)
    st = sc.to(dev).requires_grad_(True)
    out = m.run_direct_routed(xt, st, idx.to(dev))
    assert out.dtype == token_dtype
    g = torch.randn(T, H).to(torch.bfloat16)
    out.backward(g.to(dev).to(token_dtype))
    xn, sn = _np(x), _np(sc)
    ref = om.moe_forward(xn, idx.numpy(), sn, *dense, bf16=True)
    rdx, rdw = om.moe_backward_dx(xn, idx.numpy(), sn, *dense, _np(g), bf16=True)
    assert om.rel_max_err(_np(out), ref) < TOL
    assert om.rel_max_err(_np(xt.grad), rdx) < 3e-2
    assert om.rel_max_err(_np(st.grad), rdw) < 3e-2


def test_backend_reads_reference_style_buffers_in_place():
    """execute_direct on an object laid out like the reference's CompressedGroupedExperts."""
    dev = _dev()
    from mirai_b200 import ops
    from mirai_b200.backend import B200MoEKernelBackend
    T, H, E, k, I = 256, 256, 4, 2, 256
    rng = np.random.default_rng(1)
    ref_like = types.SimpleNamespace(_quant_format="nf4", num_experts=E, _nf4_shapes={}, expert_lora={},
                                     _nf4_meta=types.SimpleNamespace(blocksize=64, nested_blocksize=256))
    dense = []
    for key, shape in (("w1", (E, I, H)), ("w3", (E, I, H)), ("w2", (E, H, I))):
        gq = oq.nf4_quantize_grouped((rng.standard_normal(shape) * 0.05).astype(np.float32))
        dense.append(oq.nf4_dequantize_grouped(gq))
        setattr(ref_like, f"{key}_nf4", torch.from_numpy(gq["nf4"]).to(dev))
        setattr(ref_like, f"{key}_nf4_absmax", torch.from_numpy(gq["absmax"]).to(dev))
        setattr(ref_like, f"{key}_nf4_nabsmax", torch.from_numpy(gq["nabsmax"]).to(dev))
        setattr(ref_like, f"{key}_nf4_offset", torch.from_numpy(gq["offset"]).to(dev))
        setattr(ref_like, f"{key}_nf4_code", torch.from_numpy(gq["code"]).to(dev))
        setattr(ref_like, f"{key}_nf4_ncode", torch.from_numpy(gq["ncode"]).to(dev))
        ref_like._nf4_shapes[key] = shape
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    idx, w = om.route_topk(logits, k)
    backend = B200MoEKernelBackend()
    out = backend.execute_direct(ref_like, torch.from_numpy(x).to(torch.bfloat16).to(dev),
                                 torch.from_numpy(w).to(dev), torch.from_numpy(idx).to(dev))
    ops.check_device()
    assert out is not None
    ref = om.moe_forward(x, idx, w, *dense, bf16=True)
    assert om.rel_max_err(_np(out), ref) < TOL
    # the binding is cached and re-used while the buffers stay put
    assert backend.bind(ref_like) is backend.bind(ref_like)


def test_module_with_lora_trains_adapter():
    dev = _dev()
    from mirai_b200.experts import B200GroupedExperts
    T, H, E, k, I, r = 256, 256, 4, 2, 256, 8
    torch.manual_seed(3)
    m = B200GroupedExperts.from_empty(num_experts=E, quant_format="bf16")
    ws = {"w1": torch.randn(E, I, H) * 0.05, "w3": torch.randn(E, I, H) * 0.05, "w2": torch.randn(E, H, I) * 0.05}
    for key, w in ws.items():
        m.load_dense_weight(key, w.to(dev))
    m.attach_expert_lora(tensor_name="w2", rank=r, alpha=float(r))
    m = m.to(dev)
    with torch.no_grad():
        m.expert_lora["w2"].lora_b.add_(0.02 * torch.randn_like(m.expert_lora["w2"].lora_b))
    x = torch.randn(T, H, device=dev).to(torch.bfloat16).requires_grad_(True)
    idx = torch.randint(0, E, (T, k), device=dev)
    sc = torch.rand(T, k, device=dev) + 0.1
    out = m.run_direct_routed(x, sc, idx)
    out.float().pow(2).mean().backward()
    ad = m.expert_lora["w2"]
    assert ad.lora_a.grad is not None and ad.lora_b.grad is not None
    assert float(ad.lora_a.grad.norm()) > 0 and float(ad.lora_b.grad.norm()) > 0
    assert float(x.grad.norm()) > 0


def test_lora_operands_follow_optimizer_steps():
    """The padded adapter operands are built once per value of the factors:
    after each optimizer step the module's outputs and gradients equal those
    of freshly made factor tensors with the same values."""
    dev = _dev()
    from mirai_b200.experts import B200GroupedExperts, down_lora_of, run_routed
    T, H, E, k, I, r = 384, 256, 4, 2, 256, 16
    torch.manual_seed(5)
    m = B200GroupedExperts.from_empty(num_experts=E, quant_format="bf16")
    for key, shp in (("w1", (E, I, H)), ("w3", (E, I, H)), ("w2", (E, H, I))):
        m.load_dense_weight(key, (torch.randn(*shp) * 0.05).to(dev))
    m.attach_expert_lora(tensor_name="w2", rank=r, alpha=float(r))
    m = m.to(dev)
    ad = m.expert_lora["w2"]
    opt = torch.optim.SGD(ad.parameters(), lr=2.0)
    idx = torch.randint(0, E, (T, k), device=dev)
    sc = torch.rand(T, k, device=dev) + 0.1
    for _ in range(3):
        x = torch.randn(T, H, device=dev).to(torch.bfloat16)
        xa = x.clone().requires_grad_(True)
        out = m.run_direct_routed(xa, sc, idx)
        out.float().pow(2).mean().backward()
        a, b, scale = down_lora_of(m)
        fa = a.detach().clone().requires_grad_(True)
        fb = b.detach().clone().requires_grad_(True)
        xb = x.clone().requires_grad_(True)
        ref = run_routed(m.bound_weights(), xb, sc, idx, lora=(fa, fb, scale))
        ref.float().pow(2).mean().backward()
        assert torch.equal(out, ref)
        assert torch.equal(xa.grad, xb.grad)
        assert torch.equal(ad.lora_a.grad, fa.grad) and torch.equal(ad.lora_b.grad, fb.grad)
        opt.step()
        opt.zero_grad()


@pytest.mark.parametrize("name", ["routed_int8_bf16", "routed_int8_fp32", "routed_int8_g16_fp32"])
def test_module_int8_against_reference_goldens(golden, name):
    """The reference's own INT8 routed execution (run_direct_routed under
    chunked_dequant, forward and autograd; fixtures recorded from the
    reference) against this module loaded from the same INT8 buffers: plain
    per-channel INT8 with bf16 and fp32 tokens, and the block-Hadamard g=16
    format.  The fp32 references are held to the bf16 tolerance (the kernels
    compute in bf16 with fp32 accumulation)."""
    dev = _dev()
    from mirai_b200.experts import B200GroupedExperts
    g = golden(name)

    def act(key):
        v = g[key]
        return torch.from_numpy(oq.bf16_bits_to_f32(v) if v.dtype == np.uint16 else v.astype(np.float32))

    tdtype = torch.bfloat16 if bool(g["bf16"]) else torch.float32
    E = g["w1_int8"].shape[0]
    m = B200GroupedExperts.from_empty(num_experts=E, quant_format="int8")
    for key in ("w1", "w2", "w3"):
        m.load_quantized_weight(key, weight_int8=torch.from_numpy(g[f"{key}_int8"]).to(dev),
                                weight_scale=torch.from_numpy(g[f"{key}_scale"]).to(dev),
                                group_size=int(g["group_size"]))
    x = act("tokens").to(tdtype).to(dev).requires_grad_(True)
    sc = act("top_scores").to(tdtype).to(dev).requires_grad_(True)
    out = m.run_direct_routed(x, sc, torch.from_numpy(g["top_indices"]).to(dev))
    out.backward(act("grad").to(tdtype).to(dev))
    assert out.dtype == tdtype
    assert om.rel_max_err(_np(out), act("out").numpy()) < TOL
    assert om.rel_max_err(_np(x.grad), act("grad_tokens").numpy()) < 3e-2
    assert om.rel_max_err(_np(sc.grad), act("grad_scores").numpy().reshape(sc.shape)) < 3e-2


def _block_from_golden(g, dev, chunk=0):
    from mirai_b200.block import B200SparseMoeBlock, TokenChunkPolicy
    bits = lambda key: torch.from_numpy(oq.bf16_bits_to_f32(g[key])).to(torch.bfloat16).to(dev)
    state = {"router.weight": torch.from_numpy(g["router_weight"]).to(dev),
             "router.e_score_correction_bias": torch.from_numpy(g["correction_bias"]).to(dev)}
    for key in ("w1", "w2", "w3"):
        state[f"experts.{key}"] = bits(f"experts_{key}")
    for name in ("gate_proj", "up_proj", "down_proj"):
        state[f"shared_experts.{name}.weight"] = bits(f"shared_{name}")
    return B200SparseMoeBlock.from_state(state, top_k=int(g["top_k"]), score_func="sigmoid", norm_topk_prob=True,
                                         route_scale=float(g["route_scale"]),
                                         token_chunk_policy=TokenChunkPolicy(chunk) if chunk else None)


@pytest.mark.parametrize("chunk", [0, 48])
def test_lingbot_block_against_the_reference_block(golden, chunk):
    """The reference's own LingBotVideoSparseMoeBlock (fixture recorded from it:
    sigmoid router with correction bias, top-2 renormalised, route_scale 2.5,
    8 bf16 experts, a shared expert; built-in routed path) against this block
    on the same tensors: routed experts through B200MoEKernelBackend, shared
    expert on the one-expert GEMMs, router selection in the router kernel.
    Training forward + backward, without and with 48-token chunks
    (MoETokenChunkPolicy, checkpointed), and an eval forward with a padding mask."""
    dev = _dev()
    from mirai_b200 import ops
    from mirai_b200.block import route
    g = golden("lingbot_block")
    blk = _block_from_golden(g, dev, chunk)
    x0 = torch.from_numpy(oq.bf16_bits_to_f32(g["x"])).to(torch.bfloat16).to(dev)
    H = x0.shape[-1]
    with torch.no_grad():
        idx, sc = route(x0.reshape(-1, H), blk.router_weight, top_k=2, score_func="sigmoid",
                        correction_bias=blk.e_score_correction_bias, route_scale=2.5)
    ours_i, ours_w = om.canonical_slots(idx.cpu().numpy(), sc.float().cpu().numpy())
    ref_i, ref_w = om.canonical_slots(g["top_indices"], g["top_scores"])
    np.testing.assert_array_equal(ours_i, ref_i)
    np.testing.assert_allclose(ours_w, ref_w, rtol=1e-2)  # bf16 route weights
    blk.train()
    x = x0.clone().requires_grad_(True)
    out = blk(x)
    out.backward(torch.from_numpy(oq.bf16_bits_to_f32(g["grad"])).to(torch.bfloat16).to(dev))
    ops.check_device()
    tag = "_chunked" if chunk else ""
    assert om.rel_max_err(_np(out), oq.bf16_bits_to_f32(g[f"out{tag}"])) < TOL
    assert om.rel_max_err(_np(x.grad), oq.bf16_bits_to_f32(g[f"grad_x{tag}"])) < 3e-2
    assert blk.router_weight.grad is not None and torch.isfinite(blk.router_weight.grad).all()
    blk.eval()
    with torch.no_grad():
        masked = blk(x0, padding_mask=torch.from_numpy(g["padding_mask"]).to(dev))
    assert om.rel_max_err(_np(masked), oq.bf16_bits_to_f32(g["out_masked"])) < TOL


def test_lingbot_block_chunks_change_nothing():
    """Token chunks split the expert execution, not the routes: the chunked
    block's output and input gradient equal the unchunked block's exactly."""
    dev = _dev()
    import numpy as _n
    g = dict(_n.load(os.path.join(os.path.dirname(__file__), "golden", "lingbot_block.npz")))
    x0 = torch.from_numpy(oq.bf16_bits_to_f32(g["x"])).to(torch.bfloat16).to(dev)
    gr = torch.from_numpy(oq.bf16_bits_to_f32(g["grad"])).to(torch.bfloat16).to(dev)
    res = []
    for chunk in (0, 40):
        blk = _block_from_golden(g, dev, chunk).train()
        x = x0.clone().requires_grad_(True)
        out = blk(x)
        out.backward(gr)
        res.append((out.detach(), x.grad))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])


def test_packed_state_nf4_experts_run_on_the_gpu():
    """NF4 experts restored from a packed-state manifest entry (the reference's
    names and layout) run through the fused kernels and match the oracle's
    dequantise-then-matmul of the same buffers."""
    dev = _dev()
    from mirai_b200.experts import B200GroupedExperts
    rng = np.random.default_rng(4)
    T, H, E, k, I = 300, 256, 6, 2, 384
    shapes = {"w1": (E, I, H), "w3": (E, I, H), "w2": (E, H, I)}
    tensors, names, dense = {}, {}, {}
    for key, shp in shapes.items():
        g = oq.nf4_quantize_grouped((rng.standard_normal(shp) * 0.05).astype(np.float32))
        dense[key] = oq.nf4_dequantize_grouped(g)
        for suffix, arr in (("nf4", g["nf4"]), ("nf4_absmax", g["absmax"]), ("nf4_nabsmax", g["nabsmax"]),
                            ("nf4_offset", g["offset"]), ("nf4_code", g["code"]), ("nf4_ncode", g["ncode"])):
            names[f"{key}_{suffix}"] = f"layers.2.ffn.experts.{key}_{suffix}"
            tensors[names[f"{key}_{suffix}"]] = torch.from_numpy(np.ascontiguousarray(arr)).to(dev)
    spec = {"kind": "grouped_experts", "quant_format": "nf4", "num_experts": E, "shapes": shapes,
            "group_sizes": {}, "tensors": names, "nf4_meta": {"blocksize": 64, "nested_blocksize": 256}}
    m = B200GroupedExperts.from_packed_state(spec, tensors)
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    ridx, rw = om.route_topk(logits, k)
    out = m.run_direct_routed(torch.from_numpy(x).to(torch.bfloat16).to(dev), torch.from_numpy(rw).to(dev),
                              torch.from_numpy(ridx).to(dev))
    ref = om.moe_forward(x, ridx, rw, dense["w1"], dense["w3"], dense["w2"], bf16=True)
    assert om.rel_max_err(_np(out), ref) < TOL
