"""Generate the golden fixtures under tests/golden/ by running the reference.

Run from the repository root in a container that has the seruva19/mirai
reference checked out, naming its root in ``MIRAI_REFERENCE``:

    MIRAI_REFERENCE=<path to the mirai checkout> python tests/golden/make_golden.py

It imports the reference's own code on the CPU and records inputs and
outputs of:

* ``TokenChoiceRouter`` (mirai/core/moe/routing/routers.py:208-274);
* ``build_dispatch_plan`` (.../execution/dispatch_preprocess.py:128-179),
  including duplicate routes and empty experts;
* ``permute_routed_tokens`` / ``combine_routed_tokens`` forward and backward
  (.../execution/dispatch_ops.py);
* ``_quantize_weight`` / ``_dequantize_weight`` INT8 with and without the
  block-Hadamard rotation (.../quantization/quant.py:189-260);
* ``CompressedGroupedExperts.run_direct_routed`` (experts.py:1749) with INT8
  experts under ``chunked_dequant`` and with dense bf16 experts bound through
  ``bind_physical_weight_provider`` (experts.py:695-714), forward plus the
  input gradient (and the top-score gradient) through autograd, with and
  without a rank-4 LoRA on the down projection.

The fixtures are small ``.npz`` files; the GPU box never needs the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

REF = os.environ.get("MIRAI_REFERENCE", "")
OUT = Path(__file__).resolve().parent


def _bf16_bits(t):
    import torch
    return t.detach().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def lingbot_block() -> None:
    """``LingBotVideoSparseMoeBlock`` (transformer_lingbot_video.py:1175-2377)
    with a shared expert, sigmoid routing with a correction bias, top-k
    renormalisation and route_scale 2.5, bf16 (router fp32), run by the
    reference's built-in path: a training forward + backward, the same with a
    48-token ``MoETokenChunkPolicy``, and an eval forward with a padding mask."""
    import torch
    from mirai.core.moe.runtime.token_chunking import MoETokenChunkPolicy
    from mirai.vendors.lingbot_video.transformer_lingbot_video import LingBotVideoSparseMoeBlock

    torch.manual_seed(21)
    blk = LingBotVideoSparseMoeBlock(hidden_size=128, intermediate_size=256, num_experts=8, top_k=2,
                                     moe_intermediate_size=128, score_func="sigmoid", norm_topk_prob=True,
                                     n_group=None, topk_group=None, routed_scaling_factor=2.5, n_shared_experts=1)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0.0, 0.05)
        blk.router.e_score_correction_bias.normal_(0.0, 0.1)
    blk = blk.to(torch.bfloat16)
    blk.router.float()
    B, S, H = 2, 64, 128
    x = torch.randn(B, S, H).to(torch.bfloat16)
    grad = torch.randn(B, S, H).to(torch.bfloat16)
    res = {"x": _bf16_bits(x), "grad": _bf16_bits(grad), "top_k": np.int64(2), "route_scale": np.float32(2.5),
           "router_weight": blk.router.weight.detach().float().numpy(),
           "correction_bias": blk.router.e_score_correction_bias.detach().float().numpy()}
    for key in ("w1", "w2", "w3"):
        res[f"experts_{key}"] = _bf16_bits(getattr(blk.experts, key))
    for name in ("gate_proj", "up_proj", "down_proj"):
        res[f"shared_{name}"] = _bf16_bits(getattr(blk.shared_experts, name).weight)
    with torch.no_grad():
        idx, sc, *_ = blk.router(x.reshape(-1, H))
    res["top_indices"], res["top_scores"] = idx.numpy().astype(np.int64), sc.float().numpy()
    blk.train()
    for tag, chunk in (("", 0), ("_chunked", 48)):
        blk.set_token_chunk_policy(MoETokenChunkPolicy(token_chunk_size=chunk) if chunk else None)
        xi = x.clone().requires_grad_(True)
        out = blk(xi)
        out.backward(grad)
        res[f"out{tag}"], res[f"grad_x{tag}"] = _bf16_bits(out), _bf16_bits(xi.grad)
    blk.set_token_chunk_policy(None)
    blk.eval()
    mask = torch.ones(B * S)
    mask[S - 7:S] = 0  # the first sample's last 7 tokens are padding
    with torch.no_grad():
        res["padding_mask"] = mask.numpy()
        res["out_masked"] = _bf16_bits(blk(x, padding_mask=mask))
    np.savez_compressed(OUT / "lingbot_block.npz", **res)


def magi2_moe() -> None:
    """MAGI-2's ``CoreMultiHeadMoE`` (magi2_preview.py:2630-2829), vendored
    reference path (``_torch_forward``, swiglu7, bf16 index_add combine): 4
    heads of d_head 64, 4 experts per head (16 groups), top-2, d_expert 64,
    sigmoid routing with a per-head expert bias, L1 route norm, route_scale
    4.9, bf16.  Records the router's routes, the layer output, and the experts'
    forward and autograd given those routes (x_heads and topk_probs gradients)."""
    import torch
    from mirai.vendors.magi2_preview.model.magi2_preview import CoreMultiHeadMoE, CoreMultiHeadMoEConfig

    torch.manual_seed(31)
    cfg = CoreMultiHeadMoEConfig(hidden_size=256, num_heads=4, num_experts=4, top_k=2, expert_intermediate_size=64,
                                 num_layers=1, params_dtype=torch.bfloat16, score_func="sigmoid", route_norm=True,
                                 route_scale=4.9)
    m = CoreMultiHeadMoE(cfg)
    with torch.no_grad():
        m.gate.normal_(0.0, 0.05)
        for key in ("W_gate", "W_up", "W_down"):
            getattr(m, key).normal_(0.0, 0.05)
        m.router.expert_bias.normal_(0.0, 0.1)
    S = 96
    x = torch.randn(S, 256).to(torch.bfloat16)
    x_heads = x.view(S, 4, 64)
    with torch.no_grad():
        probs, idx = m._route(x_heads)
        out = m._forward_impl(x)
    xh = x_heads.clone().requires_grad_(True)
    pr = probs.clone().requires_grad_(True)
    eo = m._torch_forward(xh, pr, idx)
    grad = torch.randn_like(eo)
    eo.backward(grad)
    np.savez_compressed(
        OUT / "magi2_moe.npz", x=_bf16_bits(x), gate=m.gate.detach().float().numpy(),
        expert_bias=m.router.expert_bias.float().numpy(), W_gate=_bf16_bits(m.W_gate), W_up=_bf16_bits(m.W_up),
        W_down=_bf16_bits(m.W_down), heads=np.int64(4), experts=np.int64(4), top_k=np.int64(2),
        route_scale=np.float32(4.9), topk_probs=probs.float().numpy(), topk_indices=idx.numpy().astype(np.int64),
        out=_bf16_bits(out), experts_out=_bf16_bits(eo), grad=_bf16_bits(grad), grad_x_heads=_bf16_bits(xh.grad),
        grad_probs=pr.grad.float().numpy())


def main(only=None) -> None:
    if not REF or not os.path.isdir(os.path.join(REF, "mirai")):
        raise SystemExit("set MIRAI_REFERENCE to the root of a seruva19/mirai checkout (the directory holding mirai/)")
    sys.path.insert(0, REF)
    import torch

    torch.set_num_threads(4)
    only = set(only or {"basic", "routed", "lingbot_block", "magi2_moe"})
    if "lingbot_block" in only:
        lingbot_block()
    if "magi2_moe" in only:
        magi2_moe()
    if "basic" in only:
        basic_fixtures()
    if "routed" in only:
        routed_fixtures()
    print("golden fixtures written to", OUT)


def basic_fixtures() -> None:
    import torch
    from mirai.core.moe.routing.routers import TokenChoiceRouter
    from mirai.core.models.compressed_weights.execution.dispatch_preprocess import build_dispatch_plan
    from mirai.core.models.compressed_weights.execution.dispatch_ops import (
        combine_routed_tokens, permute_routed_tokens)
    from mirai.core.models.compressed_weights.quantization.quant import (
        _dequantize_weight, _quantize_weight)

    # ------------------------------------------------------------------ router
    for name, (T, H, E, k, seed) in {
        "router_e8_k2": (257, 64, 8, 2, 0),
        "router_e64_k4": (300, 96, 64, 4, 1),
        "router_e128_k8": (129, 64, 128, 8, 2),
    }.items():
        torch.manual_seed(seed)
        router = TokenChoiceRouter(hidden_size=H, num_experts=E, experts_per_token=k, layer_name=name)
        with torch.no_grad():
            router.gate.weight.normal_(0.0, 0.02)
        hs = torch.randn(1, T, H)
        with torch.no_grad():
            dec = router(hs)
            logits = router.gate(hs.reshape(T, H)).float()
        np.savez_compressed(
            OUT / f"{name}.npz",
            logits=logits.numpy(), top_indices=dec.topk_indices.numpy().astype(np.int64),
            top_weights=dec.topk_weights.float().numpy(), k=np.int64(k))

    # ------------------------------------------------------------------ dispatch plan
    g = torch.Generator().manual_seed(3)
    cases = {
        "plan_uniform": torch.randint(0, 16, (500, 4), generator=g),
        "plan_dups_empty": torch.randint(0, 5, (97, 3), generator=g) * 2,  # odd experts empty, dup routes
        "plan_single": torch.zeros((33, 1), dtype=torch.int64),
    }
    skew = torch.multinomial(torch.tensor([0.6, 0.2, 0.1, 0.05, 0.05] + [0.0] * 3), 400 * 2,
                             replacement=True, generator=g).reshape(400, 2)
    cases["plan_skew"] = skew
    for name, idx in cases.items():
        E = int(idx.max().item()) + 1 + (2 if name == "plan_dups_empty" else 0)
        scores = torch.rand(idx.shape, generator=g)
        plan = build_dispatch_plan(idx, scores, E)
        np.savez_compressed(
            OUT / f"{name}.npz", top_indices=idx.numpy().astype(np.int64), num_experts=np.int64(E),
            counts=plan.counts.numpy(), starts=plan.starts.numpy(), offsets=plan.offsets.numpy(),
            sort_positions=plan.sort_positions.numpy(), sorted_token_indices=plan.sorted_token_indices.numpy(),
            inverse_order=plan.inverse_order.numpy())

    # ------------------------------------------------------------------ permute / combine
    torch.manual_seed(7)
    tokens = torch.randn(37, 24, requires_grad=True)
    indices = torch.randint(0, 37, (90,))
    scores = torch.randn(90, requires_grad=True)
    routed = permute_routed_tokens(tokens, indices)
    expert_out = routed * 1.5 - 0.25
    out = combine_routed_tokens(expert_out, scores, indices, output_rows=37, output_dtype=tokens.dtype)
    grad = torch.randn_like(out)
    out.backward(grad)
    np.savez_compressed(OUT / "permute_combine.npz", tokens=tokens.detach().numpy(), indices=indices.numpy(),
                        scores=scores.detach().numpy(), out=out.detach().numpy(), grad=grad.numpy(),
                        grad_tokens=tokens.grad.numpy(), grad_scores=scores.grad.numpy())

    # ------------------------------------------------------------------ INT8 quantisation
    torch.manual_seed(11)
    w = torch.randn(3, 48, 256) * 0.05
    w[1, 5] = 0.0  # an all-zero row exercises the 1e-30 scale clamp
    res = {"weight": w.numpy()}
    for gsz in (0, 16, 64, 256):
        q, s, gres = _quantize_weight(w, group_size=gsz)
        deq = _dequantize_weight(q, s, group_size=gres, dtype=torch.float32, device=torch.device("cpu"))
        res[f"q_g{gsz}"] = q.numpy()
        res[f"s_g{gsz}"] = s.numpy()
        res[f"deq_g{gsz}"] = deq.numpy()
        res[f"gres_g{gsz}"] = np.int64(gres)
    np.savez_compressed(OUT / "int8_quant.npz", **res)



def routed_fixtures() -> None:
    import torch
    import torch.nn as nn
    from mirai.core.models.compressed_weights.quantization.quant import _quantize_weight
    from mirai.core.models.compressed_weights import CompressedGroupedExperts

    # ------------------------------------------------------------------ routed expert execution
    class _Base(nn.Module):
        def __init__(self, E, H, I, dtype):
            super().__init__()
            self.num_experts = E
            self.w1 = (torch.randn(E, I, H) * 0.05).to(dtype)
            self.w2 = (torch.randn(E, H, I) * 0.05).to(dtype)
            self.w3 = (torch.randn(E, I, H) * 0.05).to(dtype)

    class _DenseProvider:
        def __init__(self, base):
            self.num_experts = base.num_experts
            self._w = {"w1": base.w1, "w2": base.w2, "w3": base.w3}

        def expert_weight_shape(self, key):
            return tuple(self._w[key].shape)

        def materialize_expert(self, key, expert_idx, *, dtype, device):
            return self._w[key][int(expert_idx)].to(dtype=dtype, device=device)

    def routed_case(name, *, T, H, E, k, I, dtype, fmt, lora_rank=0, seed=0, group=0):
        torch.manual_seed(seed)
        base = _Base(E, H, I, torch.float32 if fmt == "int8" else dtype)
        if fmt == "int8":
            experts = CompressedGroupedExperts(base, group_sizes=group if group else 16,
                                               expert_weight_access="chunked_dequant",
                                               expert_dequant_chunk_size=16, quant_format="int8")
            if group == 0:
                for key in ("w1", "w2", "w3"):
                    q, s, _ = _quantize_weight(getattr(base, key), group_size=0)
                    experts.load_quantized_weight(key, weight_int8=q, weight_scale=s, group_size=0)
        else:
            experts = CompressedGroupedExperts.from_empty(num_experts=E, expert_weight_access="chunked_dequant",
                                                          expert_dequant_chunk_size=16, quant_format="int8")
            experts.bind_physical_weight_provider(_DenseProvider(base))
        lora = {}
        if lora_rank:
            experts.attach_expert_lora(tensor_name="w2", adapter_name="lora", rank=lora_rank, alpha=float(lora_rank))
            with torch.no_grad():
                experts.expert_lora["w2"].lora_b.add_(0.02 * torch.randn_like(experts.expert_lora["w2"].lora_b))
            lora = {"lora_a": experts.expert_lora["w2"].lora_a.detach().float().numpy(),
                    "lora_b": experts.expert_lora["w2"].lora_b.detach().float().numpy(),
                    "lora_scale": np.float32(1.0)}
        experts.train()
        tokens = torch.randn(T, H).to(dtype).requires_grad_(True)
        logits = torch.randn(T, E) * 1.5
        top_scores_f, top_indices = torch.topk(torch.softmax(logits, -1), k, dim=-1)
        top_scores = (top_scores_f / top_scores_f.sum(-1, keepdim=True)).to(dtype).requires_grad_(True)
        out = experts.run_direct_routed(tokens, top_scores, top_indices)
        grad = torch.randn_like(out)
        out.backward(grad)
        if fmt == "int8":
            wts = {}
            for key in ("w1", "w2", "w3"):
                wts[f"{key}_int8"] = getattr(experts, f"{key}_int8").numpy()
                wts[f"{key}_scale"] = getattr(experts, f"{key}_scale").numpy()
            wts["group_size"] = np.int64(getattr(experts, "w1_group_size"))
        else:
            wts = {key: _bf16_bits(getattr(base, key)) for key in ("w1", "w2", "w3")}
        is_bf16 = dtype == torch.bfloat16
        conv = _bf16_bits if is_bf16 else (lambda t: t.detach().float().numpy())
        np.savez_compressed(
            OUT / f"{name}.npz", tokens=conv(tokens), top_indices=top_indices.numpy().astype(np.int64),
            top_scores=conv(top_scores), out=conv(out), grad=conv(grad), grad_tokens=conv(tokens.grad),
            grad_scores=conv(top_scores.grad), bf16=np.bool_(is_bf16), **wts, **lora)

    routed_case("routed_int8_fp32", T=96, H=64, E=6, k=2, I=128, dtype=torch.float32, fmt="int8", seed=1)
    routed_case("routed_int8_g16_fp32", T=64, H=64, E=4, k=2, I=64, dtype=torch.float32, fmt="int8", seed=2, group=16)
    routed_case("routed_int8_bf16", T=80, H=128, E=20, k=4, I=64, dtype=torch.bfloat16, fmt="int8", seed=3)
    routed_case("routed_dense_bf16", T=128, H=128, E=8, k=2, I=128, dtype=torch.bfloat16, fmt="dense", seed=4)
    routed_case("routed_dense_bf16_lora", T=96, H=64, E=4, k=2, I=128, dtype=torch.bfloat16, fmt="dense",
                seed=5, lora_rank=4)


if __name__ == "__main__":
    # no arguments: every fixture; otherwise any of "basic" (router, plan, permute/combine, INT8
    # quantisation), "routed" (routed execution), "lingbot_block" and "magi2_moe"
    main(set(sys.argv[1:]) or {"basic", "routed", "lingbot_block", "magi2_moe"})
