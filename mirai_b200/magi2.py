"""MAGI-2 multi-head grouped MoE on libmirai_b200 (the second model family).

MAGI-2's routed layer (``CoreMultiHeadMoE``, magi2_preview.py:2630-2829;
Mirai's grouped execution, grouped_moe.py:583-757) splits every token's
hidden vector into ``heads`` slices of ``d_head`` features and routes each
slice among the ``E`` experts of its own head:

* router: logits = einsum("shd,hed->hse", x_heads, gate) in fp32, sigmoid (or
  softmax) scores, top-k of score + expert_bias[head] per (head, token),
  weights gathered from the unbiased scores, L1-normalised
  (``F.normalize(p=1, eps=1e-12)``) when ``route_norm``, times ``route_scale``
  (magi2_preview.py:2727-2744; flash_mh_moe/route.py:28-199);
* experts: (head, expert) flattened into heads * E groups; rows are the
  (token, head) slices of x_heads [S, heads, d_head]; gate = x W_gate[g],
  up = x W_up[g] with W_gate / W_up [G, d_head, d_expert] and W_down
  [G, d_expert, d_head] (stored input-major), h = swiglu7(gate, up), y = h W_down[g];
* combine: bf16 y * bf16(weight) index-added into bf16 rows in sorted order.

Here: the router kernel with one bias row per head (``route_topk`` with a
[heads, E] bias), the dispatch plan over heads * E groups (up to 4096), the
``*_ex`` grouped GEMMs reading the [G, in, out] weights as stored (bf16, or the
NF4 store's ``{key}_nf4*`` buffers, magi2 quantized_experts.py:278-347) with the
swiglu7 epilogue and its backward, groups beyond 1024 in consecutive
launches, and the bf16-accumulating combine.  ``B200Magi2MoEBackend`` is the
object the layer's kernel-backend seam calls
(``backend.execute(module, x_heads, topk_probs, topk_indices)``,
magi2_preview.py:2810-2817); attach it with ``attach(transformer)``.
"""

from __future__ import annotations

from typing import Any

import torch

from . import ops

LAYOUT = "in_out"
KEYS = ("W_gate", "W_up", "W_down")
NF4_STORE_ATTR = "mirai_nf4_experts"  # where the NF4 store hangs on a MAGI-2 MoE layer


class Magi2ExpertWeights:
    """The three routed tensors of one MAGI-2 MoE layer as kernel operands:
    bf16 tensors, or ``ops.NF4Tensor`` of the NF4 store's buffers."""

    def __init__(self, w_gate, w_up, w_down, *, heads: int, experts: int, d_head: int, d_expert: int):
        self.w_gate, self.w_up, self.w_down = w_gate, w_up, w_down
        self.heads, self.experts = int(heads), int(experts)
        self.d_head, self.d_expert = int(d_head), int(d_expert)
        self.groups = self.heads * self.experts

    @classmethod
    def from_module(cls, module: Any) -> "Magi2ExpertWeights":
        heads = int(getattr(module, "local_num_heads", getattr(module, "num_heads")))
        E = int(module.num_experts)
        d_head, d_expert = int(module.d_head), int(module.d_expert)
        store = getattr(module, NF4_STORE_ATTR, None)
        if store is not None and all(hasattr(store, f"{k}_nf4") for k in KEYS):
            meta = getattr(store, "_meta", None)
            bs = int(getattr(meta, "blocksize", 64)) if meta is not None else 64
            nbs = int(getattr(meta, "nested_blocksize", 256)) if meta is not None else 256
            ws = [ops.NF4Tensor(getattr(store, f"{k}_nf4"), getattr(store, f"{k}_nf4_absmax"),
                                getattr(store, f"{k}_nf4_nabsmax"), getattr(store, f"{k}_nf4_offset"),
                                getattr(store, f"{k}_nf4_code"), getattr(store, f"{k}_nf4_ncode"),
                                tuple(store._shapes[k]), bs, nbs) for k in KEYS]
        else:
            ws = [getattr(module, k).detach().to(torch.bfloat16).contiguous() for k in KEYS]
        return cls(*ws, heads=heads, experts=E, d_head=d_head, d_expert=d_expert)


def route(x_heads: torch.Tensor, gate: torch.Tensor, expert_bias: torch.Tensor | None, *, experts: int, top_k: int,
          score_func: str = "sigmoid", route_norm: bool = True, route_scale: float = 1.0):
    """(topk_probs fp32 [heads, S, k], topk_indices int64 [heads, S, k]) of the
    MAGI-2 router (magi2_preview.py:2727-2744).  The logits are one batched
    fp32 GEMM (cuBLAS); the per-head top-k is the router kernel."""
    S, H, d = x_heads.shape
    logits = torch.einsum("shd,hed->hse", x_heads.float(), gate.reshape(H, experts, d).float())
    bias = None if expert_bias is None else expert_bias.reshape(H, experts).float()
    idx, w = ops.route_topk(logits.reshape(H * S, experts).contiguous(), top_k, score_func=score_func,
                            choice_bias=bias, norm="l1" if route_norm else "none", route_scale=route_scale)
    return w.reshape(H, S, top_k), idx.reshape(H, S, top_k)


def _flat_routes(topk_probs, topk_indices, experts: int):
    """Routes of the (token, head) rows of x_heads [S, H, d] as flat group ids
    head * E + expert, in row order (each head's tokens ascend within a group,
    the order of grouped_moe.py:660-666)."""
    H, S, k = topk_indices.shape
    head = torch.arange(H, device=topk_indices.device).view(H, 1, 1)
    flat = (topk_indices + head * experts).permute(1, 0, 2).reshape(S * H, k).contiguous()
    probs = topk_probs.float().permute(1, 0, 2).reshape(S * H, k).contiguous()
    return flat, probs


class _Magi2ExpertsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_heads, topk_probs, topk_indices, weights: Magi2ExpertWeights):
        S, H, d = x_heads.shape
        flat, probs = _flat_routes(topk_probs, topk_indices, weights.experts)
        plan = ops.dispatch_plan(flat, weights.groups)
        xs = ops.permute_rows(x_heads.reshape(S * H, d).to(torch.bfloat16).contiguous(), plan.sorted_token_indices)
        need = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        res = ops.gateup_ex(xs, plan.offsets, weights.w_gate, weights.w_up, inter=weights.d_expert, layout=LAYOUT,
                            activation="swiglu7", save_gate_up=need)
        h, gu = res if need else (res, None)
        y = ops.down_ex(h, plan.offsets, weights.w_down, hidden=d, layout=LAYOUT)
        # weights rounded to bf16 as the reference's sorted_probs.to(bf16)
        pw = probs.to(torch.bfloat16).float()
        out = ops.combine(y, plan.inverse_order, pw, bf16_accumulate=True)
        if need:
            ctx.state = (plan, y, gu, pw)
            ctx.weights = weights
            ctx.shape = (S, H, d)
            ctx.dtypes = (x_heads.dtype, topk_probs.dtype)
        return out.view(S, H, d).to(x_heads.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        plan, y, gu, pw = ctx.state
        w = ctx.weights
        S, H, d = ctx.shape
        g = grad_out.reshape(S * H, d).to(torch.bfloat16).contiguous()
        gy, gw = ops.combine_backward(g, y, plan.inverse_order, pw)
        dgu = ops.down_dx_ex(gy, plan.offsets, w.w_down, gu, inter=w.d_expert, layout=LAYOUT, activation="swiglu7")
        dxs = ops.gateup_dx_ex(dgu, plan.offsets, w.w_gate, w.w_up, hidden=d, layout=LAYOUT)
        dx = ops.combine(dxs, plan.inverse_order, None, top_k=plan.top_k, bf16_accumulate=True)
        ctx.state = None
        k = plan.top_k
        dprobs = gw.reshape(S, H, k).permute(1, 0, 2).contiguous()
        return dx.view(S, H, d).to(ctx.dtypes[0]), dprobs.to(ctx.dtypes[1]), None, None


def run_experts(x_heads: torch.Tensor, topk_probs: torch.Tensor, topk_indices: torch.Tensor,
                weights: Magi2ExpertWeights) -> torch.Tensor:
    """The routed experts of one MAGI-2 MoE layer (grouped_moe.py:615-757):
    x_heads [S, H, d_head], routes [H, S, k] -> [S, H, d_head]; differentiable
    in x_heads and topk_probs (frozen experts)."""
    if not x_heads.is_cuda:
        raise ValueError("the B200 MAGI-2 expert path runs on CUDA tensors only (no CPU fallback)")
    S, H, d = x_heads.shape
    if tuple(topk_indices.shape[:2]) != (H, S) or topk_probs.shape != topk_indices.shape:
        raise ValueError(f"routes of shape {tuple(topk_indices.shape)} do not match x_heads {tuple(x_heads.shape)}")
    if H != weights.heads or d != weights.d_head:
        raise ValueError(f"x_heads [S, {H}, {d}] against experts of {weights.heads} heads x d_head {weights.d_head}")
    return _Magi2ExpertsFunction.apply(x_heads, topk_probs, topk_indices.to(torch.int64), weights)


class B200Magi2MoEBackend:
    """The MAGI-2 layer's grouped execution seam on libmirai_b200
    (``Magi2GroupedMoEBackend.execute``'s contract, grouped_moe.py:615-637).
    ``token_chunk_size`` > 0 runs the routed experts chunk by chunk over
    contiguous token ranges (the routes stay whole), as the reference's
    backend does."""

    name = "b200"

    def __init__(self, *, token_chunk_size: int = 0):
        self.token_chunk_size = int(token_chunk_size)
        self._cache: dict[int, tuple[tuple, Magi2ExpertWeights]] = {}

    def bind(self, module: Any) -> Magi2ExpertWeights:
        store = getattr(module, NF4_STORE_ATTR, None)
        src = store if store is not None else module
        key = tuple((n, b.data_ptr(), b._version) for n, b in sorted(
            list(getattr(src, "_buffers", {}).items()) + list(getattr(src, "_parameters", {}).items()))
            if isinstance(b, torch.Tensor))
        hit = self._cache.get(id(module))
        if hit is None or hit[0] != key:
            hit = (key, Magi2ExpertWeights.from_module(module))
            self._cache[id(module)] = hit
        return hit[1]

    def execute(self, module: Any, x_heads: torch.Tensor, topk_probs: torch.Tensor,
                topk_indices: torch.Tensor) -> torch.Tensor:
        weights = self.bind(module)
        S = int(x_heads.shape[0])
        c = self.token_chunk_size
        if c <= 0 or S <= c:
            return run_experts(x_heads, topk_probs, topk_indices, weights)
        outs = [run_experts(x_heads[a:min(a + c, S)], topk_probs[:, a:min(a + c, S)],
                            topk_indices[:, a:min(a + c, S)], weights) for a in range(0, S, c)]
        return torch.cat(outs, dim=0)

    # the reference backend's layout checks: this path reads any layout the weights come in
    def inspect_expert_layout(self, module: Any) -> tuple[str, ...]:
        return ()

    def validate_explicit_alignment(self) -> None:
        return None


def attach(transformer: Any, backend: B200Magi2MoEBackend | None = None) -> int:
    """Install the backend on every MAGI-2 multi-head MoE layer of a model
    (``attach_grouped_moe_backend``, grouped_moe.py:1704-1722): modules that
    carry the layer's routed tensors (W_gate, W_up, W_down) and a
    ``_mirai_moe_kernel_backend`` seam.  Returns how many were attached."""
    backend = backend or B200Magi2MoEBackend()
    n = 0
    for m in transformer.modules():
        if hasattr(m, "_mirai_moe_kernel_backend") and all(hasattr(m, k) for k in KEYS):
            m._mirai_moe_kernel_backend = backend
            n += 1
    if n == 0:
        raise ValueError("no MAGI-2 multi-head MoE layer found to attach the b200 backend to")
    return n
