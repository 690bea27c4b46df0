"""The LingBot sparse-MoE block around the routed expert path, on libmirai_b200.

The reference block (``LingBotVideoSparseMoeBlock``,
transformer_lingbot_video.py:1175-1205, forward 2218-2377) is: an fp32 router
(``LingBotVideoRouter.forward``, :962-1033: logits = x W_r^T in fp32, sigmoid or
softmax scores, choice on score + e_score_correction_bias, weights gathered
from the unbiased scores, renormalised when ``norm_topk_prob``, times
``route_scale``), an optional padding-mask renormalisation (:2283-2287), the
routed experts behind the kernel-backend seam, optionally split into token
chunks by ``MoETokenChunkPolicy`` (:2289-2345; token_chunking.py:48-117), and
a shared-expert MLP added to the routed output (:2374-2377;
``LingBotVideoMLP``, :491-499).

Two ways to use this module:

* ``install(block)`` turns a reference block (when the reference is importable)
  into one that runs here: it installs ``B200MoEKernelBackend`` on the
  kernel-backend seam (``block._mirai_moe_kernel_backend``, the attribute
  pipeline.py:4556-4561 sets) and replaces ``block.shared_experts`` by
  ``SharedExpertMLP`` holding the same parameters;
* ``B200SparseMoeBlock`` is the block itself, built from a reference block's
  tensors (``from_state``) where the reference is not importable.

Expert selection is the sm_100a router kernel; the routing weights that carry
gradients back into the router are recomputed in torch from the selected
indices (an elementwise [T, k] gather), so the router stays trainable.
"""

from __future__ import annotations

from typing import Any, Callable, Mapping

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .backend import B200MoEKernelBackend
from .experts import GroupedExpertWeights, run_routed


# ----------------------------------------------------------------------------- shared expert

class _SharedMLPFunction(torch.autograd.Function):
    """down(silu(gate(x)) * up(x)) as a one-expert grouped GEMM pair over all
    tokens (offsets = [T]); backward = dX through the frozen projections."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down):
        T, H = x.shape
        inter = w_gate.shape[0]
        offsets = torch.full((1,), T, dtype=torch.int32, device=x.device)
        xb = x.to(torch.bfloat16).contiguous()
        need = ctx.needs_input_grad[0]
        if need:
            h, gu = ops.gateup_swiglu(xb, offsets, w_gate[None], w_up[None], inter=inter, save_gate_up=True)
            ctx.save_for_backward(offsets, gu)
            ctx.weights = (w_gate, w_up, w_down)
        else:
            h = ops.gateup_swiglu(xb, offsets, w_gate[None], w_up[None], inter=inter)
        ctx.in_dtype = x.dtype
        return ops.down(h, offsets, w_down[None], hidden=H).to(x.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        offsets, gu = ctx.saved_tensors
        w_gate, w_up, w_down = ctx.weights
        inter = w_gate.shape[0]
        H = w_down.shape[0]
        gy = grad_out.to(torch.bfloat16).contiguous()
        dgu = ops.down_dx(gy, offsets, w_down[None], gu, inter=inter)
        dx = ops.gateup_dx(dgu, offsets, w_gate[None], w_up[None], hidden=H)
        return dx.to(ctx.in_dtype), None, None, None


class SharedExpertMLP(nn.Module):
    """The LingBot shared-expert MLP (``gate_proj``, ``up_proj``, ``down_proj``
    bias-free linears, transformer_lingbot_video.py:491-499) on the grouped
    GEMM kernels with a single expert.  Parameter names match the reference, so
    its state dict loads as is.  The projections are frozen (bf16); the input
    gradient flows."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)
        self._bf16 = None

    @classmethod
    def from_module(cls, mlp: nn.Module) -> "SharedExpertMLP":
        out_f, in_f = mlp.gate_proj.weight.shape
        m = cls(in_f, out_f)
        m.load_state_dict({k: v.detach() for k, v in mlp.state_dict().items()})
        return m.to(mlp.gate_proj.weight.device)

    def _weights(self):
        ws = (self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight)
        key = tuple((w.data_ptr(), w._version) for w in ws)
        if self._bf16 is None or self._bf16[0] != key:
            self._bf16 = (key, tuple(w.detach().to(torch.bfloat16).contiguous() for w in ws))
        return self._bf16[1]

    def _apply(self, fn, recurse=True):
        self._bf16 = None
        return super()._apply(fn, recurse)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        return _SharedMLPFunction.apply(flat, *self._weights()).reshape(shape)


# ----------------------------------------------------------------------------- token chunks

class TokenChunkPolicy:
    """``MoETokenChunkPolicy`` (token_chunking.py:25-117): with a positive
    ``token_chunk_size``, a routed batch of more than that many tokens runs its
    expert execution chunk by chunk in training (the route plan stays whole),
    each chunk under activation checkpointing when gradients are enabled;
    otherwise (size 0, inference, or a small batch) one call."""

    def __init__(self, token_chunk_size: int = 0):
        if int(token_chunk_size) < 0:
            raise ValueError("token chunk size must be >= 0")
        self.token_chunk_size = int(token_chunk_size)

    @property
    def enabled(self) -> bool:
        return self.token_chunk_size > 0

    def chunk_count(self, token_count: int) -> int:
        if token_count < 0:
            raise ValueError("token count must be >= 0")
        if not self.enabled or token_count == 0:
            return 1
        return -(-token_count // self.token_chunk_size)

    def execute(self, tokens, top_scores, top_indices, *, runner: Callable, training: bool):
        if tuple(top_scores.shape) != tuple(top_indices.shape) or top_indices.ndim != 2:
            raise ValueError("token chunks need matching [tokens, top_k] scores and indices")
        if tokens.ndim != 2 or tokens.shape[0] != top_indices.shape[0]:
            raise ValueError("token chunks need [tokens, hidden] tokens routed by the given indices")
        T = int(tokens.shape[0])
        if not self.enabled or T <= self.token_chunk_size or not training:
            return runner(tokens, top_scores, top_indices, 0)
        checkpointed = torch.is_grad_enabled()
        outs = []
        for start in range(0, T, self.token_chunk_size):
            end = min(start + self.token_chunk_size, T)
            args = (tokens[start:end], top_scores[start:end], top_indices[start:end])
            if checkpointed:
                from torch.utils.checkpoint import checkpoint
                outs.append(checkpoint(lambda a, b, c, s=start: runner(a, b, c, s), *args, use_reentrant=False,
                                       preserve_rng_state=True))
            else:
                outs.append(runner(*args, start))
        return torch.cat(outs, dim=0)


# ----------------------------------------------------------------------------- router

def route(tokens: torch.Tensor, weight: torch.Tensor, *, top_k: int, score_func: str = "sigmoid",
          correction_bias: torch.Tensor | None = None, norm_topk_prob: bool = True, route_scale: float = 1.0):
    """The LingBot router (transformer_lingbot_video.py:962-1033, without the
    research extensions): returns (top_indices int64 [T, k], top_scores in the
    tokens' dtype).  Selection runs in the sm_100a router kernel on fp32 logits;
    when the router weight needs a gradient the weights are re-gathered in torch
    from the unbiased scores so that autograd reaches it."""
    logits = F.linear(tokens.float(), weight.float())
    bias = None if correction_bias is None else correction_bias.float().contiguous()
    lg = logits.detach().contiguous()
    if norm_topk_prob:  # w / (sum w + 1e-20) for k > 1, then * route_scale, in the kernel
        idx, w = ops.route_topk(lg, top_k, score_func=score_func, choice_bias=bias, norm="eps",
                                route_scale=route_scale)
    else:  # the gathered scores times route_scale
        idx, w = ops.route_topk(lg, top_k, score_func=score_func, choice_bias=bias, norm="none",
                                route_scale=route_scale)
    if torch.is_grad_enabled() and logits.requires_grad:
        scores = torch.sigmoid(logits) if score_func == "sigmoid" else torch.softmax(logits, dim=-1)
        w = scores.gather(1, idx)
        if top_k > 1 and norm_topk_prob:
            w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
        w = w * route_scale
    return idx, w.to(tokens.dtype)


# ----------------------------------------------------------------------------- block

class B200SparseMoeBlock(nn.Module):
    """``LingBotVideoSparseMoeBlock`` (inference and LoRA-free training path) on
    libmirai_b200: router kernel, routed experts through the grouped-GEMM
    kernels (any format ``GroupedExpertWeights`` binds), optional token chunks,
    shared expert on the one-expert GEMMs.  ``forward(hidden_states [B, S, H],
    padding_mask [B*S] or None) -> [B, S, H]``."""

    def __init__(self, *, hidden_size: int, num_experts: int, top_k: int, score_func: str = "sigmoid",
                 norm_topk_prob: bool = True, route_scale: float = 1.0, experts: nn.Module,
                 shared_experts: nn.Module | None = None, token_chunk_policy: TokenChunkPolicy | None = None):
        super().__init__()
        if score_func not in ("sigmoid", "softmax"):
            raise ValueError(f"score_func {score_func!r}: sigmoid or softmax")
        self.hidden_size, self.num_experts, self.top_k = int(hidden_size), int(num_experts), int(top_k)
        self.score_func, self.norm_topk_prob, self.route_scale = score_func, bool(norm_topk_prob), float(route_scale)
        self.router_weight = nn.Parameter(torch.empty(num_experts, hidden_size))
        self.register_buffer("e_score_correction_bias", torch.zeros(num_experts))
        self.experts = experts
        self.shared_experts = shared_experts
        self.token_chunk_policy = token_chunk_policy
        self._backend = B200MoEKernelBackend(strict=True)

    @classmethod
    def from_state(cls, state: Mapping[str, torch.Tensor], *, top_k: int, score_func: str = "sigmoid",
                   norm_topk_prob: bool = True, route_scale: float = 1.0,
                   token_chunk_policy: TokenChunkPolicy | None = None) -> "B200SparseMoeBlock":
        """A block from a reference block's state dict: ``router.weight``,
        ``router.e_score_correction_bias``, ``experts.w1/w2/w3`` (dense, or the
        experts module passed already quantised as ``state["experts"]``) and,
        if present, ``shared_experts.{gate,up,down}_proj.weight``."""
        from .experts import B200GroupedExperts
        rw = state["router.weight"]
        E, H = rw.shape
        experts = state.get("experts")
        if experts is None:
            experts = B200GroupedExperts.from_empty(num_experts=E, quant_format="bf16")
            for key in ("w1", "w2", "w3"):
                experts.load_dense_weight(key, state[f"experts.{key}"])
        shared = None
        if "shared_experts.gate_proj.weight" in state:
            I_s = state["shared_experts.gate_proj.weight"].shape[0]
            shared = SharedExpertMLP(H, I_s).to(rw.device)
            shared.load_state_dict({k.split(".", 1)[1]: v for k, v in state.items()
                                    if k.startswith("shared_experts.")})
        blk = cls(hidden_size=H, num_experts=E, top_k=top_k, score_func=score_func, norm_topk_prob=norm_topk_prob,
                  route_scale=route_scale, experts=experts, shared_experts=shared,
                  token_chunk_policy=token_chunk_policy).to(rw.device)
        with torch.no_grad():
            blk.router_weight.copy_(rw)
            if "router.e_score_correction_bias" in state:
                blk.e_score_correction_bias.copy_(state["router.e_score_correction_bias"])
        return blk

    def _run_selected_experts(self, tokens, top_scores, top_indices, token_offset: int = 0):
        out = self._backend.execute_direct(self.experts, tokens, top_scores, top_indices)
        return out

    def forward(self, hidden_states: torch.Tensor, padding_mask: torch.Tensor | None = None) -> torch.Tensor:
        B = hidden_states.shape[0]
        tokens = hidden_states.reshape(-1, self.hidden_size)
        idx, scores = route(tokens, self.router_weight, top_k=self.top_k, score_func=self.score_func,
                            correction_bias=self.e_score_correction_bias, norm_topk_prob=self.norm_topk_prob,
                            route_scale=self.route_scale)
        if padding_mask is not None:  # transformer_lingbot_video.py:2283-2287
            pm = padding_mask.reshape(-1, 1).to(scores.dtype)
            scores = scores * pm
            scores = scores / (scores.sum(dim=-1, keepdim=True) + 1e-9)
            scores = scores * self.route_scale
        policy = self.token_chunk_policy
        if policy is not None and policy.enabled:
            out = policy.execute(tokens, scores, idx, runner=self._run_selected_experts, training=self.training)
        else:
            out = self._run_selected_experts(tokens, scores, idx)
        out = out.reshape(B, -1, self.hidden_size)
        if self.shared_experts is not None:
            out = out + self.shared_experts(hidden_states)
        return out


def install(block: Any, *, strict: bool = True) -> Any:
    """Run a reference ``LingBotVideoSparseMoeBlock`` on libmirai_b200 in place:
    the routed experts through ``B200MoEKernelBackend`` on the block's
    kernel-backend seam, the shared expert through ``SharedExpertMLP`` (same
    parameters).  Returns the block."""
    block._mirai_moe_kernel_backend = B200MoEKernelBackend(strict=strict)
    shared = getattr(block, "shared_experts", None)
    if shared is not None and not isinstance(shared, SharedExpertMLP):
        block.shared_experts = SharedExpertMLP.from_module(shared)
    return block


__all__ = ["B200SparseMoeBlock", "SharedExpertMLP", "TokenChunkPolicy", "install", "route",
           "GroupedExpertWeights", "run_routed"]
