"""Routed frozen experts executed by libmirai_b200 (the drop-in for the
reference's compressed grouped-expert layer).

``GroupedExpertWeights`` binds the three expert tensors of one MoE layer
(gate ``w1`` [E, I, H], up ``w3`` [E, I, H], down ``w2`` [E, H, I], the
reference's layout, transformer_lingbot_video.py:1143-1145) in one of three
storage formats, reading the reference's own buffers in place:

* NF4: ``{key}_nf4``, ``{key}_nf4_absmax``, ``{key}_nf4_nabsmax``,
  ``{key}_nf4_offset``, ``{key}_nf4_code``, ``{key}_nf4_ncode`` and the
  ``_Nf4Meta`` block sizes (experts.py:998-1031, 1424-1470);
* INT8 (group size 0): ``{key}_int8`` and ``{key}_scale`` (experts.py:1382-1422);
* bf16 dense tensors (the LingBot dense grouped experts).

``B200GroupedExperts`` is an ``nn.Module`` with the reference's construction
and ingest API (``from_empty``, ``load_dense_weight``,
``load_nf4_packed_weight``, ``load_quantized_weight``) and its direct-routed
entry point ``run_direct_routed(tokens, top_scores, top_indices)``
(experts.py:1749-1912), differentiable in ``tokens`` and ``top_scores``
(the dX path through frozen experts; no dense weight is kept for backward,
the invariant of linear.py:96-102).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Iterable

import torch
import torch.nn as nn

from . import ops, tables

KEYS = ("w1", "w3", "w2")  # gate, up, down (specs.py:129-230 canonical roles)


@dataclass
class Nf4Meta:
    """Static NF4 metadata (quant.py:305-312 ``_Nf4Meta``)."""

    blocksize: int = 64
    nested_blocksize: int = 256
    nested_dtype: torch.dtype = torch.float32
    weight_dtype: torch.dtype = torch.bfloat16


class GroupedExpertWeights:
    """The three weight keys of one layer as kernel descriptors."""

    def __init__(self, fmt: str, w1, w3, w2, num_experts: int, hidden: int, inter: int):
        self.fmt = fmt
        self.w1, self.w3, self.w2 = w1, w3, w2
        self.num_experts, self.hidden, self.inter = int(num_experts), int(hidden), int(inter)

    @classmethod
    def from_module(cls, module: Any) -> "GroupedExpertWeights":
        """Bind the buffers of a reference-compatible grouped-expert module.

        Accepts the reference's ``CompressedGroupedExperts`` (NF4, or INT8
        with group size 0), this package's ``B200GroupedExperts`` and dense
        modules exposing ``w1``/``w2``/``w3`` tensors.  The buffers are used
        in place (no copy); they must live on a CUDA device.
        """
        fmt = str(getattr(module, "_quant_format", "")).lower()
        E = int(getattr(module, "num_experts"))
        if fmt == "nf4":
            shapes = getattr(module, "_nf4_shapes")
            meta = getattr(module, "_nf4_meta")
            ws = {}
            for key in KEYS:
                ws[key] = ops.NF4Tensor(
                    getattr(module, f"{key}_nf4"), getattr(module, f"{key}_nf4_absmax"),
                    getattr(module, f"{key}_nf4_nabsmax"), getattr(module, f"{key}_nf4_offset"),
                    getattr(module, f"{key}_nf4_code"), getattr(module, f"{key}_nf4_ncode"),
                    shapes[key], int(meta.blocksize), int(meta.nested_blocksize))
            _, inter, hidden = shapes["w1"]
            return cls("nf4", ws["w1"], ws["w3"], ws["w2"], E, hidden, inter)
        if fmt == "int8" and hasattr(module, "w1_int8"):
            ws = {}
            for key in KEYS:
                g = int(getattr(module, f"{key}_group_size", 0))
                rot = getattr(module, "expert_rotation", None)
                if g != 0 or (callable(rot) and rot(key) is not None):
                    raise ops._lib.MiraiError(
                        2, f"INT8 expert tensor {key} uses block rotation (group size {g}); the fused kernel "
                           "reads plain per-output-channel INT8 (group_size=0)")
                ws[key] = ops.Int8Tensor(getattr(module, f"{key}_int8"), getattr(module, f"{key}_scale"))
            _, inter, hidden = ws["w1"].shape
            return cls("int8", ws["w1"], ws["w3"], ws["w2"], E, hidden, inter)
        w1, w2, w3 = (getattr(module, k, None) for k in ("w1", "w2", "w3"))
        if all(isinstance(w, torch.Tensor) for w in (w1, w2, w3)):
            bf = [w.detach().to(torch.bfloat16).contiguous() for w in (w1, w3, w2)]
            _, inter, hidden = bf[0].shape
            return cls("bf16", bf[0], bf[1], bf[2], E, hidden, inter)
        raise ops._lib.MiraiError(2, f"cannot bind expert weights of {type(module).__name__} (format {fmt!r})")


class _RoutedExpertsFunction(torch.autograd.Function):
    """Forward through the fused kernels; backward = dX, the top-score gradient
    and, with a down-projection LoRA adapter, the adapter factor gradients."""

    @staticmethod
    def forward(ctx, tokens, top_scores, top_indices, weights: GroupedExpertWeights, lora_a, lora_b, lora_scale):
        x = tokens.to(torch.bfloat16).contiguous()
        out_dtype = tokens.dtype if tokens.dtype in (torch.bfloat16, torch.float32) else torch.float32
        need_grad = any(ctx.needs_input_grad[i] for i in (0, 1, 4, 5))
        w = top_scores.float().contiguous()
        lora = None
        if lora_a is not None:
            lora = ops.DownLoRA(lora_a, lora_b, float(lora_scale),
                                compute_grads=ctx.needs_input_grad[4] or ctx.needs_input_grad[5])
        if need_grad:
            out, state = ops.moe_forward_train(x, top_indices.contiguous(), w, weights.w1, weights.w3, weights.w2,
                                               num_experts=weights.num_experts, inter=weights.inter,
                                               out_dtype=out_dtype, lora=lora)
            ctx.state = state
            ctx.weights = weights
            ctx.lora = lora
            ctx.token_dtype = tokens.dtype
            ctx.score_dtype = top_scores.dtype
            ctx.factor_dtypes = (None if lora_a is None else lora_a.dtype, None if lora_b is None else lora_b.dtype)
        else:
            plan = ops.dispatch_plan(top_indices.contiguous(), weights.num_experts)
            xs = ops.permute_rows(x, plan.sorted_token_indices)
            h = ops.gateup_swiglu(xs, plan.offsets, weights.w1, weights.w3, inter=weights.inter)
            y = ops.down(h, plan.offsets, weights.w2, hidden=weights.hidden, lora=lora)
            out = ops.combine(y, plan.inverse_order, w, out_dtype=out_dtype)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        wts = ctx.weights
        lora = ctx.lora
        dx, dw = ops.moe_backward_dx(grad_out.to(torch.bfloat16).contiguous(), ctx.state, wts.w1, wts.w3, wts.w2,
                                     inter=wts.inter, lora=lora,
                                     out_dtype=torch.float32 if ctx.token_dtype == torch.float32 else torch.bfloat16)
        ctx.state = None
        ga = gb = None
        if lora is not None and lora.compute_grads:
            ga = lora.grad_a.to(ctx.factor_dtypes[0])
            gb = lora.grad_b.to(ctx.factor_dtypes[1])
        return dx.to(ctx.token_dtype), dw.to(ctx.score_dtype), None, None, ga, gb, None


def run_routed(weights: GroupedExpertWeights, tokens: torch.Tensor, top_scores: torch.Tensor,
               top_indices: torch.Tensor, lora: tuple | None = None) -> torch.Tensor:
    """``run_direct_routed`` semantics on bound weights (experts.py:1749-1912).

    ``lora`` = (lora_a [E, r, I], lora_b [E, H, r], scale) adds a LoRA adapter
    on the down projection (active_expert_lora.py:434-478); gradients flow to
    both factors."""
    if top_scores.shape != top_indices.shape or top_indices.ndim != 2:
        raise ValueError("Direct routed execution requires matching [tokens, top_k] score and index tensors.")
    if int(top_indices.shape[0]) != int(tokens.shape[0]):
        raise ValueError("Direct routed expert indices do not match token count.")
    if not tokens.is_cuda:
        raise ValueError("the B200 expert path runs on CUDA tensors only (no CPU fallback)")
    la, lb, sc = lora if lora is not None else (None, None, 1.0)
    return _RoutedExpertsFunction.apply(tokens, top_scores, top_indices.to(torch.int64), weights, la, lb, sc)


def down_lora_of(experts: Any) -> tuple | None:
    """(lora_a, lora_b, scale) of a plain ActiveExpertLoRA on ``w2``, or None.

    The scale is the adapter's ``lora_scale(alpha, rank, rslora) * lora_scale *
    rank_schedule_scale`` (active_expert_lora.py:461-466, lora_allocation.py:163-168).
    Raises for adapters on other keys or with features the fused path does not
    run (rank / parameter dropout in training, expert selection, timestep or
    route gates, condenser)."""
    adapters = getattr(experts, "expert_lora", None)
    if adapters is None or len(adapters) == 0:
        return None
    keys = list(adapters.keys())
    if keys != ["w2"]:
        raise ops._lib.MiraiError(2, f"expert LoRA on {keys}: the fused path supports an adapter on w2 only")
    ad = adapters["w2"]
    training = bool(getattr(ad, "training", False))
    unsupported = []
    if training and float(getattr(ad, "_rank_dropout", 0.0)) > 0.0:
        unsupported.append("rank dropout")
    if training and float(getattr(ad, "_lora_parameter_dropout", 0.0)) > 0.0:
        unsupported.append("parameter dropout")
    if bool(getattr(ad, "_expert_selection_active", False)):
        unsupported.append("expert selection mask")
    if getattr(ad, "_timestep_mask_uniform", None) is not None or getattr(ad, "_tc_gate_hypernet", None) is not None:
        unsupported.append("timestep / TC gate")
    cond = getattr(ad, "_condenser", None)
    if cond is not None and callable(getattr(cond, "delta", None)):
        probe = getattr(cond, "enabled", None)
        if probe is True:
            unsupported.append("condenser")
    if unsupported:
        raise ops._lib.MiraiError(2, "expert LoRA features not fused: " + ", ".join(unsupported))
    if not all(hasattr(ad, n) for n in ("rank", "lora_a", "lora_b")):
        raise ops._lib.MiraiError(2, f"expert LoRA adapter {type(ad).__name__} on w2 is not an ActiveExpertLoRA")
    rank = int(ad.rank)
    alpha = float(ad._alpha()) if callable(getattr(ad, "_alpha", None)) else float(ad.lora_alpha)
    denom = rank ** 0.5 if bool(getattr(ad, "use_rslora", False)) else float(rank)
    scale = alpha / denom * float(getattr(ad, "_lora_scale", 1.0)) * float(getattr(ad, "_rank_schedule_scale", 1.0))
    return ad.lora_a, ad.lora_b, scale


class B200GroupedExperts(nn.Module):
    """Frozen grouped experts with the reference's ingest API, run on sm_100a."""

    def __init__(self, base: nn.Module | None = None, *, quant_format: str = "nf4",
                 nf4_blocksize: int = 64, expert_weight_access: str = "fused_kernel",
                 expert_dequant_chunk_size: int = 0, group_sizes=None, execution_spec=None):
        super().__init__()
        self._init_empty(int(getattr(base, "num_experts", 0)) if base is not None else 0, quant_format,
                         nf4_blocksize, expert_weight_access, expert_dequant_chunk_size)
        if base is not None:
            for key in ("w1", "w2", "w3"):
                self.load_dense_weight(key, getattr(base, key))

    @classmethod
    def from_empty(cls, *, num_experts: int, quant_format: str = "nf4", nf4_blocksize: int = 64,
                   expert_weight_access: str = "fused_kernel", expert_dequant_chunk_size: int = 0,
                   group_sizes=None, execution_spec=None) -> "B200GroupedExperts":
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m._init_empty(num_experts, quant_format, nf4_blocksize, expert_weight_access, expert_dequant_chunk_size)
        return m

    def _init_empty(self, num_experts, quant_format, nf4_blocksize, access, chunk):
        fmt = str(quant_format or "nf4").lower()
        if fmt not in ("nf4", "int8", "bf16"):
            raise ValueError("B200 grouped experts support quant_format 'nf4', 'int8' or 'bf16'.")
        self.num_experts = int(num_experts)
        self._quant_format = fmt
        self._nf4_blocksize = int(nf4_blocksize)
        self._nf4_meta: Nf4Meta | None = None
        self._nf4_shapes: dict[str, tuple[int, ...]] = {}
        self.expert_weight_access = access
        self.expert_dequant_chunk_size = int(chunk)
        self._loaded: set[str] = set()
        self._bound: GroupedExpertWeights | None = None
        self.expert_lora = nn.ModuleDict()

    # ------------------------------------------------------------------ ingest
    def _set_buffer(self, name: str, value: torch.Tensor) -> None:
        if name in self._buffers:
            self._buffers[name] = value
        else:
            self.register_buffer(name, value)
        self._bound = None

    def load_dense_weight(self, key: str, source: torch.Tensor, *, rotation=None) -> None:
        """Quantise one [E, out, in] tensor on the GPU (experts.py:940-996)."""
        if key not in ("w1", "w2", "w3"):
            raise ValueError(f"Unknown grouped expert tensor '{key}'.")
        if source.ndim != 3 or int(source.shape[0]) != self.num_experts:
            raise ValueError(f"grouped expert tensor {key} must be [E={self.num_experts}, out, in], "
                             f"got {tuple(source.shape)}")
        if rotation is not None:
            raise ValueError("Learned expert rotations are not supported by the fused kernels.")
        src = source.detach()
        if not src.is_cuda:
            raise ValueError("load_dense_weight needs the source on a CUDA device (quantisation runs on the GPU)")
        if self._quant_format == "nf4":
            dev = src.device
            t = ops.nf4_quantize(src, tables.nf4_code(dev), tables.dynamic_map(dev), blocksize=self._nf4_blocksize)
            self._nf4_meta = Nf4Meta(t.blocksize, t.nested_blocksize)
            self._nf4_shapes[key] = tuple(src.shape)
            self._set_buffer(f"{key}_nf4", t.packed)
            self._set_buffer(f"{key}_nf4_absmax", t.absmax)
            self._set_buffer(f"{key}_nf4_nabsmax", t.nested_absmax)
            self._set_buffer(f"{key}_nf4_offset", t.offset)
            self._set_buffer(f"{key}_nf4_code", t.code)
            self._set_buffer(f"{key}_nf4_ncode", t.nested_code)
        elif self._quant_format == "int8":
            t = ops.int8_quantize(src.float() if src.dtype not in (torch.float32, torch.bfloat16) else src)
            self._set_buffer(f"{key}_int8", t.q)
            self._set_buffer(f"{key}_scale", t.scale)
            setattr(self, f"{key}_group_size", 0)
        else:
            self._set_buffer(key, src.to(torch.bfloat16).contiguous())
        self._loaded.add(key)

    def load_nf4_packed_weight(self, key: str, *, packed, absmax, nested_absmax, offset, code, nested_code,
                               shape: Iterable[int], meta) -> None:
        """Restore one NF4 key from packed buffers (experts.py:1424-1470)."""
        if self._quant_format != "nf4":
            raise ValueError("NF4 packed state requires an NF4 grouped-expert wrapper.")
        shape = tuple(int(d) for d in shape)
        if len(shape) != 3 or shape[0] != self.num_experts:
            raise ValueError(f"NF4 grouped expert tensor {key} has invalid dense shape {shape}.")
        for name, t in {"packed": packed, "absmax": absmax, "nested_absmax": nested_absmax,
                        "offset": offset}.items():
            if t.ndim == 0 or int(t.shape[0]) != self.num_experts:
                raise ValueError(f"NF4 grouped expert {key} {name} must have expert axis {self.num_experts}, "
                                 f"got {tuple(t.shape)}.")
        m = Nf4Meta(int(meta.blocksize), int(meta.nested_blocksize))
        if self._nf4_meta is not None and (self._nf4_meta.blocksize, self._nf4_meta.nested_blocksize) != (
                m.blocksize, m.nested_blocksize):
            raise ValueError("NF4 grouped expert tensors use inconsistent quantization metadata.")
        self._nf4_meta = m
        self._nf4_shapes[key] = shape
        self._set_buffer(f"{key}_nf4", packed.detach().contiguous())
        self._set_buffer(f"{key}_nf4_absmax", absmax.detach().contiguous())
        self._set_buffer(f"{key}_nf4_nabsmax", nested_absmax.detach().contiguous())
        self._set_buffer(f"{key}_nf4_offset", offset.detach().contiguous())
        self._set_buffer(f"{key}_nf4_code", code.detach().contiguous())
        self._set_buffer(f"{key}_nf4_ncode", nested_code.detach().contiguous())
        self._loaded.add(key)

    def load_quantized_weight(self, key: str, *, weight_int8, weight_scale, group_size: int, rotation=None) -> None:
        """Restore one INT8 key (experts.py:1382-1422); only group_size 0 is executable."""
        if weight_int8.ndim != 3 or int(weight_int8.shape[0]) != self.num_experts:
            raise ValueError(f"grouped expert tensor {key} must be 3D with {self.num_experts} experts.")
        if tuple(weight_scale.shape) != (*tuple(weight_int8.shape[:-1]), 1):
            raise ValueError(f"grouped expert scale {key} has shape {tuple(weight_scale.shape)}.")
        if int(group_size) != 0 or rotation is not None:
            raise ValueError("the fused INT8 kernels read per-output-channel INT8 (group_size=0, no rotation)")
        self._quant_format = "int8"
        self._set_buffer(f"{key}_int8", weight_int8.detach().to(torch.int8).contiguous())
        self._set_buffer(f"{key}_scale", weight_scale.detach().float().contiguous())
        setattr(self, f"{key}_group_size", 0)
        self._loaded.add(key)

    def is_fully_loaded(self) -> bool:
        return self._loaded.issuperset({"w1", "w2", "w3"})

    def expert_rotation(self, key: str):
        return None

    # ------------------------------------------------------------------ execution
    def bound_weights(self) -> GroupedExpertWeights:
        if not self.is_fully_loaded():
            raise RuntimeError("grouped experts are not fully loaded (need w1, w2, w3)")
        if self._bound is None:
            self._bound = GroupedExpertWeights.from_module(self)
        return self._bound

    def _apply(self, fn, recurse=True):  # .to(device) / block swap re-binds buffers
        self._bound = None
        return super()._apply(fn, recurse)

    def prefers_for_loop(self) -> bool:
        return True

    def attach_expert_lora(self, *, tensor_name: str, adapter_name: str = "lora", rank: int, alpha: float,
                           init: str = "kaiming", use_rslora: bool = False) -> None:
        """A LoRA adapter on the down projection: lora_a [E, r, I] (kaiming-uniform),
        lora_b [E, H, r] zeros, scale alpha / rank (or / sqrt(rank) for rsLoRA)."""
        if tensor_name != "w2":
            raise ValueError("the fused path supports an expert LoRA adapter on w2 only")
        if not hasattr(self, "expert_lora"):
            self.expert_lora = nn.ModuleDict()
        _, H, I = self._shape_of("w2")
        self.expert_lora["w2"] = _DownAdapter(self.num_experts, I, H, rank, alpha, use_rslora)

    def _shape_of(self, key: str) -> tuple[int, int, int]:
        if key in self._nf4_shapes:
            return self._nf4_shapes[key]
        for name in (f"{key}_int8", key):
            t = self._buffers.get(name)
            if t is not None:
                return tuple(t.shape)
        raise RuntimeError(f"{key} is not loaded")

    def run_direct_routed(self, tokens: torch.Tensor, top_scores: torch.Tensor,
                          top_indices: torch.Tensor) -> torch.Tensor:
        return run_routed(self.bound_weights(), tokens, top_scores, top_indices, lora=down_lora_of(self))


class _DownAdapter(nn.Module):
    """Minimal expert LoRA on w2 with the reference adapter's parameter names."""

    def __init__(self, num_experts: int, in_features: int, out_features: int, rank: int, alpha: float,
                 use_rslora: bool):
        super().__init__()
        self.rank = int(rank)
        self.use_rslora = bool(use_rslora)
        self.lora_a = nn.Parameter(torch.empty(num_experts, self.rank, in_features))
        self.lora_b = nn.Parameter(torch.zeros(num_experts, out_features, self.rank))
        self.register_buffer("lora_alpha", torch.tensor(float(alpha)), persistent=True)
        for e in range(num_experts):
            nn.init.kaiming_uniform_(self.lora_a.data[e], a=5 ** 0.5)

    def _alpha(self) -> float:
        return float(self.lora_alpha.item())
