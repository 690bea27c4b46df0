"""Routed frozen experts executed by libmirai_b200 (the drop-in for the
reference's compressed grouped-expert layer).

``GroupedExpertWeights`` binds the three expert tensors of one MoE layer
(gate ``w1`` [E, I, H], up ``w3`` [E, I, H], down ``w2`` [E, H, I], the
reference's layout, transformer_lingbot_video.py:1143-1145) in one of three
storage formats, reading the reference's own buffers in place:

* NF4: ``{key}_nf4``, ``{key}_nf4_absmax``, ``{key}_nf4_nabsmax``,
  ``{key}_nf4_offset``, ``{key}_nf4_code``, ``{key}_nf4_ncode`` and the
  ``_Nf4Meta`` block sizes (experts.py:998-1031, 1424-1470);
* INT8: ``{key}_int8`` and ``{key}_scale`` with ``{key}_group_size`` 0
  (plain per-output-channel) or a power of 4 (block-Hadamard rotated,
  quant.py:103-122, 189-260; experts.py:1382-1422);
* bf16 dense tensors (the LingBot dense grouped experts).

``B200GroupedExperts`` is an ``nn.Module`` with the reference's construction
and ingest API (``from_empty``, ``load_dense_weight``,
``load_nf4_packed_weight``, ``load_quantized_weight``, and the packed-state
manifest entry of packed_state.py:441-449 through ``from_packed_state``) and
its direct-routed entry point ``run_direct_routed(tokens, top_scores,
top_indices)`` (experts.py:1749-1912), differentiable in ``tokens`` and
``top_scores`` (the dX path through frozen experts; no dense weight is kept
for backward, the invariant of linear.py:96-102).

Ingest is described by one table, ``STORAGE``: for every format the buffers
one weight key owns, their dtypes and their sizes as functions of the
key's dense ``[E, out, in]`` shape.  Every loader (dense quantisation, NF4
packed buffers, INT8 buffers, packed-state artifacts) checks its tensors
against that table and reports every mismatch at once.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable, Iterable, Mapping

import torch
import torch.nn as nn

from . import ops, tables

KEYS = ("w1", "w3", "w2")  # gate, up, down (specs.py:129-230 canonical roles)
DEFAULT_GROUP_SIZES = (256, 64, 16)  # quant.py:22


@dataclass
class Nf4Meta:
    """Static NF4 metadata (quant.py:305-312 ``_Nf4Meta``)."""

    blocksize: int = 64
    nested_blocksize: int = 256
    nested_dtype: torch.dtype = torch.float32
    weight_dtype: torch.dtype = torch.bfloat16


def best_group_size(in_features: int, group_sizes: Iterable[int] = DEFAULT_GROUP_SIZES) -> int:
    """Largest configured rotation group dividing ``in_features``, else 0 (quant.py:87-91)."""
    fits = [int(g) for g in group_sizes if int(g) > 0 and int(in_features) % int(g) == 0]
    return max(fits) if fits else 0


def _is_power_of_four(g: int) -> bool:
    return g >= 4 and (g & (g - 1)) == 0 and (g.bit_length() - 1) % 2 == 0


# ----------------------------------------------------------------------------- storage table

@dataclass(frozen=True)
class BufferSlot:
    """One buffer a weight key owns: ``{key}_{suffix}``.

    ``per_expert(out, in, meta)`` is its element count per expert (the tensor
    is ``[E, ...]``); ``fixed`` is the element count of a shared table (no
    expert axis).  Exactly one of the two is set."""

    suffix: str
    dtype: torch.dtype
    per_expert: Callable[[int, int, Any], int] | None = None
    fixed: int | None = None


STORAGE: dict[str, tuple[BufferSlot, ...]] = {
    "nf4": (
        BufferSlot("nf4", torch.uint8, per_expert=lambda o, i, m: o * i // 2),
        BufferSlot("nf4_absmax", torch.uint8, per_expert=lambda o, i, m: o * i // m.blocksize),
        BufferSlot("nf4_nabsmax", torch.float32,
                   per_expert=lambda o, i, m: -(-(o * i // m.blocksize) // m.nested_blocksize)),
        BufferSlot("nf4_offset", torch.float32, per_expert=lambda o, i, m: 1),
        BufferSlot("nf4_code", torch.float32, fixed=16),
        BufferSlot("nf4_ncode", torch.float32, fixed=256),
    ),
    "int8": (
        BufferSlot("int8", torch.int8, per_expert=lambda o, i, m: o * i),
        BufferSlot("scale", torch.float32, per_expert=lambda o, i, m: o),
    ),
}


def storage_problems(fmt: str, key: str, num_experts: int, dense_shape: tuple[int, ...], meta: Any,
                     tensors: Mapping[str, torch.Tensor]) -> list[str]:
    """Every way ``tensors`` (suffix -> tensor) fails the ``STORAGE[fmt]`` entry
    for one key of dense shape ``[E, out, in]``; empty when they fit."""
    problems = []
    if len(dense_shape) != 3 or dense_shape[0] != num_experts:
        return [f"{key}: dense shape {tuple(dense_shape)} is not [{num_experts}, out, in]"]
    _, out_f, in_f = dense_shape
    if fmt == "nf4" and (in_f * out_f) % meta.blocksize:
        problems.append(f"{key}: {out_f}x{in_f} elements are not whole blocks of {meta.blocksize}")
    for slot in STORAGE[fmt]:
        name = f"{key}_{slot.suffix}"
        t = tensors.get(slot.suffix)
        if not isinstance(t, torch.Tensor):
            problems.append(f"{name}: missing")
            continue
        if t.dtype != slot.dtype:
            problems.append(f"{name}: dtype {t.dtype}, the layout stores {slot.dtype}")
        if slot.fixed is not None:
            if t.numel() != slot.fixed:
                problems.append(f"{name}: {t.numel()} entries, the table has {slot.fixed}")
            continue
        want = slot.per_expert(out_f, in_f, meta)
        if t.ndim == 0 or int(t.shape[0]) != num_experts:
            problems.append(f"{name}: leading axis of {tuple(t.shape)} is not the {num_experts} experts")
        elif t.numel() != num_experts * want:
            problems.append(f"{name}: {t.numel() // max(num_experts, 1)} entries per expert, "
                            f"{out_f}x{in_f} needs {want}")
    return problems


def _require(problems: list[str], what: str) -> None:
    if problems:
        raise ValueError(f"{what} rejected: " + "; ".join(problems))


class GroupedExpertWeights:
    """The three weight keys of one layer as kernel descriptors.

    ``rot_in`` / ``rot_mid``: block-Hadamard group sizes of the rotated INT8
    format along the hidden (w1/w3 input) and intermediate (w2 input)
    dimensions, 0 when not rotated."""

    def __init__(self, fmt: str, w1, w3, w2, num_experts: int, hidden: int, inter: int, *,
                 rot_in: int = 0, rot_mid: int = 0):
        self.fmt = fmt
        self.w1, self.w3, self.w2 = w1, w3, w2
        self.num_experts, self.hidden, self.inter = int(num_experts), int(hidden), int(inter)
        self.rot_in, self.rot_mid = int(rot_in), int(rot_mid)

    @classmethod
    def from_module(cls, module: Any) -> "GroupedExpertWeights":
        """Bind the buffers of a reference-compatible grouped-expert module.

        Accepts the reference's ``CompressedGroupedExperts`` (NF4, or INT8
        plain or with its fixed block-Hadamard rotation), this package's
        ``B200GroupedExperts`` and dense modules exposing ``w1``/``w2``/``w3``
        tensors.  The buffers are used in place (no copy); they must live on a
        CUDA device.
        """
        fmt = str(getattr(module, "_quant_format", "")).lower()
        E = int(getattr(module, "num_experts"))
        if fmt == "nf4":
            shapes = getattr(module, "_nf4_shapes")
            meta = getattr(module, "_nf4_meta")
            ws = {}
            for key in KEYS:
                buf = {s.suffix: getattr(module, f"{key}_{s.suffix}", None) for s in STORAGE["nf4"]}
                buf["nf4_offset"] = None if buf["nf4_offset"] is None else buf["nf4_offset"].reshape(E, 1)
                problems = storage_problems("nf4", key, E, tuple(shapes.get(key, ())), meta, buf)
                if problems:
                    raise ops._lib.MiraiError(2, "NF4 expert buffers do not fit the kernel layout: "
                                              + "; ".join(problems))
                ws[key] = ops.NF4Tensor(buf["nf4"], buf["nf4_absmax"], buf["nf4_nabsmax"], buf["nf4_offset"],
                                        buf["nf4_code"], buf["nf4_ncode"], shapes[key], int(meta.blocksize),
                                        int(meta.nested_blocksize))
            _, inter, hidden = shapes["w1"]
            return cls("nf4", ws["w1"], ws["w3"], ws["w2"], E, hidden, inter)
        if fmt == "int8" and hasattr(module, "w1_int8"):
            groups = {}
            learned = getattr(module, "expert_rotation", None)
            for key in KEYS:
                g = int(getattr(module, f"{key}_group_size", 0))
                if callable(learned) and learned(key) is not None:
                    raise ops._lib.MiraiError(2, f"INT8 expert tensor {key} carries a learned rotation matrix; "
                                                 "the fused path applies the fixed block-Hadamard rotation only")
                if g and not _is_power_of_four(g):
                    raise ops._lib.MiraiError(2, f"INT8 expert tensor {key}: rotation group {g} is not a power "
                                                 "of 4")
                groups[key] = g
            if groups["w1"] != groups["w3"]:
                raise ops._lib.MiraiError(2, f"INT8 gate/up rotation groups differ ({groups['w1']} vs "
                                             f"{groups['w3']}): one activation rotation feeds both")
            ws = {key: ops.Int8Tensor(getattr(module, f"{key}_int8"), getattr(module, f"{key}_scale"),
                                      group_size=groups[key]) for key in KEYS}
            _, inter, hidden = ws["w1"].shape
            return cls("int8", ws["w1"], ws["w3"], ws["w2"], E, hidden, inter,
                       rot_in=groups["w1"], rot_mid=groups["w2"])
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
            out = ops.moe_forward(x, top_indices.contiguous(), w, weights.w1, weights.w3, weights.w2,
                                  num_experts=weights.num_experts, inter=weights.inter, lora=lora,
                                  out_dtype=out_dtype)
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
    if top_indices.ndim != 2 or tuple(top_scores.shape) != tuple(top_indices.shape):
        raise ValueError(f"routed execution takes [tokens, top_k] scores and indices of one shape, got "
                         f"{tuple(top_scores.shape)} and {tuple(top_indices.shape)}")
    if tokens.ndim != 2 or tokens.shape[0] != top_indices.shape[0]:
        raise ValueError(f"{tuple(tokens.shape)} tokens against routing for {int(top_indices.shape[0])} tokens")
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


def _meta_from_spec(raw: Any) -> Nf4Meta:
    """``nf4_meta`` of a packed-state manifest entry (packed_contract.py:58-78)."""
    if not isinstance(raw, Mapping):
        raise ValueError("packed NF4 expert entry carries no nf4_meta mapping")

    def dtype(name, default):
        value = getattr(torch, str(name or "").replace("torch.", ""), None)
        return value if isinstance(value, torch.dtype) else default

    return Nf4Meta(int(raw.get("blocksize", 64)), int(raw.get("nested_blocksize", 256)),
                   dtype(raw.get("nested_dtype"), torch.float32), dtype(raw.get("weight_dtype"), torch.bfloat16))


class B200GroupedExperts(nn.Module):
    """Frozen grouped experts with the reference's ingest API, run on sm_100a."""

    def __init__(self, base: nn.Module | None = None, *, quant_format: str = "nf4",
                 nf4_blocksize: int = 64, expert_weight_access: str = "fused_kernel",
                 expert_dequant_chunk_size: int = 0, group_sizes=None, execution_spec=None):
        super().__init__()
        self._init_empty(int(getattr(base, "num_experts", 0)) if base is not None else 0, quant_format,
                         nf4_blocksize, expert_weight_access, expert_dequant_chunk_size, group_sizes)
        if base is not None:
            for key in ("w1", "w2", "w3"):
                self.load_dense_weight(key, getattr(base, key))

    @classmethod
    def from_empty(cls, *, num_experts: int, quant_format: str = "nf4", nf4_blocksize: int = 64,
                   expert_weight_access: str = "fused_kernel", expert_dequant_chunk_size: int = 0,
                   group_sizes=None, execution_spec=None) -> "B200GroupedExperts":
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m._init_empty(num_experts, quant_format, nf4_blocksize, expert_weight_access, expert_dequant_chunk_size,
                      group_sizes)
        return m

    @classmethod
    def from_packed_state(cls, spec: Mapping[str, Any], tensors: Mapping[str, torch.Tensor]) -> "B200GroupedExperts":
        """Experts restored from one ``grouped_experts`` entry of a packed-state
        manifest (packed_state.py:331-341, 441-449) and its tensor mapping
        (safetensors names -> tensors, e.g. ``layers.3.ffn.experts.w1_nf4``).

        NF4 and INT8 entries are read; ``spec["tensors"]`` maps each local
        buffer name (``w1_nf4``, ``w1_nf4_absmax``, ... or ``w1_int8``,
        ``w1_scale``) to its tensor key, ``spec["shapes"]`` gives each key's
        dense shape, ``spec["group_sizes"]`` the INT8 rotation groups and
        ``spec["nf4_meta"]`` the NF4 block sizes.  The tensors must already be
        on the CUDA device that will run the layer (they are used in place)."""
        if str(spec.get("kind")) != "grouped_experts":
            raise ValueError(f"packed entry of kind {spec.get('kind')!r} is not grouped_experts")
        fmt = str(spec.get("quant_format", "")).lower()
        if fmt not in STORAGE:
            raise ValueError(f"packed grouped experts in format {fmt!r}: the fused path reads nf4 and int8")
        if spec.get("rotations"):
            raise ValueError("packed grouped experts with learned rotations: the fused path applies the fixed "
                             "block-Hadamard rotation only")
        names = spec.get("tensors")
        shapes = spec.get("shapes")
        if not isinstance(names, Mapping) or not isinstance(shapes, Mapping):
            raise ValueError("packed grouped-experts entry needs 'tensors' and 'shapes' mappings")
        m = cls.from_empty(num_experts=int(spec["num_experts"]), quant_format=fmt)
        meta = _meta_from_spec(spec.get("nf4_meta")) if fmt == "nf4" else None
        groups = spec.get("group_sizes") or {}
        missing = [f"{key}_{s.suffix}" for key in ("w1", "w2", "w3") for s in STORAGE[fmt]
                   if str(names.get(f"{key}_{s.suffix}", "")) not in tensors]
        if missing:
            raise KeyError(f"packed grouped experts: tensors missing from the mapping: {missing}")
        for key in ("w1", "w2", "w3"):
            buf = {s.suffix: tensors[str(names[f"{key}_{s.suffix}"])] for s in STORAGE[fmt]}
            shape = tuple(int(v) for v in shapes[key])
            if fmt == "nf4":
                m.load_nf4_packed_weight(key, packed=buf["nf4"], absmax=buf["nf4_absmax"],
                                         nested_absmax=buf["nf4_nabsmax"], offset=buf["nf4_offset"],
                                         code=buf["nf4_code"], nested_code=buf["nf4_ncode"], shape=shape, meta=meta)
            else:
                m.load_quantized_weight(key, weight_int8=buf["int8"], weight_scale=buf["scale"],
                                        group_size=int(groups.get(key, 0)))
        return m

    def _init_empty(self, num_experts, quant_format, nf4_blocksize, access, chunk, group_sizes=None):
        fmt = str(quant_format or "nf4").lower()
        if fmt not in ("nf4", "int8", "bf16"):
            raise ValueError(f"quant_format {quant_format!r}: the B200 experts store nf4, int8 or bf16")
        self.num_experts = int(num_experts)
        self._quant_format = fmt
        self._nf4_blocksize = int(nf4_blocksize)
        self._nf4_meta: Nf4Meta | None = None
        self._nf4_shapes: dict[str, tuple[int, ...]] = {}
        self._group_sizes = tuple(int(g) for g in (group_sizes or DEFAULT_GROUP_SIZES))
        self.expert_weight_access = access
        self.expert_dequant_chunk_size = int(chunk)
        self._loaded: set[str] = set()
        self._bound: GroupedExpertWeights | None = None
        self.expert_lora = nn.ModuleDict()

    # ------------------------------------------------------------------ ingest
    def _install(self, key: str, fmt: str, buffers: Mapping[str, torch.Tensor]) -> None:
        """Register one key's buffers under the reference's names (``{key}_{suffix}``)."""
        for suffix, value in buffers.items():
            name = f"{key}_{suffix}" if suffix else key
            if name in self._buffers:
                self._buffers[name] = value
            else:
                self.register_buffer(name, value)
        self._loaded.add(key)
        self._bound = None

    def _check_key(self, key: str) -> None:
        if key not in ("w1", "w2", "w3"):
            raise ValueError(f"weight key {key!r}: grouped experts hold w1 (gate), w3 (up) and w2 (down)")

    def load_dense_weight(self, key: str, source: torch.Tensor, *, rotation=None) -> None:
        """Quantise one [E, out, in] tensor on the GPU (experts.py:940-996).

        INT8 uses the rotation group ``best_group_size(in)`` of the module's
        group sizes (quant.py:87-91, 189-235): rows are block-Hadamard rotated
        in fp32 before the per-row amax/127 scale (0 = no rotation)."""
        self._check_key(key)
        if source.ndim != 3 or int(source.shape[0]) != self.num_experts:
            raise ValueError(f"dense {key} of shape {tuple(source.shape)}: expected [{self.num_experts}, out, in]")
        if rotation is not None:
            raise ValueError("learned rotation matrices are not applied by the fused kernels")
        src = source.detach()
        if not src.is_cuda:
            raise ValueError("load_dense_weight quantises on the GPU: pass the source on a CUDA device")
        if self._quant_format == "nf4":
            dev = src.device
            t = ops.nf4_quantize(src, tables.nf4_code(dev), tables.dynamic_map(dev), blocksize=self._nf4_blocksize)
            self._nf4_meta = Nf4Meta(t.blocksize, t.nested_blocksize)
            self._nf4_shapes[key] = tuple(src.shape)
            self._install(key, "nf4", {"nf4": t.packed, "nf4_absmax": t.absmax, "nf4_nabsmax": t.nested_absmax,
                                       "nf4_offset": t.offset, "nf4_code": t.code, "nf4_ncode": t.nested_code})
        elif self._quant_format == "int8":
            g = best_group_size(int(src.shape[-1]), self._group_sizes)
            t = ops.int8_quantize(src.float() if src.dtype not in (torch.float32, torch.bfloat16) else src,
                                  group_size=g)
            self._install(key, "int8", {"int8": t.q, "scale": t.scale})
            setattr(self, f"{key}_group_size", g)
        else:
            self._install(key, "bf16", {"": src.to(torch.bfloat16).contiguous()})

    def load_nf4_packed_weight(self, key: str, *, packed, absmax, nested_absmax, offset, code, nested_code,
                               shape: Iterable[int], meta) -> None:
        """Restore one NF4 key from packed buffers (experts.py:1424-1470)."""
        self._check_key(key)
        if self._quant_format != "nf4":
            raise ValueError(f"NF4 buffers for {key} offered to {self._quant_format} experts")
        m = Nf4Meta(int(meta.blocksize), int(meta.nested_blocksize))
        if self._nf4_meta is not None and (self._nf4_meta.blocksize, self._nf4_meta.nested_blocksize) != (
                m.blocksize, m.nested_blocksize):
            raise ValueError(f"{key}: NF4 block sizes ({m.blocksize}, {m.nested_blocksize}) differ from the keys "
                             f"already loaded ({self._nf4_meta.blocksize}, {self._nf4_meta.nested_blocksize})")
        dense = tuple(int(d) for d in shape)
        buf = {"nf4": packed, "nf4_absmax": absmax, "nf4_nabsmax": nested_absmax,
               "nf4_offset": offset.reshape(offset.shape[0], -1) if offset.ndim else offset,
               "nf4_code": code, "nf4_ncode": nested_code}
        _require(storage_problems("nf4", key, self.num_experts, dense, m, buf), f"NF4 buffers for {key}")
        self._nf4_meta = m
        self._nf4_shapes[key] = dense
        self._install(key, "nf4", {"nf4": packed.detach().contiguous(), "nf4_absmax": absmax.detach().contiguous(),
                                   "nf4_nabsmax": nested_absmax.detach().contiguous(),
                                   "nf4_offset": offset.detach().reshape(-1).contiguous(),
                                   "nf4_code": code.detach().contiguous(),
                                   "nf4_ncode": nested_code.detach().contiguous()})

    def load_quantized_weight(self, key: str, *, weight_int8, weight_scale, group_size: int, rotation=None) -> None:
        """Restore one INT8 key (experts.py:1382-1422): group 0 is plain
        per-output-channel INT8, a power of 4 the fixed block-Hadamard rotation."""
        self._check_key(key)
        g = int(group_size)
        if rotation is not None:
            raise ValueError(f"{key}: learned rotation matrices are not applied by the fused kernels")
        if weight_int8.ndim != 3:
            raise ValueError(f"INT8 {key} of shape {tuple(weight_int8.shape)}: expected [E, out, in]")
        dense = tuple(int(d) for d in weight_int8.shape)
        problems = storage_problems("int8", key, self.num_experts, dense, None,
                                    {"int8": weight_int8.to(torch.int8), "scale": weight_scale.float()})
        if tuple(weight_scale.shape) != (*dense[:-1], 1):
            problems.append(f"{key}_scale: shape {tuple(weight_scale.shape)}, expected {(*dense[:-1], 1)}")
        if g and (not _is_power_of_four(g) or dense[-1] % g):
            problems.append(f"{key}: rotation group {g} is not a power of 4 dividing in_features {dense[-1]}")
        _require(problems, f"INT8 buffers for {key}")
        self._quant_format = "int8"
        self._install(key, "int8", {"int8": weight_int8.detach().to(torch.int8).contiguous(),
                                    "scale": weight_scale.detach().float().contiguous()})
        setattr(self, f"{key}_group_size", g)

    def is_fully_loaded(self) -> bool:
        return self._loaded.issuperset({"w1", "w2", "w3"})

    def expert_rotation(self, key: str):
        return None

    # ------------------------------------------------------------------ execution
    def bound_weights(self) -> GroupedExpertWeights:
        if not self.is_fully_loaded():
            raise RuntimeError(f"grouped experts are not fully loaded: have {sorted(self._loaded)}, need w1, w2, w3")
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
            nn.init.kaiming_uniform_(self.lora_a.data[e], a=math.sqrt(5))

    def _alpha(self) -> float:
        return float(self.lora_alpha.item())
