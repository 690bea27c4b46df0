"""Torch-facing wrappers of the sm_100a kernels (device memory + streams only).

PyTorch is used here for allocation, streams and dtypes; every computation
below is a call into ``libmirai_b200.so``.  Inputs must be CUDA tensors; there
is no CPU path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib

SCORE_FUNCS = {"softmax": 0, "sigmoid": 1}
NORM_MODES = {"none": 0, "clamp": 1, "eps": 2, "l1": 3}
LAYOUTS = {"out_in": 0, "in_out": 1}      # [G, out, in] (compressed experts) / [G, in, out] (MAGI-2)
ACTIVATIONS = {"swiglu": 0, "swiglu7": 1}
COMBINE_BF16_ACCUM = 2


def _ptr(t: torch.Tensor | None) -> _lib.c_vp:
    return _lib.c_vp(0 if t is None else t.data_ptr())


def _stream() -> _lib.c_vp:
    return _lib.c_vp(torch.cuda.current_stream().cuda_stream)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return t.contiguous()


def device_status() -> tuple[int, int]:
    """Synchronise the current stream and return (and clear) the device error word."""
    return _lib.device_status(torch.cuda.current_stream().cuda_stream)


def launch_count() -> int:
    """Kernels libmirai_b200 has enqueued since it was loaded (host-side count:
    every kernel an entry point launched, on any stream)."""
    return _lib.launch_count()


def check_device() -> None:
    code, info = device_status()
    if code:
        raise _lib.MiraiError(code, f"raised on the device at site {info}")


def set_gemm_sm_limit(max_sms: int) -> None:
    """Cap the SMs the persistent grouped GEMMs occupy (0 = all), process-wide,
    so that communication kernels on another stream can run beside them."""
    _lib.call("mirai_b200_set_gemm_sm_limit", int(max_sms))


# ----------------------------------------------------------------------------- a1

def route_topk(logits: torch.Tensor, top_k: int, *, score_func: str = "softmax",
               choice_bias: torch.Tensor | None = None, norm: str = "clamp",
               route_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 top-k routing (routers.py:241-249; transformer_lingbot_video.py:1002-1033).

    Returns (top_indices int64 [T, k], top_weights fp32 [T, k]); slots are in
    descending choice order, ties to the lower expert id.
    """
    logits = _cuda(logits, "logits", torch.float32)
    T, E = logits.shape
    bias = None if choice_bias is None else _cuda(choice_bias, "choice_bias", torch.float32)
    idx = torch.empty((T, top_k), dtype=torch.int64, device=logits.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=logits.device)
    if bias is not None and bias.ndim == 2:  # one bias row per T / rows tokens (per head)
        period = T // bias.shape[0] if bias.shape[0] else 0
        if period * bias.shape[0] != T:
            raise ValueError(f"{bias.shape[0]} bias rows do not split {T} tokens evenly")
        _lib.call("mirai_route_topk_rows", _ptr(logits), T, E, top_k, SCORE_FUNCS[score_func], _ptr(bias), period,
                  NORM_MODES[norm], float(route_scale), _ptr(idx), _ptr(w), _stream())
        return idx, w
    _lib.call("mirai_route_topk", _ptr(logits), T, E, top_k, SCORE_FUNCS[score_func], _ptr(bias),
              NORM_MODES[norm], float(route_scale), _ptr(idx), _ptr(w), _stream())
    return idx, w


# ----------------------------------------------------------------------------- a2

@dataclass(frozen=True)
class DispatchPlan:
    """Device-resident routing layout (dispatch_preprocess.py:22-40)."""

    counts: torch.Tensor                # [E] int64
    starts: torch.Tensor                # [E] int64
    offsets: torch.Tensor               # [E] int32 inclusive cumsum
    sort_positions: torch.Tensor        # [S] int64
    sorted_token_indices: torch.Tensor  # [S] int64
    inverse_order: torch.Tensor         # [S] int64
    total_slots: int
    top_k: int


def dispatch_plan(top_indices: torch.Tensor, num_experts: int,
                  workspace: torch.Tensor | None = None) -> DispatchPlan:
    top_indices = _cuda(top_indices, "top_indices", torch.int64)
    T, k = top_indices.shape
    S = T * k
    dev = top_indices.device
    counts = torch.empty(num_experts, dtype=torch.int64, device=dev)
    starts = torch.empty(num_experts, dtype=torch.int64, device=dev)
    offsets = torch.empty(num_experts, dtype=torch.int32, device=dev)
    sp = torch.empty(S, dtype=torch.int64, device=dev)
    st = torch.empty(S, dtype=torch.int64, device=dev)
    inv = torch.empty(S, dtype=torch.int64, device=dev)
    need = plan_workspace_bytes(T, k, num_experts)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    _lib.call("mirai_dispatch_plan", _ptr(top_indices), T, k, num_experts, _ptr(counts), _ptr(starts),
              _ptr(offsets), _ptr(sp), _ptr(st), _ptr(inv), _ptr(workspace),
              workspace.numel() * workspace.element_size(), _stream())
    return DispatchPlan(counts, starts, offsets, sp, st, inv, S, k)


def plan_workspace_bytes(num_tokens: int, top_k: int, num_experts: int) -> int:
    return int(_lib.load().mirai_dispatch_plan_workspace_bytes(num_tokens, top_k, num_experts))


# ----------------------------------------------------------------------------- a3

def permute_rows(tokens: torch.Tensor, sorted_token_indices: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    tokens = _cuda(tokens, "tokens", torch.bfloat16)
    idx = _cuda(sorted_token_indices, "sorted_token_indices", torch.int64)
    S = idx.numel()
    H = tokens.shape[1]
    if out is None:
        out = torch.empty((S, H), dtype=torch.bfloat16, device=tokens.device)
    _lib.call("mirai_permute_rows_bf16", _ptr(tokens), tokens.shape[0], _ptr(idx), S, H, _ptr(out), _stream())
    return out


# ----------------------------------------------------------------------------- weight descriptors

class NF4Tensor:
    """Device buffers of one NF4 grouped-expert key, in the reference's layout
    (experts.py:998-1031): ``packed`` uint8 [E, out*in/2(, 1)], ``absmax`` uint8
    [E, out*in/64], ``nested_absmax`` fp32 [E, n], ``offset`` fp32 [E],
    ``code`` fp32 [16], ``nested_code`` fp32 [256]."""

    def __init__(self, packed, absmax, nested_absmax, offset, code, nested_code, shape,
                 blocksize: int = 64, nested_blocksize: int = 256):
        self.packed = _cuda(packed, "packed", torch.uint8)
        self.absmax = _cuda(absmax, "absmax", torch.uint8)
        self.nested_absmax = _cuda(nested_absmax, "nested_absmax", torch.float32)
        self.offset = _cuda(offset.reshape(-1), "offset", torch.float32)
        self.code = _cuda(code, "code", torch.float32)
        self.nested_code = _cuda(nested_code, "nested_code", torch.float32)
        self.shape = tuple(int(s) for s in shape)
        self.blocksize = int(blocksize)
        self.nested_blocksize = int(nested_blocksize)
        self._struct = _lib.Nf4Weight(self.packed.data_ptr(), self.absmax.data_ptr(),
                                      self.nested_absmax.data_ptr(), self.offset.data_ptr(),
                                      self.code.data_ptr(), self.nested_code.data_ptr(),
                                      self.blocksize, self.nested_blocksize)

    def struct(self) -> _lib.Nf4Weight:
        return self._struct


class Int8Tensor:
    """Device buffers of one INT8 grouped-expert key: ``q`` int8 [E, out, in]
    and ``scale`` fp32 [E, out, 1] (experts.py:1382-1422).  ``group_size`` 0 is
    plain per-output-channel INT8 (q * s = W); a power of 4 is the reference's
    default block-Hadamard format (q * s = W H along groups of ``in``,
    quant.py:189-235), run by rotating activations (``rotate_rows``)."""

    def __init__(self, q, scale, group_size: int = 0):
        self.q = _cuda(q, "int8 weight", torch.int8)
        self.scale = _cuda(scale, "int8 scale", torch.float32)
        self.shape = tuple(int(s) for s in self.q.shape)
        self.group_size = int(group_size)
        if self.group_size and self.shape[-1] % self.group_size:
            raise ValueError(f"rotation group {self.group_size} does not divide in_features {self.shape[-1]}")
        self._struct = _lib.Int8Weight(self.q.data_ptr(), self.scale.data_ptr())

    def struct(self) -> _lib.Int8Weight:
        return self._struct


def nf4_quantize(weight: torch.Tensor, code: torch.Tensor, nested_code: torch.Tensor, *,
                 blocksize: int = 64, nested_blocksize: int = 256) -> NF4Tensor:
    """Quantise a [E, out, in] stack to NF4 on the GPU (experts.py:998-1031)."""
    w = _cuda(weight.to(torch.bfloat16), "weight")
    E, out_f, in_f = w.shape
    dev = w.device
    bpe = out_f * in_f // blocksize
    n_nested = -(-bpe // nested_blocksize)
    packed = torch.empty((E, out_f * in_f // 2, 1), dtype=torch.uint8, device=dev)
    absmax = torch.empty((E, bpe), dtype=torch.uint8, device=dev)
    nabs = torch.empty((E, n_nested), dtype=torch.float32, device=dev)
    offset = torch.empty((E,), dtype=torch.float32, device=dev)
    code = _cuda(code, "code", torch.float32)
    nested_code = _cuda(nested_code, "nested_code", torch.float32)
    need = int(_lib.load().mirai_nf4_quantize_workspace_bytes(E, out_f, in_f))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    _lib.call("mirai_nf4_quantize", _ptr(w), E, out_f, in_f, _ptr(code), _ptr(nested_code), blocksize,
              nested_blocksize, _ptr(packed), _ptr(absmax), _ptr(nabs), _ptr(offset), _ptr(ws), need, _stream())
    return NF4Tensor(packed, absmax, nabs, offset, code, nested_code, (E, out_f, in_f), blocksize, nested_blocksize)


def nf4_dequantize(w: NF4Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [E, out, in] of an NF4 key (quant.py:380-434), bit-identical to the
    values the grouped GEMMs decode in their main loops."""
    E, out_f, in_f = w.shape
    if out is None:
        out = torch.empty((E, out_f, in_f), dtype=torch.bfloat16, device=w.packed.device)
    _cuda(out, "out", torch.bfloat16)
    _lib.call("mirai_nf4_dequantize", _ptr(w.packed), _ptr(w.absmax), _ptr(w.nested_absmax), _ptr(w.offset),
              _ptr(w.code), _ptr(w.nested_code), E, out_f, in_f, w.blocksize, w.nested_blocksize, _ptr(out),
              _stream())
    return out


def int8_quantize(weight: torch.Tensor, group_size: int = 0) -> Int8Tensor:
    """Symmetric per-output-channel INT8 of a [E, out, in] stack (quant.py:189-235).

    ``group_size`` > 0 first rotates each row's groups of that many input
    features by the block-Hadamard matrix, in fp32 (the reference's default
    format); codes can differ from the reference's by one step where the
    rotated value lies on a rounding boundary (the rotation's fp32 sums are
    ordered differently from a matrix product)."""
    w = _cuda(weight, "weight")
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    *lead, in_f = w.shape
    rows = w.numel() // in_f
    if group_size:
        w = rotate_rows(w.float().reshape(rows, in_f), group_size, out_dtype=torch.float32).reshape(w.shape)
    q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    s = torch.empty((*lead, 1), dtype=torch.float32, device=w.device)
    _lib.call("mirai_int8_quantize_rows", _ptr(w), 1 if w.dtype == torch.float32 else 0, rows, in_f, _ptr(q),
              _ptr(s), _stream())
    return Int8Tensor(q, s, group_size)


_DTYPE_CODES = {torch.bfloat16: 0, torch.float32: 1}


def rotate_rows(x: torch.Tensor, group: int, *, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """x H along every ``group``-wide block of the last dimension (H the
    block-Hadamard matrix of quant.py:103-122; H = H^T = H^-1), computed in
    fp32; bf16 or fp32 in and out.  ``out`` may be ``x`` itself."""
    x = _cuda(x, "x")
    if x.dtype not in _DTYPE_CODES:
        raise TypeError(f"rotate_rows takes bf16 or fp32, got {x.dtype}")
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _lib.call("mirai_rotate_rows", _ptr(x), _DTYPE_CODES[x.dtype], rows, cols, int(group), _ptr(out),
              _DTYPE_CODES[out.dtype], _stream())
    return out


def swiglu_backward_rotated(dh_raw: torch.Tensor, gate_up: torch.Tensor, group: int) -> torch.Tensor:
    """grad_gate_up [S, 2I] = SwiGLU backward of the saved (gate, up) given
    dh = rotate(dh_raw): the down projection's input gradient in the rotated
    INT8 format (dh_raw = grad_y (q s) from ``down_dh``)."""
    dh_raw = _cuda(dh_raw, "dh", torch.bfloat16)
    gate_up = _cuda(gate_up, "gate_up", torch.bfloat16)
    S, I = dh_raw.shape
    dgu = torch.empty((S, 2 * I), dtype=torch.bfloat16, device=dh_raw.device)
    _lib.call("mirai_swiglu_backward_rotated", _ptr(dh_raw), _ptr(gate_up), S, I, int(group), _ptr(dgu), _stream())
    return dgu


def _group(w) -> int:
    return int(getattr(w, "group_size", 0) or 0)


def _as_weight(w):
    if isinstance(w, (NF4Tensor, Int8Tensor)):
        return w.struct()
    return w


# ----------------------------------------------------------------------------- a6 / a7

def gateup_swiglu(x_sorted: torch.Tensor, offsets: torch.Tensor, w1, w3, *, inter: int,
                  save_gate_up: bool = False, out: torch.Tensor | None = None, sources: int = 1):
    """h = silu(x W1^T) * (x W3^T) per expert segment.  ``w1``/``w3`` are bf16
    tensors [E, I, H], or ``Nf4Weight`` / ``Int8Weight`` descriptors.
    ``sources`` > 1: ``offsets`` ends ``sources * E`` source-major segments
    (segment s*E + e = source s's rows for expert e)."""
    w1, w3 = _as_weight(w1), _as_weight(w3)
    x_sorted = _cuda(x_sorted, "x_sorted", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, H = x_sorted.shape
    h = out if out is not None else torch.empty((S, inter), dtype=torch.bfloat16, device=x_sorted.device)
    gu = torch.empty((S, 2 * inter), dtype=torch.bfloat16, device=x_sorted.device) if save_gate_up else None
    if sources > 1:
        if offsets.numel() % sources:
            raise ValueError("source-major segments: offsets must be a multiple of sources")
        E = offsets.numel() // sources
        _lib.call(f"mirai_moe_gateup_swiglu_src_{_fmt_suffix(w1)}", _ptr(x_sorted), _ptr(offsets), sources, E, S, H,
                  inter, _wptr(w1), _wptr(w3), _ptr(h), _ptr(gu), _stream())
        return (h, gu) if save_gate_up else h
    E = offsets.numel()
    if isinstance(w1, torch.Tensor):
        w1 = _cuda(w1, "w1", torch.bfloat16)
        w3 = _cuda(w3, "w3", torch.bfloat16)
        _lib.call("mirai_moe_gateup_swiglu_bf16", _ptr(x_sorted), _ptr(offsets), E, S, H, inter, _ptr(w1),
                  _ptr(w3), _ptr(h), _ptr(gu), _stream())
    elif isinstance(w1, _lib.Nf4Weight):
        _lib.call("mirai_moe_gateup_swiglu_nf4", _ptr(x_sorted), _ptr(offsets), E, S, H, inter, w1, w3, _ptr(h),
                  _ptr(gu), _stream())
    elif isinstance(w1, _lib.Int8Weight):
        _lib.call("mirai_moe_gateup_swiglu_int8", _ptr(x_sorted), _ptr(offsets), E, S, H, inter, w1, w3, _ptr(h),
                  _ptr(gu), _stream())
    else:
        raise TypeError(f"unsupported weight type {type(w1)}")
    return (h, gu) if save_gate_up else h


def down(h: torch.Tensor, offsets: torch.Tensor, w2, *, hidden: int, out: torch.Tensor | None = None,
         lora: "DownLoRA | None" = None, rank_a: torch.Tensor | None = None, sources: int = 1):
    """y = h W2^T per expert segment (+ the fused LoRA rank block when ``lora``;
    ``rank_a`` is its [S, 64] projection of h when the caller already has it).
    ``sources`` > 1: source-major segments as in ``gateup_swiglu``."""
    w2 = _as_weight(w2)
    h = _cuda(h, "h", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, I = h.shape
    y = out if out is not None else torch.empty((S, hidden), dtype=torch.bfloat16, device=h.device)
    if sources > 1:
        if offsets.numel() % sources:
            raise ValueError("source-major segments: offsets must be a multiple of sources")
        E = offsets.numel() // sources
        if lora is None:
            _lib.call(f"mirai_moe_down_src_{_fmt_suffix(w2)}", _ptr(h), _ptr(offsets), sources, E, S, I, hidden,
                      _wptr(w2), _ptr(y), _stream())
            return y
        low = rank_a if rank_a is not None else lora_project(h, offsets, lora, forward=True, sources=sources)
        _lib.call(f"mirai_moe_down_lora_src_{_fmt_suffix(w2)}", _ptr(h), _ptr(offsets), sources, E, S, I, hidden,
                  _wptr(w2), _ptr(low), _ptr(lora.b_pad()), _ptr(y), _stream())
        return y
    E = offsets.numel()
    if lora is None:
        _lib.call(f"mirai_moe_down_{_fmt_suffix(w2)}", _ptr(h), _ptr(offsets), E, S, I, hidden, _wptr(w2), _ptr(y),
                  _stream())
        return y
    low = rank_a if rank_a is not None else lora_project(h, offsets, lora, forward=True)
    _lib.call(f"mirai_moe_down_lora_{_fmt_suffix(w2)}", _ptr(h), _ptr(offsets), E, S, I, hidden, _wptr(w2),
              _ptr(low), _ptr(lora.b_pad()), _ptr(y), _stream())
    return y


_PAD_ATTR = "_mirai_lora_pads"


def _factor_pads(src: torch.Tensor) -> dict:
    """The padded kernel operands built from one adapter factor, kept on the
    factor tensor itself (the caller's parameter) so that they are built once
    per binding and rebuilt only when the factor changes: a moved version
    counter (an in-place optimizer step) or new storage drops them."""
    tag = (src._version, src.data_ptr())
    held = getattr(src, _PAD_ATTR, None)
    if held is None or held[0] != tag:
        held = (tag, {})
        try:
            setattr(src, _PAD_ATTR, held)
        except (AttributeError, RuntimeError):
            pass  # a tensor that takes no attributes gets pads for this call only
    return held[1]


class DownLoRA:
    """A LoRA adapter on the expert down projection (w2): y += scale (h A^T) B^T
    with A [E, r, I] and B [E, H, r] (active_expert_lora.py:43-116, 434-478)."""

    def __init__(self, a: torch.Tensor, b: torch.Tensor, scale: float, *, compute_grads: bool = False):
        self._src_a, self._src_b = a, b
        self.a = _cuda(a.detach().to(torch.bfloat16), "lora_a")
        self.b = _cuda(b.detach().to(torch.bfloat16), "lora_b")
        # when set, moe_backward_dx also fills grad_a [E, r, I] / grad_b [E, H, r] (fp32)
        self.compute_grads = bool(compute_grads)
        self.grad_a: torch.Tensor | None = None
        self.grad_b: torch.Tensor | None = None
        E, r, I = self.a.shape
        if tuple(self.b.shape[::2]) != (E, r) or r > 32:
            raise ValueError(f"LoRA factors must be A [E, r, I] and B [E, H, r] with r <= 32, got "
                             f"{tuple(self.a.shape)} and {tuple(self.b.shape)}")
        self.rank = int(r)
        self.scale = float(scale)

    def b_pad(self) -> torch.Tensor:
        """B zero-padded to [E*H, 64]: the K-major rank-block operand of the
        down GEMM.  Built once per value of the factor."""
        pads = _factor_pads(self._src_b)
        if "b" not in pads:
            E, H, r = self.b.shape
            pad = torch.zeros((E, H, 64), dtype=torch.bfloat16, device=self.b.device)
            pad[:, :, :r] = self.b
            pads["b"] = pad.reshape(E * H, 64)
        return pads["b"]

    def a_pad(self, rotation: int = 0) -> torch.Tensor:
        """A zero-padded to [E*64, I]: the MN-major rank-block operand of the
        down dX GEMM; with ``rotation`` > 0 each row rotated by the
        block-Hadamard matrix of that group size (A H), for the rotated INT8
        format whose dh is rotated after the GEMM (H H = 1).  Built once per
        value of the factor and group."""
        pads = _factor_pads(self._src_a)
        key = ("a", int(rotation))
        if key not in pads:
            E, r, I = self.a.shape
            pad = torch.zeros((E, 64, I), dtype=torch.bfloat16, device=self.a.device)
            pad[:, :r, :] = self.a
            pad = pad.reshape(E * 64, I)
            if rotation:
                pad = rotate_rows(pad, rotation)
            pads[key] = pad
        return pads[key]


LORA_FACTOR_ROWS, LORA_FACTOR_COLS = 0, 1


def lora_project(x: torch.Tensor, offsets: torch.Tensor, lora: DownLoRA, *, forward: bool,
                 sources: int = 1) -> torch.Tensor:
    """[S, 64] bf16 rank-block operand bf16(scale * x F_e^T), zero past the rank:
    F = A ([E, r, I], x = h) when ``forward``, else B^T ([E, H, r], x = grad_y).
    ``sources`` > 1: source-major segments (offsets [sources * E])."""
    x = _cuda(x, "x", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, K = x.shape
    out = torch.empty((S, 64), dtype=torch.bfloat16, device=x.device)
    factor, layout = (lora.a_pad(), LORA_FACTOR_ROWS) if forward else (lora.b_pad(), LORA_FACTOR_COLS)
    if offsets.numel() % sources:
        raise ValueError("source-major segments: offsets must be a multiple of sources")
    _lib.call("mirai_moe_lora_project_src", _ptr(x), _ptr(offsets), int(sources), offsets.numel() // sources, S, K,
              _ptr(factor), layout, int(lora.rank), float(lora.scale), _ptr(out), _stream())
    return out


# ----------------------------------------------------------------------------- a8

def combine(y_sorted: torch.Tensor, inverse_order: torch.Tensor, top_weights: torch.Tensor | None,
            out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None,
            top_k: int | None = None, bf16_accumulate: bool = False) -> torch.Tensor:
    """Weighted un-permute; ``top_weights=None`` sums the routes (permute backward).
    ``bf16_accumulate``: bf16 products summed in bf16, route by route (MAGI-2's
    index_add on bf16 tensors) instead of one fp32 sum."""
    y_sorted = _cuda(y_sorted, "y_sorted", torch.bfloat16)
    inv = _cuda(inverse_order, "inverse_order", torch.int64)
    if top_weights is None:
        k = int(top_k)
        T = inv.numel() // k
        w = None
    else:
        w = _cuda(top_weights.float(), "top_weights", torch.float32)
        T, k = w.shape
    H = y_sorted.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=out_dtype, device=y_sorted.device)
    code = {torch.bfloat16: 0, torch.float32: 1}[out.dtype]
    if bf16_accumulate:
        if out.dtype != torch.bfloat16:
            raise TypeError("bf16 accumulation writes a bf16 output")
        code = COMBINE_BF16_ACCUM
    _lib.call("mirai_moe_combine", _ptr(y_sorted), _ptr(inv), _ptr(w), T, k, H, _ptr(out), code, _stream())
    return out


def combine_backward(grad_out: torch.Tensor, y_sorted: torch.Tensor, inverse_order: torch.Tensor,
                     top_weights: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(grad_y_sorted bf16 [S, H], grad_weights fp32 [T, k]) (dispatch_ops.py:36-44)."""
    g = _cuda(grad_out.to(torch.bfloat16), "grad_out", torch.bfloat16)
    y_sorted = _cuda(y_sorted, "y_sorted", torch.bfloat16)
    inv = _cuda(inverse_order, "inverse_order", torch.int64)
    w = _cuda(top_weights.float(), "top_weights", torch.float32)
    T, k = w.shape
    H = y_sorted.shape[1]
    gy = torch.empty_like(y_sorted)
    gw = torch.empty((T, k), dtype=torch.float32, device=y_sorted.device)
    _lib.call("mirai_moe_combine_backward", _ptr(g), _ptr(y_sorted), _ptr(inv), _ptr(w), T, k, H, _ptr(gy),
              _ptr(gw), _stream())
    return gy, gw


# ----------------------------------------------------------------------------- a9 dX

def _fmt_suffix(w) -> str:
    if isinstance(w, torch.Tensor):
        return "bf16"
    if isinstance(w, _lib.Nf4Weight):
        return "nf4"
    if isinstance(w, _lib.Int8Weight):
        return "int8"
    raise TypeError(f"unsupported weight type {type(w)}")


def _wptr(w):
    return _ptr(_cuda(w, "weight", torch.bfloat16)) if isinstance(w, torch.Tensor) else w


def down_dx(grad_y: torch.Tensor, offsets: torch.Tensor, w2, gate_up: torch.Tensor | None, *, inter: int,
            out: torch.Tensor | None = None, lora: DownLoRA | None = None,
            rank_a: torch.Tensor | None = None, sources: int = 1) -> torch.Tensor:
    """grad_gate_up [S, 2I] = SwiGLU backward of (gate, up) given dh = grad_y W2
    (+ the LoRA path's input gradient when ``lora``).  ``sources`` > 1:
    source-major segments (an expert owner's rows); there ``gate_up=None``
    returns dh [S, I] itself."""
    group = getattr(w2, "group_size", 0)  # block-Hadamard INT8: the rotation group of dh
    w2 = _as_weight(w2)
    gy = _cuda(grad_y, "grad_y", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, H = gy.shape
    if sources > 1:
        if offsets.numel() % sources:
            raise ValueError("source-major segments: offsets must be a multiple of sources")
        E = offsets.numel() // sources
        gu = None if gate_up is None else _cuda(gate_up, "gate_up", torch.bfloat16)
        width = inter if gu is None else 2 * inter
        dgu = out if out is not None else torch.empty((S, width), dtype=torch.bfloat16, device=gy.device)
        if lora is None:
            _lib.call(f"mirai_moe_down_dx_src_{_fmt_suffix(w2)}", _ptr(gy), _ptr(offsets), sources, E, S, H, inter,
                      _wptr(w2), _ptr(gu), _ptr(dgu), _stream())
            return dgu
        glow = rank_a if rank_a is not None else lora_project(gy, offsets, lora, forward=False, sources=sources)
        # dh alone in the block-Hadamard INT8 format is rotated afterwards: its A factor is rotated too
        rot = group if gu is None else 0
        _lib.call(f"mirai_moe_down_dx_lora_src_{_fmt_suffix(w2)}", _ptr(gy), _ptr(offsets), sources, E, S, H, inter,
                  _wptr(w2), _ptr(gu), _ptr(glow), _ptr(lora.a_pad(rotation=rot)), _ptr(dgu), _stream())
        return dgu
    gu = _cuda(gate_up, "gate_up", torch.bfloat16)
    dgu = out if out is not None else torch.empty((S, 2 * inter), dtype=torch.bfloat16, device=gy.device)
    if lora is None:
        _lib.call(f"mirai_moe_down_dx_{_fmt_suffix(w2)}", _ptr(gy), _ptr(offsets), offsets.numel(), S, H, inter,
                  _wptr(w2), _ptr(gu), _ptr(dgu), _stream())
        return dgu
    glow = rank_a if rank_a is not None else lora_project(gy, offsets, lora, forward=False)
    _lib.call(f"mirai_moe_down_dx_lora_{_fmt_suffix(w2)}", _ptr(gy), _ptr(offsets), offsets.numel(), S, H, inter,
              _wptr(w2), _ptr(gu), _ptr(glow), _ptr(lora.a_pad()), _ptr(dgu), _stream())
    return dgu


def down_dh(grad_y: torch.Tensor, offsets: torch.Tensor, w2: Int8Tensor, *, inter: int,
            lora: DownLoRA | None = None, rank_a: torch.Tensor | None = None) -> torch.Tensor:
    """dh_raw [S, I] = grad_y (q s) (+ the rank block with the LoRA A factor
    rotated, so that rotating the sum gives the true dh): the INT8 down dX
    without the SwiGLU backward, for the rotated format."""
    if not isinstance(w2, Int8Tensor):
        raise TypeError("down_dh reads INT8 experts")
    gy = _cuda(grad_y, "grad_y", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, H = gy.shape
    dh = torch.empty((S, inter), dtype=torch.bfloat16, device=gy.device)
    if lora is None:
        _lib.call("mirai_moe_down_dh_int8", _ptr(gy), _ptr(offsets), offsets.numel(), S, H, inter, w2.struct(),
                  _ptr(dh), _stream())
        return dh
    glow = rank_a if rank_a is not None else lora_project(gy, offsets, lora, forward=False)
    _lib.call("mirai_moe_down_dh_lora_int8", _ptr(gy), _ptr(offsets), offsets.numel(), S, H, inter, w2.struct(),
              _ptr(glow), _ptr(lora.a_pad(rotation=w2.group_size)), _ptr(dh), _stream())
    return dh


def lora_grad(x: torch.Tensor, g_rank: torch.Tensor, offsets: torch.Tensor, rank: int, out: torch.Tensor,
              strides, sources: int = 1) -> torch.Tensor:
    """out[e][j][k] = sum over the rows of expert e of g_rank[s, j] * x[s, k]
    (fp32, by strides); ``sources`` > 1: source-major segments, summed in
    source order."""
    x = _cuda(x, "x", torch.bfloat16)
    g = _cuda(g_rank, "g_rank", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, K = x.shape
    se, sr, sk = (int(v) for v in strides)
    if offsets.numel() % sources:
        raise ValueError("source-major segments: offsets must be a multiple of sources")
    _lib.call("mirai_moe_lora_grad_src", _ptr(x), _ptr(g), _ptr(offsets), int(sources), offsets.numel() // sources,
              S, K, int(rank), _ptr(out), se, sr, sk, _stream())
    return out


def gateup_dx(grad_gate_up: torch.Tensor, offsets: torch.Tensor, w1, w3, *, hidden: int,
              out: torch.Tensor | None = None, sources: int = 1) -> torch.Tensor:
    """dx_sorted [S, H] = dgate W1 + dup W3 per expert segment (``sources`` > 1:
    source-major segments)."""
    w1, w3 = _as_weight(w1), _as_weight(w3)
    dgu = _cuda(grad_gate_up, "grad_gate_up", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, I2 = dgu.shape
    dxs = out if out is not None else torch.empty((S, hidden), dtype=torch.bfloat16, device=dgu.device)
    if sources > 1:
        if offsets.numel() % sources:
            raise ValueError("source-major segments: offsets must be a multiple of sources")
        _lib.call(f"mirai_moe_gateup_dx_src_{_fmt_suffix(w1)}", _ptr(dgu), _ptr(offsets), sources,
                  offsets.numel() // sources, S, I2 // 2, hidden, _wptr(w1), _wptr(w3), _ptr(dxs), _stream())
        return dxs
    _lib.call(f"mirai_moe_gateup_dx_{_fmt_suffix(w1)}", _ptr(dgu), _ptr(offsets), offsets.numel(), S, I2 // 2,
              hidden, _wptr(w1), _wptr(w3), _ptr(dxs), _stream())
    return dxs


# ----------------------------------------------------------------------------- any layout / activation / group count

def _ex_suffix(w) -> str:
    if isinstance(w, torch.Tensor):
        return "bf16"
    if isinstance(w, _lib.Nf4Weight):
        return "nf4"
    raise TypeError(f"the *_ex GEMMs read bf16 or NF4 weights, not {type(w)}")


def gateup_ex(x_sorted, offsets, w1, w3, *, inter: int, layout: str, activation: str, save_gate_up: bool = False):
    """gate/up + activation over any number of groups, weights in ``layout``
    ("out_in" [G, I, H] or "in_out" [G, H, I]); returns h (and gate_up)."""
    w1, w3 = _as_weight(w1), _as_weight(w3)
    x_sorted = _cuda(x_sorted, "x_sorted", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, H = x_sorted.shape
    h = torch.empty((S, inter), dtype=torch.bfloat16, device=x_sorted.device)
    gu = torch.empty((S, 2 * inter), dtype=torch.bfloat16, device=x_sorted.device) if save_gate_up else None
    _lib.call(f"mirai_moe_gateup_ex_{_ex_suffix(w1)}", _ptr(x_sorted), _ptr(offsets), offsets.numel(), S, H, inter,
              _wptr(w1), _wptr(w3), LAYOUTS[layout], ACTIVATIONS[activation], _ptr(h), _ptr(gu), _stream())
    return (h, gu) if save_gate_up else h


def down_ex(h, offsets, w2, *, hidden: int, layout: str):
    w2 = _as_weight(w2)
    h = _cuda(h, "h", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, I = h.shape
    y = torch.empty((S, hidden), dtype=torch.bfloat16, device=h.device)
    _lib.call(f"mirai_moe_down_ex_{_ex_suffix(w2)}", _ptr(h), _ptr(offsets), offsets.numel(), S, I, hidden,
              _wptr(w2), LAYOUTS[layout], _ptr(y), _stream())
    return y


def down_dx_ex(grad_y, offsets, w2, gate_up, *, inter: int, layout: str, activation: str):
    w2 = _as_weight(w2)
    gy = _cuda(grad_y, "grad_y", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    gu = _cuda(gate_up, "gate_up", torch.bfloat16)
    S, H = gy.shape
    dgu = torch.empty((S, 2 * inter), dtype=torch.bfloat16, device=gy.device)
    _lib.call(f"mirai_moe_down_dx_ex_{_ex_suffix(w2)}", _ptr(gy), _ptr(offsets), offsets.numel(), S, H, inter,
              _wptr(w2), LAYOUTS[layout], ACTIVATIONS[activation], _ptr(gu), _ptr(dgu), _stream())
    return dgu


def gateup_dx_ex(grad_gate_up, offsets, w1, w3, *, hidden: int, layout: str):
    w1, w3 = _as_weight(w1), _as_weight(w3)
    dgu = _cuda(grad_gate_up, "grad_gate_up", torch.bfloat16)
    offsets = _cuda(offsets, "offsets", torch.int32)
    S, I2 = dgu.shape
    dxs = torch.empty((S, hidden), dtype=torch.bfloat16, device=dgu.device)
    _lib.call(f"mirai_moe_gateup_dx_ex_{_ex_suffix(w1)}", _ptr(dgu), _ptr(offsets), offsets.numel(), S, I2 // 2,
              hidden, _wptr(w1), _wptr(w3), LAYOUTS[layout], _ptr(dxs), _stream())
    return dxs


# ----------------------------------------------------------------------------- whole forward

def _rotations(w1, w3, w2) -> tuple[int, int]:
    """(input group, intermediate group) of a layer's weights: non-zero for the
    rotated INT8 format (w1 and w3 share one activation rotation)."""
    g1, g3 = _group(w1), _group(w3)
    if g1 != g3:
        raise ValueError(f"gate/up rotation groups differ ({g1} vs {g3})")
    return g1, _group(w2)


def moe_forward(tokens: torch.Tensor, top_indices: torch.Tensor, top_weights: torch.Tensor, w1, w3, w2, *,
                num_experts: int, inter: int, lora: "DownLoRA | None" = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Routed expert FFN forward: plan, permute, gate/up+SwiGLU, down, combine.

    Rotated INT8 weights: the tokens are rotated before the permute (T rows,
    not S) and h before the down GEMM; the LoRA rank block is projected from
    the unrotated h."""
    g_in, g_mid = _rotations(w1, w3, w2)
    (w1, w3, w2), join = _stage_beside((w1, w3, w2), top_indices.numel(), num_experts, training=False)
    plan = dispatch_plan(top_indices, num_experts)
    xs = permute_rows(rotate_rows(tokens, g_in) if g_in else tokens, plan.sorted_token_indices)
    join()
    h = gateup_swiglu(xs, plan.offsets, w1, w3, inter=inter)
    low = lora_project(h, plan.offsets, lora, forward=True) if lora is not None else None
    y = down(rotate_rows(h, g_mid) if g_mid else h, plan.offsets, w2, hidden=tokens.shape[1], lora=lora,
             rank_a=low)
    return combine(y, plan.inverse_order, top_weights, out_dtype=out_dtype or tokens.dtype)


@dataclass
class ForwardState:
    """What the dX pass needs from the forward (no dense weights are kept)."""

    plan: DispatchPlan
    y_sorted: torch.Tensor   # [S, H] bf16 expert outputs
    gate_up: torch.Tensor    # [S, 2I] bf16 saved pre-activations
    top_weights: torch.Tensor
    h: torch.Tensor | None = None         # [S, I] bf16, kept when LoRA factor grads are wanted
    rank_a: torch.Tensor | None = None    # [S, 64] LoRA rank block of h (scaled)
    staged: tuple | None = None           # (the NF4 keys, their bf16 copies) when the forward staged them


# NF4 staging: the grouped GEMMs decode NF4 inside their main loops, once per
# 256-row tile of an expert, and that decode (table lookups on the integer
# pipe) limits them below the bf16 kernels' rate.  A training step multiplies
# every expert's weights four times (gate/up and down forward, both dX
# GEMMs), so with many rows per expert it is faster to decode each key once
# into a bf16 copy (one HBM pass, bit-identical values) and run the bf16
# kernels.  The training forward keeps its copies in the state it returns and
# the backward multiplies them again (the reference's frozen linears decode a
# second time instead); they are freed with the state, so a layer holds
# 2 bytes per expert weight from its forward until its backward.
# A forward-only pass multiplies each weight twice as rarely, so "auto" stages
# it from four times the rows per expert: at c2's 2048 the two forms measured
# the same, at c4's 4096 the staged one is faster.
NF4_STAGING_MODES = ("auto", "always", "never")
_nf4_staging = "auto"
STAGE_MIN_ROWS_PER_EXPERT = 1024          # "auto", training passes: at least 4 tiles per expert
STAGE_MIN_ROWS_PER_EXPERT_FORWARD = 4096  # "auto", forward-only passes


def set_nf4_staging(mode: str) -> None:
    """"auto" (default: training passes with at least 1024 rows per expert on
    average, forward-only passes with at least 4096), "always" (every pass) or
    "never" (always decode inside the GEMMs)."""
    global _nf4_staging
    if mode not in NF4_STAGING_MODES:
        raise ValueError(f"NF4 staging mode must be one of {NF4_STAGING_MODES}, not {mode!r}")
    _nf4_staging = mode


def _staging_pays(weights, rows: int, num_experts: int, training: bool) -> bool:
    if _nf4_staging == "never" or not any(isinstance(w, NF4Tensor) for w in weights):
        return False
    least = STAGE_MIN_ROWS_PER_EXPERT if training else STAGE_MIN_ROWS_PER_EXPERT_FORWARD
    return _nf4_staging == "always" or rows >= least * max(1, num_experts)


def stage_nf4(weights, rows: int, num_experts: int, *, training: bool):
    """The weights a pass over ``rows`` routed rows should multiply: NF4 keys
    decoded to bf16 where staging pays (see ``set_nf4_staging``), others as
    given."""
    if not _staging_pays(weights, rows, num_experts, training):
        return tuple(weights)
    return tuple(nf4_dequantize(w) if isinstance(w, NF4Tensor) else w for w in weights)


_side_streams: dict = {}


def _stage_beside(weights, rows: int, num_experts: int, *, training: bool):
    """``stage_nf4`` with the decode on a side stream, so that it runs beside the
    dispatch plan and the permute the caller issues next (both HBM traffic, the
    plan kernels mostly latency).  Returns (weights, join): ``join()`` makes the
    current stream wait for the copies; call it before the first GEMM."""
    if not _staging_pays(weights, rows, num_experts, training):
        return tuple(weights), (lambda: None)
    main = torch.cuda.current_stream()
    dev = next(w for w in weights if isinstance(w, NF4Tensor)).packed.device
    side = _side_streams.get(dev.index)
    if side is None:
        side = _side_streams.setdefault(dev.index, torch.cuda.Stream(device=dev))
    outs = [torch.empty(w.shape, dtype=torch.bfloat16, device=dev) if isinstance(w, NF4Tensor) else None
            for w in weights]  # allocated on the caller's stream, written on the side stream
    side.wait_stream(main)
    with torch.cuda.stream(side):
        for w, o in zip(weights, outs):
            if o is not None:
                nf4_dequantize(w, out=o)
        done = torch.cuda.Event()
        done.record(side)
    for o in outs:
        if o is not None:
            o.record_stream(side)
    return tuple(w if o is None else o for w, o in zip(weights, outs)), (lambda: main.wait_event(done))


def moe_forward_train(tokens, top_indices, top_weights, w1, w3, w2, *, num_experts: int, inter: int,
                      out_dtype: torch.dtype | None = None, lora: DownLoRA | None = None):
    """Forward that also returns the state the dX pass consumes."""
    g_in, g_mid = _rotations(w1, w3, w2)
    keys = (w1, w3, w2)
    (w1, w3, w2), join = _stage_beside(keys, top_indices.numel(), num_experts, training=True)
    staged = (keys, (w1, w3, w2)) if w1 is not keys[0] else None
    plan = dispatch_plan(top_indices, num_experts)
    xs = permute_rows(rotate_rows(tokens, g_in) if g_in else tokens, plan.sorted_token_indices)
    join()
    h, gu = gateup_swiglu(xs, plan.offsets, w1, w3, inter=inter, save_gate_up=True)
    low = None
    if lora is not None:
        low = lora_project(h, plan.offsets, lora, forward=True)
    y = down(rotate_rows(h, g_mid) if g_mid else h, plan.offsets, w2, hidden=tokens.shape[1], lora=lora,
             rank_a=low)
    out = combine(y, plan.inverse_order, top_weights, out_dtype=out_dtype or tokens.dtype)
    keep = lora is not None and lora.compute_grads
    return out, ForwardState(plan, y, gu, top_weights.float(), h if keep else None, low if keep else None, staged)


def moe_backward_dx(grad_out: torch.Tensor, state: ForwardState, w1, w3, w2, *, inter: int,
                    out_dtype: torch.dtype = torch.bfloat16, lora: DownLoRA | None = None):
    """Input gradient through the frozen experts and the top-weight gradient.

    grad_out [T, H] -> (dx [T, H], d_top_weights fp32 [T, k])."""
    plan = state.plan
    H = state.y_sorted.shape[1]
    if state.staged is not None and all(a is b for a, b in zip(state.staged[0], (w1, w3, w2))):
        w1, w3, w2 = state.staged[1]  # the forward's bf16 copies of these NF4 keys
        state.staged = None
    else:
        w1, w3, w2 = stage_nf4((w1, w3, w2), state.y_sorted.shape[0], plan.offsets.numel(), training=True)
    gy, gw = combine_backward(grad_out, state.y_sorted, plan.inverse_order, state.top_weights)
    glow = None
    if lora is not None:
        E, Hb, r = lora.b.shape
        glow = lora_project(gy, plan.offsets, lora, forward=False)
        if lora.compute_grads:
            if state.h is None or state.rank_a is None:
                raise RuntimeError("LoRA factor gradients need the forward run with compute_grads=True")
            Ia = lora.a.shape[2]
            lora.grad_a = lora_grad(state.h, glow, plan.offsets, r,
                                    torch.empty((E, r, Ia), dtype=torch.float32, device=gy.device), (r * Ia, Ia, 1))
            lora.grad_b = lora_grad(gy, state.rank_a, plan.offsets, r,
                                    torch.empty((E, Hb, r), dtype=torch.float32, device=gy.device), (Hb * r, 1, r))
    g_in, g_mid = _rotations(w1, w3, w2)
    if g_mid:  # rotated INT8: dh = rotate(grad_y (q s)), then the SwiGLU backward
        dh = down_dh(gy, plan.offsets, w2, inter=inter, lora=lora, rank_a=glow)
        dgu = swiglu_backward_rotated(dh, state.gate_up, g_mid)
    else:
        dgu = down_dx(gy, plan.offsets, w2, state.gate_up, inter=inter, lora=lora, rank_a=glow)
    dxs = gateup_dx(dgu, plan.offsets, w1, w3, hidden=H)
    if g_in:  # sum the routes in fp32, then rotate the token rows (T, not S)
        dx32 = combine(dxs, plan.inverse_order, None, out_dtype=torch.float32, top_k=plan.top_k)
        return rotate_rows(dx32, g_in, out_dtype=out_dtype), gw
    dx = combine(dxs, plan.inverse_order, None, out_dtype=out_dtype, top_k=plan.top_k)
    return dx, gw
