"""Kernel backend for the reference's MoE ``execute_direct`` seam.

The reference's MoE block calls
``kernel_backend.execute_direct(experts, tokens, top_scores, top_indices)``
(transformer_lingbot_video.py:1790-1796) on the object installed as
``block.ffn._mirai_moe_kernel_backend`` (lingbot_video/pipeline.py:4556-4561);
a return value of ``None`` hands the call back to the built-in path
(:1797-1838).  ``B200MoEKernelBackend`` implements that protocol
(``TorchChunkedKernelBackend``, moe/runtime/kernels.py:131-149, is the
reference's default implementation) on libmirai_b200: it binds the expert
module's own NF4 / INT8 / bf16 buffers in place and runs the fused kernels.

Selection semantics follow the reference's GEMM-backend registry
(moe/runtime/gemm.py:526-548): an explicit selection (``strict=True``, the
default) fails fast with an error naming the problem; ``strict=False`` is the
"auto" behaviour and returns ``None`` so the host keeps its own path.
"""

from __future__ import annotations

from typing import Any

import torch

from . import _lib
from .experts import GroupedExpertWeights, down_lora_of, run_routed

BACKEND_NAME = "b200"


class B200MoEKernelBackend:
    name = BACKEND_NAME
    direct_only = True
    mode = "direct"
    supports_routed_output_observer = False
    supports_routed_intermediate_observer = False

    def __init__(self, *, strict: bool = True):
        self.strict = bool(strict)
        self._cache: dict[int, tuple[tuple, GroupedExpertWeights]] = {}

    @staticmethod
    def _fingerprint(experts: Any) -> tuple:
        ptrs = []
        for name, buf in sorted(getattr(experts, "_buffers", {}).items()):
            if isinstance(buf, torch.Tensor):
                ptrs.append((name, buf.data_ptr(), tuple(buf.shape)))
        for k in ("w1", "w2", "w3"):
            t = getattr(experts, k, None)
            if isinstance(t, torch.Tensor):
                ptrs.append((k, t.data_ptr(), t._version))
        return tuple(ptrs)

    def bind(self, experts: Any) -> GroupedExpertWeights:
        """Weight descriptors for ``experts`` (re-bound when its buffers move)."""
        fp = self._fingerprint(experts)
        hit = self._cache.get(id(experts))
        if hit is not None and hit[0] == fp:
            return hit[1]
        w = GroupedExpertWeights.from_module(experts)
        self._cache[id(experts)] = (fp, w)
        return w

    @staticmethod
    def module_reason(experts: Any) -> str | None:
        """Why this expert module cannot run here (None when it can)."""
        try:
            down_lora_of(experts)
        except _lib.MiraiError as exc:
            return str(exc)
        if callable(getattr(experts, "has_logical_expert_aliases", None)) and experts.has_logical_expert_aliases():
            return "logical expert aliases are not supported"
        return None

    def unsupported_reason(self, experts: Any, tokens: torch.Tensor, top_scores: torch.Tensor,
                           top_indices: torch.Tensor) -> str | None:
        if not isinstance(tokens, torch.Tensor) or not tokens.is_cuda:
            return "tokens are not on a CUDA device"
        if top_indices.ndim != 2 or top_scores.shape != top_indices.shape:
            return "top_scores/top_indices must be matching [tokens, top_k] tensors"
        return self.module_reason(experts)

    def execute_direct(self, experts: Any, tokens: torch.Tensor, top_scores: torch.Tensor,
                       top_indices: torch.Tensor) -> torch.Tensor | None:
        reason = self.unsupported_reason(experts, tokens, top_scores, top_indices)
        if reason is None:
            try:
                weights = self.bind(experts)
            except _lib.MiraiError as exc:
                reason = str(exc)
        if reason is not None:
            if self.strict:
                raise RuntimeError(f"memory.moe_kernel_backend='{BACKEND_NAME}' cannot run this layer: {reason}")
            return None
        return run_routed(weights, tokens, top_scores, top_indices, lora=down_lora_of(experts))


def build_moe_kernel_backend(value: str | None, *, direct_routed: bool = False):
    """Registry hook mirroring ``build_moe_kernel_backend`` (kernels.py:185-213):
    ``"b200"`` selects this backend explicitly (fail fast)."""
    name = str(value or "").strip().lower()
    if name != BACKEND_NAME:
        raise ValueError(f"unknown MoE kernel backend {value!r} (this package provides '{BACKEND_NAME}')")
    if not direct_routed:
        raise ValueError("the b200 backend requires a direct-routed expert provider")
    return B200MoEKernelBackend(strict=True)
