"""Expert parallelism for the routed expert FFN over torch.distributed.

The layer shards by expert: rank r of G owns the contiguous experts
[r*E/G, (r+1)*E/G) and routes its own shard of the tokens.  One layer is

  route (a1) -> global dispatch plan (a2) -> permute (a3)        on the token owner
  all-to-all: rows (and their local expert ids) to the expert owners
  local plan -> permute -> gate/up + down grouped GEMMs          on the expert owner
  un-permute -> all-to-all back -> weighted combine (a8)          on the token owner

Because experts are contiguous per rank, the rows of the global plan (sorted
by expert id) are already grouped by destination rank, so the send buffer is
the permuted activation itself.  The received rows arrive source-rank-major
and, within a source, in expert order; the local plan re-sorts them stably by
local expert, which reproduces the single-GPU row order of every expert
segment when tokens are sharded contiguously by rank, so the result equals
the single-GPU layer.  The reference runs MoE on one GPU (it has no expert
parallelism); the exchange is this package's.  (Receiving each (rank, expert)
block straight into an expert-major layout with grouped NCCL send/recv was
measured slower on B200 than one all_to_all_single plus the local re-sort:
18.8 vs 25.7 M tokens/s for c2 on 2 GPUs.)

Split sizes must be known on the host for NCCL's all-to-all, so each layer
reads G counts back once (the reference's own host sync per layer,
experts.py:2382, is of the same kind).

`StepOps` names the per-rank steps.  The product path uses `CudaStepOps`
(the sm_100a kernels); tests of the exchange logic on CPU ranks pass their own.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Protocol

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ExpertShard:
    """This rank's block of experts."""

    num_experts: int
    world: int
    rank: int

    def __post_init__(self):
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside a world of {self.world}")
        if self.num_experts % self.world != 0:
            raise ValueError(f"{self.num_experts} experts do not split evenly over {self.world} ranks")

    @property
    def local(self) -> int:
        return self.num_experts // self.world

    @property
    def first(self) -> int:
        return self.rank * self.local


class StepOps(Protocol):
    def route(self, logits: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]: ...
    def plan(self, top_indices: torch.Tensor, num_experts: int) -> Any: ...
    def permute(self, x: torch.Tensor, sorted_token_indices: torch.Tensor) -> torch.Tensor: ...
    def experts(self, x_sorted: torch.Tensor, offsets: torch.Tensor, weights: Any, inter: int) -> torch.Tensor: ...
    def combine(self, y_sorted: torch.Tensor, inverse_order: torch.Tensor, top_weights: torch.Tensor | None,
                top_k: int, out_dtype: torch.dtype) -> torch.Tensor: ...


class CudaStepOps:
    """The per-rank steps on the sm_100a kernels (mirai_b200.ops)."""

    def __init__(self):
        from . import ops
        self.ops = ops

    def route(self, logits, top_k):
        return self.ops.route_topk(logits, top_k)

    def plan(self, top_indices, num_experts):
        return self.ops.dispatch_plan(top_indices, num_experts)

    def permute(self, x, sorted_token_indices):
        return self.ops.permute_rows(x, sorted_token_indices)

    def experts(self, x_sorted, offsets, weights, inter):
        w1, w3, w2 = weights
        h = self.ops.gateup_swiglu(x_sorted, offsets, w1, w3, inter=inter)
        return self.ops.down(h, offsets, w2, hidden=x_sorted.shape[1])

    def combine(self, y_sorted, inverse_order, top_weights, top_k, out_dtype):
        return self.ops.combine(y_sorted, inverse_order, top_weights, out_dtype=out_dtype, top_k=top_k)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group) -> None:
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def ep_moe_forward(tokens: torch.Tensor, logits: torch.Tensor, local_weights: Any, *, shard: ExpertShard,
                   top_k: int, inter: int, group=None, ops: StepOps | None = None) -> torch.Tensor:
    """One expert-parallel routed FFN layer for this rank's tokens.

    tokens [T_r, H] bf16 and router logits [T_r, E] fp32 are this rank's token
    shard; ``local_weights`` = (w1, w3, w2) of this rank's E/G experts, in any
    format the GEMMs take.  Returns [T_r, H] in the tokens' dtype.  Every rank
    must call it (the exchange is collective), with or without tokens."""
    ops = ops or CudaStepOps()
    G, E, El = shard.world, shard.num_experts, shard.local
    T, H = tokens.shape
    dev = tokens.device
    idx, tw = ops.route(logits, top_k)
    plan = ops.plan(idx, E)
    xs = ops.permute(tokens, plan.sorted_token_indices)
    if G == 1:  # one rank owns every expert: no exchange
        y = ops.experts(xs, plan.offsets, local_weights, inter)
        return ops.combine(y, plan.inverse_order, tw, top_k, tokens.dtype)
    # rows per destination rank (experts are contiguous per rank) and, per row,
    # the expert's index inside its owner's block
    send_counts = plan.counts.view(G, El).sum(1)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.cat([send_counts, recv_counts]).tolist()  # the one host read per layer
    sc, rc = counts[:G], counts[G:]
    # expert of sorted row s = the segment containing s (offsets are inclusive ends)
    S = xs.shape[0]
    rows = torch.arange(S, device=dev, dtype=plan.offsets.dtype)
    local_ids = (torch.searchsorted(plan.offsets, rows, right=True) % El).to(torch.int64)
    R = sum(rc)
    x_recv = torch.empty((R, H), dtype=xs.dtype, device=dev)
    e_recv = torch.empty((R,), dtype=torch.int64, device=dev)
    _a2a(x_recv, xs, rc, sc, group)
    _a2a(e_recv, local_ids, rc, sc, group)
    # expert owner: group the received rows by local expert, run the experts, restore the order
    if R > 0:
        lplan = ops.plan(e_recv.view(R, 1), El)
        xl = ops.permute(x_recv, lplan.sorted_token_indices)
        yl = ops.experts(xl, lplan.offsets, local_weights, inter)
        y_recv = ops.combine(yl, lplan.inverse_order, None, 1, yl.dtype)
    else:
        y_recv = torch.empty((0, H), dtype=xs.dtype, device=dev)
    y_back = torch.empty_like(xs)
    _a2a(y_back, y_recv, sc, rc, group)
    if T == 0:
        return torch.empty((0, H), dtype=tokens.dtype, device=dev)
    return ops.combine(y_back, plan.inverse_order, tw, top_k, tokens.dtype)


def shard_tokens(num_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous token shard (the first T % G ranks take one more)."""
    base, extra = divmod(num_tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)
