"""Expert parallelism for the routed expert FFN over torch.distributed.

The layer shards by expert: rank r of G owns the contiguous experts
[r*E/G, (r+1)*E/G) and routes its own shard of the tokens.  One layer is

  route (a1) -> global dispatch plan (a2) -> permute (a3)        on the token owner
  all-to-all: rows to the expert owners
  gate/up + down grouped GEMMs over source-major segments         on the expert owner
  all-to-all back -> weighted combine (a8)                        on the token owner

Because experts are contiguous per rank, the rows of the global plan (sorted
by expert id) are already grouped by destination rank and, inside, by
expert, so the send buffer is the permuted activation itself.  The received
rows arrive source-major, each source's rows in expert order; the grouped
GEMMs take those G x E/G (source, expert) segments as they are (weight =
expert; each segment cut into 128-row blocks, an expert's blocks paired into
256-row tiles, tiles visited expert-major), so the owner neither re-sorts nor
restores the order, and its output goes back through the reverse all-to-all
in the layout the token owner sent.  (``ExpertParallelMoE``, the copy-engine
transport, receives source-major too by default; it can instead place the
blocks expert-major, or regroup a chunk's rows expert-major before the GEMMs.)
Per row the products are those of the single-GPU layer, so the result is
identical to it.  The reference runs MoE
on one GPU (it has no expert parallelism); the exchange is this package's.
(Receiving each (rank, expert) block straight into an expert-major layout
with grouped NCCL send/recv was measured slower on B200 than one
all_to_all_single: 18.8 vs 25.7 M tokens/s for c2 on 2 GPUs.)

Split sizes must be known on the host for NCCL's all-to-all, so each layer
reads the [G, chunks, E/G] count matrices back once (the reference's own host
sync per layer, experts.py:2382, is of the same kind).

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
    def experts(self, x_sorted: torch.Tensor, offsets: torch.Tensor, weights: Any, inter: int,
                sources: int = 1) -> torch.Tensor: ...
    def combine(self, y_sorted: torch.Tensor, inverse_order: torch.Tensor, top_weights: torch.Tensor | None,
                top_k: int, out_dtype: torch.dtype) -> torch.Tensor: ...
    # training (the dX pass through frozen experts)
    def experts_train(self, x_sorted: torch.Tensor, offsets: torch.Tensor, weights: Any, inter: int,
                      sources: int = 1) -> tuple[torch.Tensor, Any]: ...
    def experts_backward(self, grad_y: torch.Tensor, offsets: torch.Tensor, weights: Any, inter: int,
                         sources: int, saved: Any) -> torch.Tensor: ...
    def combine_backward(self, grad_out: torch.Tensor, y_sorted: torch.Tensor, inverse_order: torch.Tensor,
                         top_weights: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]: ...


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

    def experts(self, x_sorted, offsets, weights, inter, sources=1):
        return self.experts_train(x_sorted, offsets, weights, inter, sources, save=False)[0]

    def stage(self, weights, rows, training):
        """The weights a layer's owner GEMMs multiply over ``rows`` received rows
        (NF4 keys decoded once to bf16 where that pays: ``ops.stage_nf4``)."""
        return self.ops.stage_nf4(tuple(weights), rows, weights[0].shape[0], training=training)

    def experts_train(self, x_sorted, offsets, weights, inter, sources=1, save=True, lora=None):
        """The owner's GEMMs over its received (source, expert) segments; the
        block-Hadamard INT8 format rotates the received rows and h here (a row's
        rotation does not depend on where it runs).  A LoRA adapter on w2 (this
        rank's experts' factors) runs on the same segments: its projections and
        rank blocks read each segment's expert."""
        w1, w3, w2 = weights
        g_in, g_mid = self.ops._rotations(w1, w3, w2)
        x = self.ops.rotate_rows(x_sorted, g_in) if g_in else x_sorted
        res = self.ops.gateup_swiglu(x, offsets, w1, w3, inter=inter, sources=sources, save_gate_up=save)
        h, gu = res if save else (res, None)
        low = self.ops.lora_project(h, offsets, lora, forward=True, sources=sources) if lora is not None else None
        y = self.ops.down(self.ops.rotate_rows(h, g_mid) if g_mid else h, offsets, w2, hidden=x_sorted.shape[1],
                          sources=sources, lora=lora, rank_a=low)
        keep = lora is not None and lora.compute_grads
        return y, (gu, h if keep else None, low if keep else None)

    def experts_backward(self, grad_y, offsets, weights, inter, sources, saved, lora=None):
        if isinstance(saved, tuple) and saved and isinstance(saved[0], str):
            _, order, inverse, ends, inner = saved
            dxs = self.experts_backward(self.ops.permute_rows(grad_y, order), ends, weights, inter, 1, inner, lora)
            return self.ops.permute_rows(dxs, inverse)
        gu, h, low = saved
        w1, w3, w2 = weights
        g_in, g_mid = self.ops._rotations(w1, w3, w2)
        glow = None
        if lora is not None:
            glow = self.ops.lora_project(grad_y, offsets, lora, forward=False, sources=sources)
            if lora.compute_grads:  # this chunk's share of the factor gradients, added up over chunks
                E, Hb, r = lora.b.shape
                Ia = lora.a.shape[2]
                ga = self.ops.lora_grad(h, glow, offsets, r, torch.empty((E, r, Ia), dtype=torch.float32,
                                                                         device=grad_y.device), (r * Ia, Ia, 1),
                                        sources=sources)
                gb = self.ops.lora_grad(grad_y, low, offsets, r, torch.empty((E, Hb, r), dtype=torch.float32,
                                                                             device=grad_y.device), (Hb * r, 1, r),
                                        sources=sources)
                lora.grad_a = ga if lora.grad_a is None else lora.grad_a + ga
                lora.grad_b = gb if lora.grad_b is None else lora.grad_b + gb
        if g_mid:
            dh = (self.ops.down_dx(grad_y, offsets, w2, None, inter=inter, sources=sources, lora=lora, rank_a=glow)
                  if sources > 1 else self.ops.down_dh(grad_y, offsets, w2, inter=inter, lora=lora, rank_a=glow))
            dgu = self.ops.swiglu_backward_rotated(dh, gu, g_mid)
        else:
            dgu = self.ops.down_dx(grad_y, offsets, w2, gu, inter=inter, sources=sources, lora=lora, rank_a=glow)
        dxs = self.ops.gateup_dx(dgu, offsets, w1, w3, hidden=grad_y.shape[1], sources=sources)
        return self.ops.rotate_rows(dxs, g_in) if g_in else dxs

    def combine(self, y_sorted, inverse_order, top_weights, top_k, out_dtype):
        return self.ops.combine(y_sorted, inverse_order, top_weights, out_dtype=out_dtype, top_k=top_k)

    def combine_backward(self, grad_out, y_sorted, inverse_order, top_weights, top_k):
        return self.ops.combine_backward(grad_out, y_sorted, inverse_order, top_weights)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group) -> None:
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


@dataclass
class EPTrainState:
    """What ``ep_moe_backward`` needs from a training forward, per chunk: the
    token-owner side (route weights, plan, the returned expert outputs, split
    sizes) and the expert-owner side (segment ends, the saved gate/up of the
    rows it received)."""

    bounds: list            # [(begin, end)] token range of each chunk
    chunks: list            # per chunk: dict(tw, plan, y_back, sc, rc, offs, saved)
    top_k: int
    hidden: int
    dtype: torch.dtype
    staged: tuple | None = None  # (the local NF4 keys, their bf16 copies) when the forward staged them


def _stage(ops, weights, rows: int, training: bool):
    """(weights the owner's GEMMs multiply, (keys, copies) or None): NF4 keys
    decoded once per layer where that pays (``CudaStepOps.stage``)."""
    f = getattr(ops, "stage", None)
    staged = tuple(weights) if f is None else f(weights, rows, training)
    return staged, ((tuple(weights), staged) if staged[0] is not weights[0] else None)


def _weights_for(staged, local_weights):
    """The forward's bf16 copies when the backward gets the same keys."""
    if staged is not None and all(a is b for a, b in zip(staged[0], local_weights)):
        return staged[1]
    return local_weights


def ep_moe_forward(tokens: torch.Tensor, logits: torch.Tensor, local_weights: Any, *, shard: ExpertShard,
                   top_k: int, inter: int, group=None, ops: StepOps | None = None, chunks: int = 1,
                   comm_stream: torch.cuda.Stream | None = None, train: bool = False, lora=None):
    """One expert-parallel routed FFN layer for this rank's tokens.

    tokens [T_r, H] bf16 and router logits [T_r, E] fp32 are this rank's token
    shard; ``local_weights`` = (w1, w3, w2) of this rank's E/G experts, in any
    format the GEMMs take.  Returns [T_r, H] in the tokens' dtype.  Every rank
    must call it (the exchange is collective) with the same ``chunks``, with or
    without tokens.

    ``chunks`` > 1 splits the tokens into that many contiguous chunks whose
    exchanges run on ``comm_stream`` while the other chunks' GEMMs run on the
    current stream (chunk i's rows travel while chunk i-1 computes, and its
    results return while chunk i+1 computes).  The result is the same as with
    one chunk.  For the overlap to happen the GEMMs must leave SMs free for the
    communication kernels (``ops.set_gemm_sm_limit``).

    ``train=True`` returns ``(out, state)``: the owners keep the gate/up
    pre-activations of the rows they received, the token owners the expert
    outputs that came back, for ``ep_moe_backward`` (chunks then run one after
    another, on the current stream).  ``lora`` (``ops.DownLoRA`` over this
    rank's experts) adds a LoRA adapter on w2 (training only); its factor
    gradients are this rank's experts' and come out of ``ep_moe_backward``."""
    if lora is not None and not train:
        raise ValueError("the expert-parallel forward takes a LoRA adapter in training (train=True)")
    ops = ops or CudaStepOps()
    G, E, El = shard.world, shard.num_experts, shard.local
    T, H = tokens.shape
    dev = tokens.device
    if G == 1:  # one rank owns every expert: no exchange
        idx, tw = ops.route(logits, top_k)
        plan = ops.plan(idx, E)
        xs = ops.permute(tokens, plan.sorted_token_indices)
        if not train:
            y = ops.experts(xs, plan.offsets, _stage(ops, local_weights, xs.shape[0], False)[0], inter)
            return ops.combine(y, plan.inverse_order, tw, top_k, tokens.dtype)
        wts, staged = _stage(ops, local_weights, xs.shape[0], True)
        y, saved = ops.experts_train(xs, plan.offsets, wts, inter, **({"lora": lora} if lora else {}))
        out = ops.combine(y, plan.inverse_order, tw, top_k, tokens.dtype)
        return out, EPTrainState([(0, T)], [dict(tw=tw, plan=plan, y_back=y, sc=None, rc=None, offs=plan.offsets,
                                                 saved=saved)], top_k, H, tokens.dtype, staged)
    C = max(1, int(chunks))
    bounds = [((T * c) // C, (T * (c + 1)) // C) for c in range(C)]
    # ---- per chunk, on the current stream: route, plan, permute
    prep = []
    for b, e in bounds:
        idx, tw = ops.route(logits[b:e], top_k)
        plan = ops.plan(idx, E)
        prep.append((tw, plan, ops.permute(tokens[b:e], plan.sorted_token_indices)))
    # rows per (destination rank, chunk, local expert): experts are contiguous per
    # rank, so chunk c's permuted rows for rank d are one run ordered by expert.
    # One exchange of the count matrices and one host read for the whole layer.
    send_mat = torch.stack([p[1].counts.view(G, El) for p in prep], dim=1).contiguous()  # [dest, chunk, expert]
    recv_mat = torch.empty_like(send_mat)                                                 # [source, chunk, expert]
    dist.all_to_all_single(recv_mat, send_mat, group=group)
    flat = torch.cat([send_mat.reshape(-1), recv_mat.reshape(-1)]).tolist()
    n = G * C * El
    # this rank's counts [1, dest, chunk, expert] and what it received; both must be sane
    import numpy as np
    check_counts(np.asarray(flat[:n]).reshape(1, G, C, El), 0, [p[2].shape[0] for p in prep])
    if min(flat[n:], default=0) < 0:
        raise ValueError("expert-parallel exchange: negative row count received")
    sm_ = [[flat[(d * C + c) * El:(d * C + c + 1) * El] for d in range(G)] for c in range(C)]
    rm_ = [[flat[n + (s_ * C + c) * El:n + (s_ * C + c + 1) * El] for s_ in range(G)] for c in range(C)]
    sc = [[sum(sm_[c][d]) for d in range(G)] for c in range(C)]
    rc = [[sum(rm_[c][s_]) for s_ in range(G)] for c in range(C)]
    # received rows of chunk c: source-major, each source's rows in expert order;
    # the GEMMs take these G * El segments as they are (ends = running sum)
    seg_ends = []
    for c in range(C):
        run, ends = 0, []
        for s_ in range(G):
            for e in range(El):
                run += rm_[c][s_][e]
                ends.append(run)
        seg_ends.append(ends)
    offs_dev = torch.tensor(seg_ends, dtype=torch.int32).to(dev, non_blocking=True) if tokens.is_cuda else \
        torch.tensor(seg_ends, dtype=torch.int32)

    comp = torch.cuda.current_stream(dev) if tokens.is_cuda else None
    comm = comm_stream if (C > 1 and tokens.is_cuda and not train) else None

    def keep(t, stream):
        # a tensor used on a stream other than its own is not reused before that stream is done with it
        if stream is not None and t.is_cuda:
            t.record_stream(stream)
        return t

    def on_comm(fn, after):
        comm.wait_event(after)
        with torch.cuda.stream(comm):
            out = fn()
            ev = torch.cuda.Event()
            ev.record(comm)
        return out, ev

    def mark():
        ev = torch.cuda.Event()
        ev.record(comp)
        return ev

    def dispatch(c):
        xs = keep(prep[c][2], comm)
        x_recv = keep(torch.empty((sum(rc[c]), H), dtype=xs.dtype, device=dev), comp if comm is not None else None)
        _a2a(x_recv, xs, rc[c], sc[c], group)
        return x_recv

    fwd_weights = None

    def compute(c, x_recv):
        nonlocal fwd_weights
        if x_recv.shape[0] == 0:
            return torch.empty((0, H), dtype=x_recv.dtype, device=dev)
        if fwd_weights is None:  # NF4 keys decoded once for the layer where that pays
            fwd_weights = _stage(ops, local_weights, sum(sum(r) for r in rc), False)[0]
        return ops.experts(x_recv, offs_dev[c], fwd_weights, inter, sources=G)

    def give_back(c, y_recv):
        keep(y_recv, comm)
        y_back = keep(torch.empty_like(prep[c][2]), comp if comm is not None else None)
        _a2a(y_back, y_recv, sc[c], rc[c], group)
        return y_back

    out = torch.empty((T, H), dtype=tokens.dtype, device=dev)
    if train:
        state = []
        wts, staged = _stage(ops, local_weights, sum(sum(r) for r in rc), True)
        for c, (b, e) in enumerate(bounds):
            x_recv = dispatch(c)
            if x_recv.shape[0]:
                y_recv, saved = ops.experts_train(x_recv, offs_dev[c], wts, inter, sources=G,
                                                  **({"lora": lora} if lora else {}))
            else:
                y_recv, saved = torch.empty((0, H), dtype=x_recv.dtype, device=dev), None
            y_back = give_back(c, y_recv)
            if e > b:
                out[b:e] = ops.combine(y_back, prep[c][1].inverse_order, prep[c][0], top_k, tokens.dtype)
            state.append(dict(tw=prep[c][0], plan=prep[c][1], y_back=y_back, sc=sc[c], rc=rc[c], offs=offs_dev[c],
                              saved=saved))
        return out, EPTrainState(bounds, state, top_k, H, tokens.dtype, staged)
    if comm is None:
        for c, (b, e) in enumerate(bounds):
            y_back = give_back(c, compute(c, dispatch(c)))
            if e > b:
                out[b:e] = ops.combine(y_back, prep[c][1].inverse_order, prep[c][0], top_k, tokens.dtype)
        return out
    # pipelined: dispatch c+1 and return c-1 on `comm` overlap compute c on the current stream
    ready = mark()
    sent = [on_comm(lambda c=c: dispatch(c), ready) for c in range(C)]
    backs = []
    for c in range(C):
        x_recv, ev = sent[c]
        comp.wait_event(ev)
        y_recv = compute(c, x_recv)
        backs.append(on_comm(lambda c=c, y=y_recv: give_back(c, y), mark()))
    for c, (b, e) in enumerate(bounds):
        y_back, ev = backs[c]
        comp.wait_event(ev)
        if e > b:
            out[b:e] = ops.combine(y_back, prep[c][1].inverse_order, prep[c][0], top_k, tokens.dtype)
    return out


def ep_moe_backward(grad_out: torch.Tensor, state: EPTrainState, local_weights: Any, *, shard: ExpertShard,
                    inter: int, group=None, ops: StepOps | None = None, lora=None) -> tuple[torch.Tensor, torch.Tensor]:
    """dX of ``ep_moe_forward(train=True)`` through the frozen experts:
    grad_out [T_r, H] -> (dx [T_r, H] in the tokens' dtype, d_top_weights fp32
    [T_r, k]).  Collective, like the forward (every rank calls it).

    Per chunk, mirroring the forward: the combine backward on the token owner
    (linear.py's frozen-linear backward inputs, dispatch_ops.py:36-44); the
    gradient rows travel to the expert owners with the forward's split sizes;
    the owner's down dX (SwiGLU backward fused, on the gate/up it kept) and
    gate/up dX run over the same source-major segments; dX rows travel back
    and the token owner sums each token's routes (the permute backward,
    dispatch_ops.py:15-20).  Every row's products are those of the single-GPU
    backward, so the result equals it."""
    ops = ops or CudaStepOps()
    G = shard.world
    k, H = state.top_k, state.hidden
    kw = {"lora": lora} if lora is not None else {}
    if lora is not None and lora.compute_grads:
        lora.grad_a = lora.grad_b = None  # summed over this call's chunks
    T = grad_out.shape[0]
    dev = grad_out.device
    dx = torch.empty((T, H), dtype=state.dtype, device=dev)
    dw = torch.empty((T, k), dtype=torch.float32, device=dev)
    local_weights = _weights_for(state.staged, local_weights)
    state.staged = None
    for (b, e), st in zip(state.bounds, state.chunks):
        plan = st["plan"]
        if e > b:
            gy, gw = ops.combine_backward(grad_out[b:e], st["y_back"], plan.inverse_order, st["tw"], k)
            dw[b:e] = gw
        else:  # no tokens here: an empty block of the gradient rows' dtype (the collectives need one dtype)
            gy = torch.empty((0, H), dtype=st["y_back"].dtype, device=dev)
        if G == 1:
            dxs = ops.experts_backward(gy, st["offs"], local_weights, inter, 1, st["saved"], **kw)
        else:
            gy_recv = torch.empty((sum(st["rc"]), H), dtype=gy.dtype, device=dev)
            _a2a(gy_recv, gy.contiguous(), st["rc"], st["sc"], group)
            if gy_recv.shape[0]:
                dx_recv = ops.experts_backward(gy_recv, st["offs"], local_weights, inter, G, st["saved"], **kw)
            else:
                dx_recv = torch.empty((0, H), dtype=gy.dtype, device=dev)
            dxs = torch.empty((sum(st["sc"]), H), dtype=dx_recv.dtype, device=dev)
            _a2a(dxs, dx_recv.contiguous(), st["sc"], st["rc"], group)
        if e > b:
            dx[b:e] = ops.combine(dxs, plan.inverse_order, None, k, state.dtype)
    return dx, dw


def check_counts(M, rank: int, sent_rows: list[int]) -> None:
    """Reject an exchange whose gathered counts M [source, dest, chunk, local
    expert] cannot be right before any row moves: a negative count anywhere,
    or this rank's counts for a chunk not summing to the rows it permuted for
    that chunk (a corrupted or foreign plan).  Raises ValueError; a peer that
    goes on to the row exchange then ends in the process group's timeout."""
    import numpy as np
    M = np.asarray(M)
    if (M < 0).any():
        raise ValueError("expert-parallel exchange: negative row count in the gathered counts")
    mine = M[rank].sum(axis=(0, 2))
    for c, rows in enumerate(sent_rows):
        if int(mine[c]) != int(rows):
            raise ValueError(f"expert-parallel exchange: rank {rank} chunk {c} counts {int(mine[c])} routed rows "
                             f"but permuted {int(rows)}")


def shard_tokens(num_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous token shard (the first T % G ranks take one more)."""
    base, extra = divmod(num_tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


@dataclass
class BlockPlan:
    """Where every block of one rank's copy-engine exchange goes.

    Rows are counted, not bytes.  A "dispatch" block moves this rank's rows of
    one chunk for one (owner, local expert) from its permuted send rows to the
    owner's receive region; a "return" block moves the owner's results for one
    (source, local expert) of a chunk back to the source's return region.  Each
    block list is four int64 arrays: peer rank, row in the peer's region, row
    in this rank's chunk rows, row count."""

    in_cap: int                   # receive region rows, the same on every rank
    ret_cap: int                  # return region rows, the same on every rank
    in_base: list[int]            # first row of chunk c in this rank's receive region
    in_rows: list[int]            # rows this rank receives in chunk c
    ret_base: list[int]           # first row of chunk c in this rank's return region
    ret_rows: list[int]           # rows this rank sends (and gets back) in chunk c
    gemm_ends: list[list[int]]    # [chunk][segment] running row ends of the receive rows
    sources: int                  # segments per expert in gemm_ends (1: expert-major; G: source-major)
    dispatch: list[tuple]         # per chunk: (peer, peer_row, my_row, rows)
    give_back: list[tuple]        # per chunk: (peer, peer_row, my_row, rows)
    # per chunk, source-major layout only: None, or the running ends of the
    # expert segments when the owner regroups the chunk's received rows
    # expert-major before its GEMMs (``regroup_order``)
    regroup: list = None


def _merge_runs(peer, peer_row, my_row, rows):
    """Join consecutive blocks that continue each other on both sides."""
    import numpy as np
    if len(rows) < 2:
        return peer, peer_row, my_row, rows
    cont = (peer[1:] == peer[:-1]) & (peer_row[1:] == peer_row[:-1] + rows[:-1]) & \
        (my_row[1:] == my_row[:-1] + rows[:-1])
    start = np.concatenate([[True], ~cont])
    idx = np.nonzero(start)[0]
    return peer[idx], peer_row[idx], my_row[idx], np.add.reduceat(rows, idx)


# Costs that decide whether an owner regroups a chunk's received rows (two row
# gathers through HBM) to save the GEMM tiles that source boundaries cut:
# measured on B200 for the NF4 grouped GEMMs and the row-gather kernel.  The
# GEMM rate is the marginal one of an extra 256-row tile (5.8 us at H=4096,
# I=1536 on segment lengths near 256: a tile-equivalent 1.6 PFLOP/s; the
# kernels' average rate is about 1.0 PFLOP/s).
GEMM_FLOPS_PER_S = 1.6e15
GATHER_BYTES_PER_S = 6.0e12
TILE_ROWS = 256


def regroup_pays(L, hidden: int, inter: int, row_bytes: int) -> bool:
    """L [sources, experts] rows of one received chunk, source-major.  True if
    regrouping them expert-major (a gather of the rows there and one of the
    results back) costs less than the GEMM tiles it saves.  On source-major
    rows the GEMMs cut each segment into 128-row blocks and pair an expert's
    blocks into 256-row tiles, so a segment wastes at most part of a block."""
    import numpy as np
    return bool(_regroup_pays_chunks(np.asarray(L, dtype=np.int64)[:, None, :], hidden, inter, row_bytes)[0])


def _regroup_pays_chunks(L, hidden: int, inter: int, row_bytes: int):
    """``regroup_pays`` for every chunk at once: L [sources, chunks, experts]."""
    half = TILE_ROWS // 2  # source-major segments are tiled in half-tile blocks, two per tile
    tiles_src = ((((L + half - 1) // half).sum(axis=0) + 1) // 2).sum(axis=1)
    tiles_exp = ((L.sum(axis=0) + TILE_ROWS - 1) // TILE_ROWS).sum(axis=1)
    saved = (tiles_src - tiles_exp) * (6.0 * TILE_ROWS * hidden * inter / GEMM_FLOPS_PER_S)
    cost = L.sum(axis=(0, 2)) * (4.0 * row_bytes / GATHER_BYTES_PER_S)  # two gathers, each a read and a write
    return (saved > cost) & (L.sum(axis=(0, 2)) > 0)


def regroup_order(L: torch.Tensor, total: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(order, inverse) for the ``total`` rows of one chunk received
    source-major with L [sources, experts] rows per segment (a tensor on the
    rows' device, so no host round trip): rows ``order`` of the chunk are its
    rows expert-major (source order inside an expert); ``inverse[order[i]] = i``."""
    L = L.to(torch.int64)
    flat = L.reshape(-1)
    start = (torch.cumsum(flat, 0) - flat).view(L.shape)        # source-major start of each (s, e)
    lens = L.t().reshape(-1)                                     # expert-major segment order (e, s)
    starts = start.t().reshape(-1)
    shift = starts - (torch.cumsum(lens, 0) - lens)
    rows = torch.arange(total, dtype=torch.int64, device=L.device)
    order = torch.repeat_interleave(shift, lens, output_size=total) + rows
    inverse = torch.empty_like(order).scatter_(0, order, rows)
    return order, inverse


def exchange_blocks(M, rank: int, layout: str = "expert", *, regroup: str = "never", hidden: int = 0,
                    inter: int = 0, row_bytes: int = 0) -> BlockPlan:
    """Block plan of ``rank`` for the count tensor M [source, dest, chunk, local
    expert] (rows every rank sends every owner, per chunk and owner's expert),
    which every rank holds after the count gather.

    ``layout`` "expert": receive regions are expert-major — chunk c of owner d
    holds, for each of its experts in turn, that expert's rows from source 0,
    1, ... in order, so the owner's grouped GEMMs see one contiguous segment
    per expert (tiles are not split at source boundaries), at the price of one
    copy per (peer, expert) block.  "source": source-major — each source's rows
    of the chunk in one run, in expert order, one copy per peer and chunk; the
    GEMMs then take G x E/G (source, expert) segments (``gemm_ends`` holds G*El
    ends per chunk).  A source's send rows of a chunk are ordered by global
    expert (the dispatch plan's order), i.e. by owner, then local expert; its
    return region uses the same order, so the combine reads it like the
    single-GPU layer's expert output.  Blocks that continue each other on both
    sides are merged into one copy, and each list visits the peers starting
    from ``rank`` itself (a rotated schedule, so that the ranks' copies do not
    all converge on one peer).

    ``regroup`` ("never", "auto", "always"; source-major layout only): whether
    the owner regroups a chunk's received rows expert-major before its GEMMs
    (``BlockPlan.regroup``); "auto" does so where ``regroup_pays`` for the
    layer's ``hidden``/``inter`` sizes and ``row_bytes``."""
    import numpy as np
    if layout not in ("expert", "source"):
        raise ValueError(f"layout must be 'expert' or 'source', not {layout!r}")
    M = np.asarray(M, dtype=np.int64)
    if (M < 0).any():
        raise ValueError("exchange_blocks: negative row count")
    G, _, C, El = M.shape
    R = M.sum(axis=(0, 3))                    # rows each owner receives [dest, chunk]
    S = M.sum(axis=(1, 3))                    # rows each source sends [source, chunk]
    in_base = np.concatenate([np.zeros((G, 1), np.int64), np.cumsum(R, axis=1)[:, :-1]], axis=1)
    ret_base = np.concatenate([np.zeros((G, 1), np.int64), np.cumsum(S, axis=1)[:, :-1]], axis=1)
    me = rank
    rot = (me + np.arange(G)) % G  # peers in the order me, me+1, ... (mod G): at each step of the
    # copy schedule every rank targets a different peer, so no peer's inbound links are shared by all
    # senders at once
    dispatch, give_back, ends = [], [], []
    if layout == "source":
        # one block per (peer, chunk): a source's rows for an owner are one run on both sides
        n = M.sum(axis=3)                                     # rows [source, dest, chunk]
        src_off = np.cumsum(n, axis=0) - n                    # rows of lower sources in d's chunk block
        send_off = np.cumsum(n, axis=1) - n                   # rows for lower owners in s's chunk rows
        for c in range(C):
            rows = n[me, rot, c]
            keep = rows > 0
            d = rot[keep]
            dispatch.append((d, in_base[d, c] + src_off[me, d, c], send_off[me, d, c], rows[keep]))
            rows = n[rot, me, c]
            keep = rows > 0
            s_ = rot[keep]
            give_back.append((s_, ret_base[s_, c] + send_off[s_, me, c], src_off[s_, me, c], rows[keep]))
            ends.append(np.cumsum(M[:, me, c, :].reshape(-1)).tolist())
    else:
        # send position of block (s, d, c, e) in s's chunk-c rows: order (d, e)
        flat = M.transpose(0, 2, 1, 3).reshape(G, C, G * El)
        send_pos = (np.cumsum(flat, axis=2) - flat).reshape(G, C, G, El).transpose(0, 2, 1, 3)
        # receive position of block (s, d, c, e) in d's chunk-c rows: order (e, s)
        flat = M.transpose(1, 2, 3, 0).reshape(G, C, El * G)
        recv_pos = (np.cumsum(flat, axis=2) - flat).reshape(G, C, El, G).transpose(3, 0, 1, 2)

        def rotated(peer, *cols):
            order = np.argsort((peer - me) % G, kind="stable")
            return _merge_runs(peer[order], *(col[order] for col in cols))

        for c in range(C):
            d, e = np.nonzero(M[me, :, c, :])
            dispatch.append(rotated(d, in_base[d, c] + recv_pos[me, d, c, e], send_pos[me, d, c, e],
                                    M[me, d, c, e]))
            s_, e = np.nonzero(M[:, me, c, :])
            give_back.append(rotated(s_, ret_base[s_, c] + send_pos[s_, me, c, e], recv_pos[s_, me, c, e],
                                     M[s_, me, c, e]))
            ends.append(np.cumsum(M[:, me, c, :].sum(axis=0)).tolist())
    groups = [None] * C
    if layout == "source" and regroup != "never":
        L = M[:, me]                                          # [source, chunk, expert]
        take = L.sum(axis=(0, 2)) > 0 if regroup == "always" else _regroup_pays_chunks(L, hidden, inter, row_bytes)
        for c in np.nonzero(take)[0]:
            groups[c] = np.cumsum(L[:, c, :].sum(axis=0)).tolist()
    return BlockPlan(in_cap=int(R.sum(axis=1).max()), ret_cap=int(S.sum(axis=1).max()),
                     in_base=in_base[me].tolist(), in_rows=R[me].tolist(),
                     ret_base=ret_base[me].tolist(), ret_rows=S[me].tolist(),
                     gemm_ends=ends, sources=1 if layout == "expert" else G, dispatch=dispatch,
                     give_back=give_back, regroup=groups)


class PeerBuffers:
    """One device buffer per rank of the group, mapped into every other rank
    (CUDA IPC; one process per GPU), so a rank can write its blocks straight
    into a peer's buffer with copy-engine transfers over NVLink.  Each buffer
    starts with FLAG_BYTES of arrival flags (one uint64 per rank, zeroed before
    the buffer is shared); data regions follow.  `ensure` is collective: every
    rank calls it with the same byte count (derived from data all ranks hold)
    and the buffers are re-exported only when they must grow."""

    FLAG_BYTES = 4096

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local: torch.Tensor | None = None
        self.ptrs: list[int] = []
        self._bases: list[int | None] = []

    def ensure(self, nbytes: int, dev: torch.device) -> list[int]:
        """Buffer pointers of every rank (data regions start FLAG_BYTES in)."""
        if self.local is not None and self.local.numel() >= nbytes + self.FLAG_BYTES:
            return self.ptrs
        import ctypes
        from . import _lib
        self.release()
        cap = (int((nbytes + self.FLAG_BYTES) * 1.25) + (2 << 20) - 1) // (2 << 20) * (2 << 20)
        self.local = torch.empty(cap, dtype=torch.uint8, device=dev)
        # flags start at zero; the handle exchange below orders this before any peer's signal
        self.local[:self.FLAG_BYTES].zero_()
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_uint64(0)
        _lib.call("mirai_ipc_export", self.local.data_ptr(), handle, ctypes.byref(off))
        infos: list = [None] * self.world
        dist.all_gather_object(infos, (bytes(handle), off.value), group=self.group)
        self.ptrs, self._bases = [], []
        for r, (h, o) in enumerate(infos):
            if r == self.rank:
                self.ptrs.append(self.local.data_ptr())
                self._bases.append(None)
                continue
            hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            p, b = _lib.c_vp(0), _lib.c_vp(0)
            _lib.call("mirai_ipc_import", hb, o, ctypes.byref(p), ctypes.byref(b))
            self.ptrs.append(p.value)
            self._bases.append(b.value)
        return self.ptrs

    def release(self) -> None:
        """Collective: unmap the peers' buffers and drop this rank's."""
        if self.local is None:
            return
        from . import _lib
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # nobody still writes into an old buffer
        for b in self._bases:
            if b:
                _lib.call("mirai_ipc_release", _lib.c_vp(b))
        dist.barrier(group=self.group)  # nobody still maps this rank's old buffer
        self.local, self.ptrs, self._bases = None, [], []


class ExpertParallelMoE:
    """The expert-parallel layer with a copy-engine exchange (transport "ipc").

    Same contract and result as ``ep_moe_forward``; the rows move differently:
    every rank maps every other rank's exchange buffer (``PeerBuffers``) and a
    token owner copies its rows straight into each owner's receive region
    (copy engines, no SMs), at the places ``exchange_blocks`` gives them; the
    owner copies the results straight back into the token owner's return
    region, in the order the token owner sent.

    ``layout="source"`` (default): one copy per peer and chunk; the owner's
    GEMMs take the G source segments of each expert (128-row blocks paired
    into tiles), or — where ``regroup_pays`` ("auto"; or "always"/"never") —
    first gather the chunk's rows expert-major and the results back.
    ``layout="expert"``: one copy per (peer, expert) block into an
    expert-major region, so the GEMMs see one segment per expert; a copy
    costs about 4 µs of copy-engine time, so this pays only with few blocks.
    With ``chunks`` > 1 the copies of one chunk run beside the GEMMs of
    another; ``copy_streams`` > 1 spreads a chunk's copies over that many side
    streams by peer, so several are in flight at once.
    Arrival is signalled with flags in the peers' buffers: after a chunk's
    copies a rank stores the exchange's epoch into its slot of every peer's
    flag array, and a consumer's stream waits (bounded) for all its slots to
    reach the epoch before the GEMMs or the combine read the data."""

    def __init__(self, shard: ExpertShard, *, top_k: int, inter: int, group=None, chunks: int = 2,
                 ops: StepOps | None = None, copy_streams: int = 1, layout: str = "source",
                 regroup: str = "auto", check_device: bool = True):
        self.shard, self.top_k, self.inter, self.group = shard, top_k, inter, group
        self.chunks = max(1, int(chunks))
        self.ops = ops or CudaStepOps()
        self.buffers = PeerBuffers(group)
        self.comm: torch.cuda.Stream | None = None
        if layout not in ("expert", "source"):
            raise ValueError(f"layout must be 'expert' or 'source', not {layout!r}")
        self.layout = layout
        if regroup not in ("never", "auto", "always"):
            raise ValueError(f"regroup must be 'never', 'auto' or 'always', not {regroup!r}")
        self.regroup = regroup
        self.n_copy_streams = max(1, int(copy_streams))
        self.copy_streams: list[torch.cuda.Stream] = []  # side streams when n_copy_streams > 1
        self.epoch = 0  # exchanges so far; the same sequence on every rank
        self._gen = 0   # forwards so far (a training state is valid until the next one)
        # read the device error word at the host sync each call already makes (the count read)
        self.check_device = bool(check_device)
        # optional probe: called as on_phase(name, stream) at phase boundaries
        self.on_phase = None

    def close(self) -> None:
        self.buffers.release()

    def check(self) -> None:
        """Raise ``MiraiError`` if a kernel or an arrival wait of this device
        recorded an error since the last check (a wait gives up after 2 s and
        leaves partly arrived rows behind it).  ``forward`` does this at the
        start of every call (``check_device=True``); call it after the last
        layer of a step, or call ``ops.check_device()``."""
        from . import ops as _ops
        code, info = _ops.device_status()
        if code:
            raise _ops._lib.MiraiError(code, f"expert-parallel layer on rank {self.shard.rank}: device error at "
                                             f"site {info} (700 + peer slot: an arrival wait that gave up)")

    def _copy_blocks(self, blocks, peer_base: list[int], my_base: int, row_bytes: int, stream) -> None:
        """Issue one block list of a ``BlockPlan`` on ``stream`` (or spread over
        the side copy streams by peer, joined back into ``stream``)."""
        import numpy as np
        from . import _lib
        peer, peer_row, my_row, rows = blocks
        if len(rows) == 0:
            return
        rb = np.uint64(row_bytes)
        dst = np.asarray(peer_base, dtype=np.uint64)[peer] + peer_row.astype(np.uint64) * rb
        src = np.uint64(my_base) + my_row.astype(np.uint64) * rb
        nbytes = rows.astype(np.uint64) * rb
        n = len(self.copy_streams)
        if n == 0:
            _lib.call("mirai_copy_blocks", len(rows), dst.ctypes.data, src.ctypes.data, nbytes.ctypes.data,
                      _lib.c_vp(stream.cuda_stream))
            return
        start = torch.cuda.Event()
        start.record(stream)
        for i, side in enumerate(self.copy_streams):
            sel = (peer % n) == i
            if not sel.any():
                continue
            side.wait_event(start)
            d, s_, b = (np.ascontiguousarray(a[sel]) for a in (dst, src, nbytes))
            _lib.call("mirai_copy_blocks", len(b), d.ctypes.data, s_.ctypes.data, b.ctypes.data,
                      _lib.c_vp(side.cuda_stream))
            done = torch.cuda.Event()
            done.record(side)
            stream.wait_event(done)

    def forward(self, tokens: torch.Tensor, logits: torch.Tensor, local_weights: Any, *, train: bool = False,
                lora=None):
        """The layer for this rank's tokens (``ep_moe_forward``'s contract).

        ``train=True`` returns ``(out, state)`` for ``backward``: the owners
        keep the gate/up of the rows they received, and the expert outputs
        stay where they came back, in this rank's exchange buffer, so one
        instance serves one layer of a training step (a second forward on the
        same instance before ``backward`` makes ``backward`` refuse the state).
        ``lora`` (``ops.DownLoRA`` over this rank's experts) adds the adapter
        on w2 (training only)."""
        if lora is not None and not train:
            raise ValueError("the expert-parallel forward takes a LoRA adapter in training (train=True)")
        ops, shard, k = self.ops, self.shard, self.top_k
        G, E, El, me = shard.world, shard.num_experts, shard.local, shard.rank
        T, H = tokens.shape
        dev = tokens.device
        if G == 1:
            return ep_moe_forward(tokens, logits, local_weights, shard=shard, top_k=k, inter=self.inter, ops=ops,
                                  train=train, lora=lora)
        self._gen += 1
        if self.comm is None:
            self.comm = torch.cuda.Stream(device=dev)
            if self.n_copy_streams > 1:
                self.copy_streams = [torch.cuda.Stream(device=dev) for _ in range(self.n_copy_streams)]
        comp, comm = torch.cuda.current_stream(dev), self.comm
        mark = self.on_phase or (lambda name, stream: None)
        mark("start", comp)
        C = self.chunks
        bounds = [((T * c) // C, (T * (c + 1)) // C) for c in range(C)]
        routed = []
        for b, e in bounds:
            idx, tw = ops.route(logits[b:e], k)
            routed.append((tw, ops.plan(idx, E), idx.numel()))
        mark("route+plan", comp)
        # every rank's rows per (destination, chunk, local expert): one gather, one host read
        mine = torch.stack([p[1].counts.view(G, El) for p in routed], dim=1).contiguous()  # [dest, chunk, expert]
        allm = torch.empty((G,) + tuple(mine.shape), dtype=mine.dtype, device=dev)        # [source, dest, chunk, expert]
        dist.all_gather_into_tensor(allm, mine, group=self.group)
        row_bytes = H * tokens.element_size()
        counts = allm.cpu().numpy()
        if self.check_device and tokens.is_cuda:
            # The stream has just drained up to the count gather: an arrival wait of an earlier call
            # that gave up (a peer more than 2 s late) or a failed kernel check is reported here,
            # before this call moves any row.  The last call's status is read by check().
            self.check()
        # the permutes run on the GPU while this host plans the exchange
        prep = [(tw, plan, ops.permute(tokens[b:e], plan.sorted_token_indices))
                for (tw, plan, _), (b, e) in zip(routed, bounds)]
        check_counts(counts, me, [n for _, _, n in routed])
        plan = exchange_blocks(counts, me, self.layout, regroup=self.regroup, hidden=H,
                               inter=self.inter, row_bytes=row_bytes)
        in_cap = (plan.in_cap * row_bytes + 255) // 256 * 256
        ret_cap = (plan.ret_cap * row_bytes + 255) // 256 * 256
        F = PeerBuffers.FLAG_BYTES
        # regions: received rows | returned expert outputs | (training) returned dX rows
        ptrs = self.buffers.ensure(in_cap + ret_cap * (2 if train else 1), dev)
        local = self.buffers.local[F:]
        data = [p + F for p in ptrs]
        ret = [p + in_cap for p in data]
        x_in = local[:in_cap].view(tokens.dtype)[: sum(plan.in_rows) * H].view(-1, H)
        y_ret = local[in_cap:in_cap + ret_cap].view(tokens.dtype)[: sum(plan.ret_rows) * H].view(-1, H)
        # segment ends per chunk: the received layout's, or the regrouped experts'
        seg_ends = [plan.gemm_ends[c] if plan.regroup[c] is None else plan.regroup[c] for c in range(C)]
        flat_ends = torch.tensor([v for ends in seg_ends for v in ends], dtype=torch.int32).to(dev, non_blocking=True)
        offs_dev, pos = [], 0
        for ends in seg_ends:
            offs_dev.append(flat_ends[pos:pos + len(ends)])
            pos += len(ends)
        mark("count gather + host read", comp)

        ex = _Exchange(self, ptrs, comp)
        ready = torch.cuda.Event()
        ready.record(comp)
        comm.wait_event(ready)
        landed = []
        for c in range(C):
            xs = prep[c][2]
            xs.record_stream(comm)
            self._copy_blocks(plan.dispatch[c], data, xs.data_ptr(), row_bytes, comm)
            landed.append(ex.arrived(comm))
            mark(f"dispatch copies + arrival, chunk {c}", comm)
        returned, saved = [], []
        kw = {"lora": lora} if lora is not None else {}
        # NF4 keys decoded once for this layer where that pays (kept for the backward when training)
        local_weights, staged = _stage(ops, local_weights, sum(plan.in_rows), train)
        if not train:
            staged = None
        for c in range(C):
            ex.wait(landed[c])
            rows_c = plan.in_rows[c]
            xc = x_in[plan.in_base[c]:plan.in_base[c] + rows_c]
            sv = None
            if not rows_c:
                yc = xc
            elif plan.regroup[c] is None:
                if train:
                    yc, sv = ops.experts_train(xc, offs_dev[c], local_weights, self.inter, sources=plan.sources, **kw)
                else:
                    yc = ops.experts(xc, offs_dev[c], local_weights, self.inter, sources=plan.sources)
            else:
                # expert-major for the GEMMs (no tile cut at a source boundary), then back
                order, inverse = regroup_order(allm[:, me, c, :], rows_c)
                xe = ops.permute(xc, order)
                if train:
                    ye, inner = ops.experts_train(xe, offs_dev[c], local_weights, self.inter, **kw)
                    sv = ("regrouped", order, inverse, offs_dev[c], inner)
                else:
                    ye = ops.experts(xe, offs_dev[c], local_weights, self.inter)
                yc = ops.permute(ye, inverse)
            saved.append(sv)
            mark(f"gate/up + down GEMMs, chunk {c}", comp)
            done = torch.cuda.Event()
            done.record(comp)
            comm.wait_event(done)
            yc.record_stream(comm)
            self._copy_blocks(plan.give_back[c], ret, yc.data_ptr(), row_bytes, comm)
            returned.append(ex.arrived(comm))
            mark(f"return copies + arrival, chunk {c}", comm)
        out = torch.empty((T, H), dtype=tokens.dtype, device=dev)
        y_back = []
        for c, (b, e) in enumerate(bounds):
            ex.wait(returned[c])
            yb = y_ret[plan.ret_base[c]:plan.ret_base[c] + plan.ret_rows[c]]
            y_back.append(yb)
            if e > b:
                out[b:e] = ops.combine(yb, prep[c][1].inverse_order, prep[c][0], k, tokens.dtype)
        mark("combine", comp)
        if not train:
            return out
        dx_ret = local[in_cap + ret_cap:in_cap + 2 * ret_cap].view(tokens.dtype)[: sum(plan.ret_rows) * H].view(-1, H)
        return out, IPCTrainState(gen=self._gen, bounds=bounds, prep=[(p[0], p[1]) for p in prep], plan=plan,
                                  offs=offs_dev, saved=saved, y_back=y_back, x_in=x_in, dx_ret=dx_ret,
                                  ptrs=list(ptrs), data=data, ret2=[p + in_cap + ret_cap for p in data],
                                  row_bytes=row_bytes, top_k=k, hidden=H, dtype=tokens.dtype, staged=staged)

    def backward(self, grad_out: torch.Tensor, state: "IPCTrainState", local_weights: Any, *,
                 lora=None) -> tuple[torch.Tensor, torch.Tensor]:
        """dX of ``forward(train=True)``: grad_out [T_r, H] -> (dx [T_r, H],
        d_top_weights fp32 [T_r, k]), with the rank's adapter gradients in
        ``lora``.  Collective.  Per chunk, as ``ep_moe_backward`` does, over
        the copy-engine exchange: the combine backward here; the gradient rows
        copied into the owners' receive regions (the forward's rows are no
        longer needed there: every owner finished its GEMMs on them before the
        last expert outputs came back); the owner's dX GEMMs on the gate/up it
        kept; dX rows copied back into the third region of the token owner's
        buffer; the permute backward sums each token's routes."""
        ops, shard = self.ops, self.shard
        if shard.world == 1:
            return ep_moe_backward(grad_out, state, local_weights, shard=shard, inter=self.inter, ops=ops, lora=lora)
        if not isinstance(state, IPCTrainState) or state.gen != self._gen:
            raise RuntimeError("expert-parallel backward: this layer's exchange buffers were used by another forward "
                               "since the training forward (use one ExpertParallelMoE per layer in training)")
        if lora is not None and lora.compute_grads:
            lora.grad_a = lora.grad_b = None  # summed over this call's chunks
        dev = grad_out.device
        comp, comm = torch.cuda.current_stream(dev), self.comm
        mark = self.on_phase or (lambda name, stream: None)
        plan, k, H = state.plan, state.top_k, state.hidden
        T = grad_out.shape[0]
        ex = _Exchange(self, state.ptrs, comp)
        dx = torch.empty((T, H), dtype=state.dtype, device=dev)
        dw = torch.empty((T, k), dtype=torch.float32, device=dev)
        local_weights = _weights_for(state.staged, local_weights)
        state.staged = None
        sent = []
        for c, (b, e) in enumerate(state.bounds):
            tw, dplan = state.prep[c]
            if e > b:
                gy, gw = ops.combine_backward(grad_out[b:e], state.y_back[c], dplan.inverse_order, tw, k)
                dw[b:e] = gw
            else:
                gy = torch.empty((0, H), dtype=state.y_back[c].dtype, device=dev)
            done = torch.cuda.Event()
            done.record(comp)
            comm.wait_event(done)
            gy.record_stream(comm)
            self._copy_blocks(plan.dispatch[c], state.data, gy.data_ptr(), state.row_bytes, comm)
            sent.append(ex.arrived(comm))
            mark(f"combine backward + gradient copies, chunk {c}", comm)
        kw = {"lora": lora} if lora is not None else {}
        returned = []
        for c in range(len(state.bounds)):
            ex.wait(sent[c])
            rows_c = plan.in_rows[c]
            gc = state.x_in[plan.in_base[c]:plan.in_base[c] + rows_c]
            if rows_c:
                dc = ops.experts_backward(gc, state.offs[c], local_weights, self.inter, plan.sources,
                                          state.saved[c], **kw)
            else:
                dc = gc
            mark(f"dX GEMMs, chunk {c}", comp)
            done = torch.cuda.Event()
            done.record(comp)
            comm.wait_event(done)
            dc.record_stream(comm)
            self._copy_blocks(plan.give_back[c], state.ret2, dc.data_ptr(), state.row_bytes, comm)
            returned.append(ex.arrived(comm))
        for c, (b, e) in enumerate(state.bounds):
            ex.wait(returned[c])
            if e > b:
                rows = state.dx_ret[plan.ret_base[c]:plan.ret_base[c] + plan.ret_rows[c]]
                dx[b:e] = ops.combine(rows, state.prep[c][1].inverse_order, None, k, state.dtype)
        mark("dX un-permute", comp)
        return dx, dw


class _Exchange:
    """Arrival signalling of one layer's copy-engine exchanges: ``arrived``
    stores the next epoch into this rank's slot of every peer's flags after a
    block list's copies; ``wait`` holds the compute stream (bounded, 2 s)
    until every peer's slot in this rank's flags reaches an epoch."""

    def __init__(self, layer: "ExpertParallelMoE", ptrs: list[int], comp):
        from . import _lib
        self.layer, self.ptrs, self.comp, self._lib = layer, ptrs, comp, _lib
        G, me = layer.shard.world, layer.shard.rank
        self.slots = (_lib.c_vp * G)(*[None if d == me else ptrs[d] + 8 * me for d in range(G)])

    def arrived(self, stream):
        """Signal this exchange to every peer; return (epoch, event after the local copy)."""
        lay = self.layer
        lay.epoch += 1
        self._lib.call("mirai_ep_signal", self.slots, lay.shard.world, lay.epoch, self._lib.c_vp(stream.cuda_stream))
        ev = torch.cuda.Event()
        ev.record(stream)
        return lay.epoch, ev

    def wait(self, arrival):
        epoch, ev = arrival
        self.comp.wait_event(ev)  # this rank's own block
        lay = self.layer
        self._lib.call("mirai_ep_wait", self._lib.c_vp(self.ptrs[lay.shard.rank]), lay.shard.world, lay.shard.rank,
                       epoch, self._lib.c_vp(self.comp.cuda_stream))


@dataclass
class IPCTrainState:
    """What ``ExpertParallelMoE.backward`` needs from ``forward(train=True)``."""

    gen: int                 # the layer's forward count when this state was made
    bounds: list             # [(begin, end)] token range of each chunk
    prep: list               # per chunk: (route weights, dispatch plan)
    plan: "BlockPlan"
    offs: list               # per chunk: segment ends of the owner's GEMMs (device)
    saved: list              # per chunk: what the owner's GEMMs kept (None without rows)
    y_back: list             # per chunk: the expert outputs that came back (views of the buffer)
    x_in: torch.Tensor       # this rank's receive region (the gradient rows land here)
    dx_ret: torch.Tensor     # this rank's dX return region
    ptrs: list               # every rank's buffer (flags first)
    data: list               # every rank's receive region
    ret2: list               # every rank's dX return region
    row_bytes: int
    top_k: int
    hidden: int
    dtype: torch.dtype
    staged: tuple | None = None  # (the local NF4 keys, their bf16 copies) when the forward staged them
