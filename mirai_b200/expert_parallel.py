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
expert, tiles visited expert-major), so the owner neither re-sorts nor
restores the order, and its output goes back through the reverse all-to-all
in the layout the token owner sent.  Per row the products are those of the
single-GPU layer, so the result is identical to it.  The reference runs MoE
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
        w1, w3, w2 = weights
        h = self.ops.gateup_swiglu(x_sorted, offsets, w1, w3, inter=inter, sources=sources)
        return self.ops.down(h, offsets, w2, hidden=x_sorted.shape[1], sources=sources)

    def combine(self, y_sorted, inverse_order, top_weights, top_k, out_dtype):
        return self.ops.combine(y_sorted, inverse_order, top_weights, out_dtype=out_dtype, top_k=top_k)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group) -> None:
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def ep_moe_forward(tokens: torch.Tensor, logits: torch.Tensor, local_weights: Any, *, shard: ExpertShard,
                   top_k: int, inter: int, group=None, ops: StepOps | None = None, chunks: int = 1,
                   comm_stream: torch.cuda.Stream | None = None) -> torch.Tensor:
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
    communication kernels (``ops.set_gemm_sm_limit``)."""
    ops = ops or CudaStepOps()
    G, E, El = shard.world, shard.num_experts, shard.local
    T, H = tokens.shape
    dev = tokens.device
    if G == 1:  # one rank owns every expert: no exchange
        idx, tw = ops.route(logits, top_k)
        plan = ops.plan(idx, E)
        xs = ops.permute(tokens, plan.sorted_token_indices)
        y = ops.experts(xs, plan.offsets, local_weights, inter)
        return ops.combine(y, plan.inverse_order, tw, top_k, tokens.dtype)
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
    comm = comm_stream if (C > 1 and tokens.is_cuda) else None

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

    def compute(c, x_recv):
        if x_recv.shape[0] == 0:
            return torch.empty((0, H), dtype=x_recv.dtype, device=dev)
        return ops.experts(x_recv, offs_dev[c], local_weights, inter, sources=G)

    def give_back(c, y_recv):
        keep(y_recv, comm)
        y_back = keep(torch.empty_like(prep[c][2]), comp if comm is not None else None)
        _a2a(y_back, y_recv, sc[c], rc[c], group)
        return y_back

    out = torch.empty((T, H), dtype=tokens.dtype, device=dev)
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


def shard_tokens(num_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous token shard (the first T % G ranks take one more)."""
    base, extra = divmod(num_tokens, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


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
    every rank maps every other rank's exchange buffer (``PeerBuffers``), a
    token owner copies each of its per-owner blocks straight into that owner's
    receive region (source-major, the layout the source-major GEMMs take) with
    one cudaMemcpyAsync (copy engines, no SMs), and the owner copies each
    source's results straight back into the token owner's return region.  A
    one-element NCCL all-reduce after the copies of a chunk, on the same
    stream, tells every rank that all of that chunk's blocks have landed.  With
    ``chunks`` > 1 the copies of one chunk run beside the GEMMs of another.
    Arrival is signalled with flags in the peers' buffers: after a chunk's
    copies a rank stores the exchange's epoch into its slot of every peer's
    flag array, and a consumer's stream waits (bounded) for all its slots to
    reach the epoch before the GEMMs or the combine read the data."""

    def __init__(self, shard: ExpertShard, *, top_k: int, inter: int, group=None, chunks: int = 2,
                 ops: StepOps | None = None):
        self.shard, self.top_k, self.inter, self.group = shard, top_k, inter, group
        self.chunks = max(1, int(chunks))
        self.ops = ops or CudaStepOps()
        self.buffers = PeerBuffers(group)
        self.comm: torch.cuda.Stream | None = None
        self.epoch = 0  # exchanges so far; the same sequence on every rank
        # optional probe: called as on_phase(name, stream) at phase boundaries
        self.on_phase = None

    def close(self) -> None:
        self.buffers.release()

    def _copy(self, dst: int, src: int, nbytes: int, stream) -> None:
        from . import _lib
        _lib.call("mirai_copy_async", _lib.c_vp(dst), _lib.c_vp(src), nbytes, _lib.c_vp(stream.cuda_stream))

    def forward(self, tokens: torch.Tensor, logits: torch.Tensor, local_weights: Any) -> torch.Tensor:
        ops, shard, k = self.ops, self.shard, self.top_k
        G, E, El, me = shard.world, shard.num_experts, shard.local, shard.rank
        T, H = tokens.shape
        dev = tokens.device
        if G == 1:
            return ep_moe_forward(tokens, logits, local_weights, shard=shard, top_k=k, inter=self.inter, ops=ops)
        if self.comm is None:
            self.comm = torch.cuda.Stream(device=dev)
        comp, comm = torch.cuda.current_stream(dev), self.comm
        mark = self.on_phase or (lambda name, stream: None)
        mark("start", comp)
        C = self.chunks
        bounds = [((T * c) // C, (T * (c + 1)) // C) for c in range(C)]
        prep = []
        for b, e in bounds:
            idx, tw = ops.route(logits[b:e], k)
            plan = ops.plan(idx, E)
            prep.append((tw, plan, ops.permute(tokens[b:e], plan.sorted_token_indices)))
        mark("route+plan+permute", comp)
        # every rank's rows per (destination, chunk, local expert): one gather, one host read
        mine = torch.stack([p[1].counts.view(G, El) for p in prep], dim=1).contiguous()  # [dest, chunk, expert]
        allm = torch.empty((G,) + tuple(mine.shape), dtype=mine.dtype, device=dev)      # [source, dest, chunk, expert]
        dist.all_gather_into_tensor(allm, mine, group=self.group)
        M = allm.cpu().numpy()
        n = M.sum(axis=3)                                   # rows [source, dest, chunk]
        R = n.sum(axis=0)                                   # rows each destination receives [dest, chunk]
        S = n.sum(axis=1)                                   # rows each source sends [source, chunk]
        row_bytes = H * tokens.element_size()
        in_cap = int(R.sum(axis=1).max()) * row_bytes       # receive region, the same on every rank
        ret_cap = int(S.sum(axis=1).max()) * row_bytes      # return region
        in_cap = (in_cap + 255) // 256 * 256
        F = PeerBuffers.FLAG_BYTES
        ptrs = self.buffers.ensure(in_cap + ret_cap, dev)
        local = self.buffers.local[F:]
        data = [p + F for p in ptrs]

        def in_base(d, c):      # rows before chunk c in d's receive region
            return int(R[d, :c].sum())

        def src_off(d, c, s):   # rows of sources < s in d's chunk-c receive block
            return int(n[:s, d, c].sum())

        def send_off(s, d, c):  # rows for destinations < d in s's chunk-c send order
            return int(n[s, :d, c].sum())

        def ret_base(s, c):     # rows before chunk c in s's return region
            return int(S[s, :c].sum())

        x_in = local[:in_cap].view(tokens.dtype)[: int(R[me].sum()) * H].view(-1, H)
        y_ret = local[in_cap:in_cap + ret_cap].view(tokens.dtype)[: int(S[me].sum()) * H].view(-1, H)
        offs = []
        for c in range(C):
            ends, run = [], 0
            for s in range(G):
                for e in range(El):
                    run += int(M[s, me, c, e])
                    ends.append(run)
            offs.append(ends)
        offs_dev = torch.tensor(offs, dtype=torch.int32).to(dev, non_blocking=True)
        mark("count gather + host read", comp)

        from . import _lib
        slots = (_lib.c_vp * G)(*[None if d == me else ptrs[d] + 8 * me for d in range(G)])

        def arrived(stream):
            """Signal this exchange to every peer; return (epoch, event after the local copy)."""
            self.epoch += 1
            _lib.call("mirai_ep_signal", slots, G, self.epoch, _lib.c_vp(stream.cuda_stream))
            ev = torch.cuda.Event()
            ev.record(stream)
            return self.epoch, ev

        def wait(arrival):
            epoch, ev = arrival
            comp.wait_event(ev)  # this rank's own block
            _lib.call("mirai_ep_wait", _lib.c_vp(ptrs[me]), G, me, epoch, _lib.c_vp(comp.cuda_stream))

        ready = torch.cuda.Event()
        ready.record(comp)
        comm.wait_event(ready)
        landed = []
        for c in range(C):
            xs = prep[c][2]
            xs.record_stream(comm)
            for d in range(G):
                rows = int(n[me, d, c])
                if rows:
                    dst = data[d] + (in_base(d, c) + src_off(d, c, me)) * row_bytes
                    self._copy(dst, xs.data_ptr() + send_off(me, d, c) * row_bytes, rows * row_bytes, comm)
            landed.append(arrived(comm))
            mark(f"dispatch copies + arrival, chunk {c}", comm)
        returned = []
        for c in range(C):
            wait(landed[c])
            rows_c = int(R[me, c])
            xc = x_in[in_base(me, c):in_base(me, c) + rows_c]
            yc = ops.experts(xc, offs_dev[c], local_weights, self.inter, sources=G) if rows_c else xc
            mark(f"gate/up + down GEMMs, chunk {c}", comp)
            done = torch.cuda.Event()
            done.record(comp)
            comm.wait_event(done)
            yc.record_stream(comm)
            for s in range(G):
                rows = int(n[s, me, c])
                if rows:
                    dst = data[s] + in_cap + (ret_base(s, c) + send_off(s, me, c)) * row_bytes
                    self._copy(dst, yc.data_ptr() + src_off(me, c, s) * row_bytes, rows * row_bytes, comm)
            returned.append(arrived(comm))
            mark(f"return copies + arrival, chunk {c}", comm)
        out = torch.empty((T, H), dtype=tokens.dtype, device=dev)
        for c, (b, e) in enumerate(bounds):
            wait(returned[c])
            if e > b:
                yb = y_ret[ret_base(me, c):ret_base(me, c) + int(S[me, c])]
                out[b:e] = ops.combine(yb, prep[c][1].inverse_order, prep[c][0], k, tokens.dtype)
        mark("combine", comp)
        return out
