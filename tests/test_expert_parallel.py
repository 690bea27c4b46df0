"""Expert-parallel exchange on CPU ranks (gloo, world size 2 and 4).

The exchange logic of mirai_b200.expert_parallel (count matrices and split
sizes, the all-to-all to the expert owners, the source-major segments the
owner's GEMMs take, the return trip and the final weighted combine) runs for
real over torch.distributed; the per-rank steps are the
oracle's (the CUDA kernels need a GPU).  The concatenated per-rank outputs
must equal the single-process oracle layer, and ranks without tokens or
experts without rows must not break the collective.
"""

import os
import types

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as om
from oracle import quant as oq


class OracleStepOps:
    """The per-rank steps restated on the CPU with the oracle."""

    def route(self, logits, top_k):
        idx, w = om.route_topk(logits.numpy(), top_k)
        return torch.from_numpy(idx.astype(np.int64)), torch.from_numpy(w.astype(np.float32))

    def plan(self, top_indices, num_experts):
        p = om.dispatch_plan(top_indices.numpy(), num_experts)
        return types.SimpleNamespace(**{k: torch.from_numpy(v) for k, v in p.items()})

    def permute(self, x, sorted_token_indices):
        return torch.from_numpy(om.permute(x.numpy(), sorted_token_indices.numpy()))

    def experts(self, x_sorted, offsets, weights, inter, sources=1):
        # segment s*E + e holds source s's rows for expert e: gather each expert's
        # rows in source order (one block per expert, as the single-process layer
        # has them, so numpy's blocking and summation order match), run, scatter back
        x, ends = x_sorted.numpy(), offsets.numpy().astype(np.int64)
        E = ends.size // sources
        starts = np.concatenate([[0], ends[:-1]])
        order = [np.arange(starts[s_ * E + e], ends[s_ * E + e]) for e in range(E) for s_ in range(sources)]
        perm = np.concatenate(order) if order else np.zeros(0, np.int64)
        per_expert = np.cumsum([sum(ends[s_ * E + e] - starts[s_ * E + e] for s_ in range(sources)) for e in range(E)])
        y = om.expert_ffn_forward(x[perm], per_expert, *weights, bf16=True)
        out = np.empty_like(y)
        out[perm] = y
        return torch.from_numpy(out)

    def _by_expert(self, offsets, sources):
        ends = offsets.numpy().astype(np.int64)
        E = ends.size // sources
        starts = np.concatenate([[0], ends[:-1]])
        order = [np.arange(starts[s_ * E + e], ends[s_ * E + e]) for e in range(E) for s_ in range(sources)]
        perm = np.concatenate(order) if order else np.zeros(0, np.int64)
        per_expert = np.cumsum([sum(ends[s_ * E + e] - starts[s_ * E + e] for s_ in range(sources))
                                for e in range(E)])
        return perm, per_expert

    def experts_train(self, x_sorted, offsets, weights, inter, sources=1):
        perm, per_expert = self._by_expert(offsets, sources)
        y, mids = om.expert_ffn_forward(x_sorted.numpy()[perm], per_expert, *weights, bf16=True, keep=True)
        out = np.empty_like(y)
        out[perm] = y
        return torch.from_numpy(out), (perm, per_expert, mids)

    def experts_backward(self, grad_y, offsets, weights, inter, sources, saved):
        perm, per_expert, mids = saved
        dxs = om.expert_ffn_backward(grad_y.numpy()[perm], per_expert, *weights, mids, bf16=True)
        out = np.empty_like(dxs)
        out[perm] = dxs
        return torch.from_numpy(out)

    def combine_backward(self, grad_out, y_sorted, inverse_order, top_weights, top_k):
        """dispatch_ops.py:36-44 for bf16 tensors: grad_y = bf16(g * w), grad_w = <g, y> (fp32)."""
        g, y = grad_out.numpy(), y_sorted.numpy()
        inv = inverse_order.numpy().reshape(-1, top_k)
        w = top_weights.numpy()
        gy = np.zeros_like(y)
        gw = np.zeros(w.shape, np.float32)
        for t in range(inv.shape[0]):
            for j in range(top_k):
                gy[inv[t, j]] = oq.bf16_round(g[t] * w[t, j])
                gw[t, j] = np.dot(g[t].astype(np.float64), y[inv[t, j]].astype(np.float64))
        return torch.from_numpy(gy), torch.from_numpy(gw)

    def combine(self, y_sorted, inverse_order, top_weights, top_k, out_dtype):
        y = y_sorted.numpy()
        inv = inverse_order.numpy().reshape(-1, top_k)
        T, H = inv.shape[0], y.shape[1]
        out = np.zeros((T, H), np.float32)
        w = np.ones((T, top_k), np.float32) if top_weights is None else top_weights.numpy()
        for t in range(T):
            for j in np.argsort(inv[t], kind="stable"):  # ascending sorted position
                out[t] += y[inv[t, j]] * w[t, j]
        return torch.from_numpy(oq.bf16_round(out))


def _problem(T, H, E, k, I, seed):
    rng = np.random.default_rng(seed)
    x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    logits = (rng.standard_normal((T, E)) * 1.5).astype(np.float32)
    ws = [oq.bf16_round((rng.standard_normal(s) * 0.05).astype(np.float32)) for s in ((E, I, H), (E, I, H), (E, H, I))]
    return x, logits, ws


def _rank_main(rank, world, rdv, cfg, results):
    dist.init_process_group("gloo", init_method=f"file://{rdv}", rank=rank, world_size=world)
    try:
        from mirai_b200.expert_parallel import ExpertShard, ep_moe_forward, shard_tokens
        T, H, E, k, I, seed, token_split, chunks = cfg
        x, logits, ws = _problem(T, H, E, k, I, seed)
        shard = ExpertShard(E, world, rank)
        b, e = token_split[rank] if token_split else shard_tokens(T, world, rank)
        lo, hi = shard.first, shard.first + shard.local
        out = ep_moe_forward(torch.from_numpy(x[b:e]), torch.from_numpy(logits[b:e]),
                             tuple(w[lo:hi] for w in ws), shard=shard, top_k=k, inter=I, ops=OracleStepOps(),
                             chunks=chunks)
        results[rank] = (b, e, out.numpy())
    finally:
        dist.destroy_process_group()


def _rendezvous():
    """A fresh rendezvous file for one process group (file:// init: no TCP port
    to collide with another test's group)."""
    import tempfile
    fd, path = tempfile.mkstemp(prefix="mirai_pg_")
    os.close(fd)
    return path


def _run(world, cfg):
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _rendezvous(), cfg, results), nprocs=world, start_method="spawn")
        return dict(results)


@pytest.mark.parametrize("world,cfg", [
    (2, (96, 64, 8, 2, 128, 3, None, 1)),
    (4, (150, 64, 8, 3, 64, 5, None, 1)),
    (2, (80, 32, 4, 2, 64, 7, [(0, 0), (0, 80)], 1)),  # rank 0 has no tokens
    (2, (97, 64, 8, 2, 64, 9, None, 3)),               # three chunks per rank
    (4, (60, 32, 8, 2, 64, 11, [(0, 40), (40, 41), (41, 41), (41, 60)], 2)),  # ragged shards and chunks
])
def test_expert_parallel_matches_single_process_layer(world, cfg):
    T, H, E, k, I, seed, _, _ = cfg
    res = _run(world, cfg)
    x, logits, ws = _problem(T, H, E, k, I, seed)
    idx, w = om.route_topk(logits, k)
    ref = om.moe_forward(x, idx, w, *ws, bf16=True)
    got = np.zeros_like(ref)
    for r in range(world):
        b, e, out = res[r]
        got[b:e] = out
    np.testing.assert_array_equal(got, ref)


def test_shard_arithmetic():
    from mirai_b200.expert_parallel import ExpertShard, shard_tokens
    assert [shard_tokens(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    s = ExpertShard(128, 8, 3)
    assert (s.local, s.first) == (16, 48)
    with pytest.raises(ValueError):
        ExpertShard(10, 4, 0)


@pytest.mark.parametrize("layout", ["expert", "source"])
@pytest.mark.parametrize("G,C,El,seed", [(2, 1, 4, 0), (4, 2, 3, 1), (8, 2, 16, 2), (3, 3, 2, 3), (2, 2, 2, 4)])
def test_exchange_blocks_round_trip(G, C, El, seed, layout):
    """Every rank's dispatch and return block lists, run on simulated memory,
    put each owner's receive rows expert-major (source order inside an expert)
    or source-major (expert order inside a source), and bring every source's
    rows back in its send order."""
    from mirai_b200.expert_parallel import exchange_blocks
    rng = np.random.default_rng(seed)
    M = rng.integers(0, 6, size=(G, G, C, El))
    M[0, :, 0, :] = 0             # a source with nothing in one chunk
    M[:, G - 1, C - 1, 0] = 0     # an expert that gets nothing in one chunk
    if seed == 4:
        M[:] = 0                  # an empty layer
    plans = [exchange_blocks(M, r, layout) for r in range(G)]
    assert len({(p.in_cap, p.ret_cap) for p in plans}) == 1
    for r, p in enumerate(plans):  # rotated schedule: peers visited from r upwards (mod G)
        for blocks in p.dispatch + p.give_back:
            steps = (blocks[0] - r) % G
            assert np.all(np.diff(steps) >= 0)

    def label(s, d, c, e, i):
        return (((s * G + d) * C + c) * El + e) * 1000 + i

    send = [[np.array([label(s, d, c, e, i) for d in range(G) for e in range(El) for i in range(M[s, d, c, e])],
                      dtype=np.int64) for c in range(C)] for s in range(G)]
    recv = [np.full(plans[0].in_cap, -1, np.int64) for _ in range(G)]
    for s in range(G):
        for c in range(C):
            for peer, prow, mrow, rows in zip(*plans[s].dispatch[c]):
                assert rows > 0
                recv[peer][prow:prow + rows] = send[s][c][mrow:mrow + rows]
    for d in range(G):
        p = plans[d]
        assert p.in_base == np.concatenate([[0], np.cumsum(p.in_rows)[:-1]]).tolist()
        for c in range(C):
            got = recv[d][p.in_base[c]:p.in_base[c] + p.in_rows[c]]
            if layout == "expert":
                want = [label(s, d, c, e, i) for e in range(El) for s in range(G) for i in range(M[s, d, c, e])]
                assert p.gemm_ends[c] == np.cumsum(M[:, d, c, :].sum(axis=0)).tolist() and p.sources == 1
            else:
                want = [label(s, d, c, e, i) for s in range(G) for e in range(El) for i in range(M[s, d, c, e])]
                assert p.gemm_ends[c] == np.cumsum(M[:, d, c, :].reshape(-1)).tolist() and p.sources == G
                assert len(p.dispatch[c][0]) == len(set(p.dispatch[c][0].tolist()))  # one copy per peer
            assert got.tolist() == want
    ret = [np.full(plans[0].ret_cap, -1, np.int64) for _ in range(G)]
    for d in range(G):
        p = plans[d]
        for c in range(C):
            yc = recv[d][p.in_base[c]:p.in_base[c] + p.in_rows[c]]   # the owner's output rows, same order
            for peer, prow, mrow, rows in zip(*p.give_back[c]):
                ret[peer][prow:prow + rows] = yc[mrow:mrow + rows]
    for s in range(G):
        p = plans[s]
        for c in range(C):
            assert ret[s][p.ret_base[c]:p.ret_base[c] + p.ret_rows[c]].tolist() == send[s][c].tolist()


@pytest.mark.parametrize("G,El,seed", [(2, 4, 0), (8, 16, 1), (3, 5, 2)])
def test_regroup_order_is_expert_major(G, El, seed):
    """Rows received source-major, taken in ``order``, are expert-major with
    source order kept inside an expert; ``inverse`` restores the received order."""
    from mirai_b200.expert_parallel import regroup_order
    rng = np.random.default_rng(seed)
    L = rng.integers(0, 7, size=(G, El))
    L[0, :] = 0
    L[:, El - 1] = 0
    labels = np.array([s * 1000 * El + e * 1000 + i for s in range(G) for e in range(El) for i in range(L[s, e])])
    order, inverse = regroup_order(torch.from_numpy(L).to(torch.int32), int(L.sum()))
    got = labels[order.numpy()]
    want = [s * 1000 * El + e * 1000 + i for e in range(El) for s in range(G) for i in range(L[s, e])]
    assert got.tolist() == want
    assert np.array_equal(got[inverse.numpy()], labels)


def test_regroup_cost_rule():
    """The owner regroups where cut tiles cost more than moving the rows twice:
    ~64-row segments from each of 8 sources (paired 128-row blocks half
    empty), not c4's shapes at 2 GPUs (~1024 rows per source and expert)."""
    from mirai_b200.expert_parallel import exchange_blocks, regroup_pays
    rng = np.random.default_rng(0)
    H, I = 4096, 1536
    assert regroup_pays(64 + rng.integers(-16, 16, size=(8, 16)), H, I, 2 * H)
    assert not regroup_pays(1024 + rng.integers(-32, 32, size=(2, 64)), H, I, 2 * H)
    M = 64 + rng.integers(-16, 16, size=(8, 8, 2, 16))
    p = exchange_blocks(M, 3, "source", regroup="auto", hidden=H, inter=I, row_bytes=2 * H)
    assert all(r is not None for r in p.regroup)
    assert p.regroup[1] == np.cumsum(M[:, 3, 1, :].sum(axis=0)).tolist()
    assert all(r is None for r in exchange_blocks(M, 3, "source").regroup)


class CorruptCountsOps(OracleStepOps):
    """A rank whose dispatch plan reports one routed row more than it permuted."""

    def plan(self, top_indices, num_experts):
        p = super().plan(top_indices, num_experts)
        p.counts = p.counts.clone()
        p.counts[0] += 1
        return p


def _fault_rank_main(rank, world, rdv, mode, results):
    import time
    from datetime import timedelta
    dist.init_process_group("gloo", init_method=f"file://{rdv}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    try:
        from mirai_b200.expert_parallel import ExpertShard, ep_moe_forward, shard_tokens
        T, H, E, k, I = 64, 32, 4, 2, 64
        x, logits, ws = _problem(T, H, E, k, I, 3)
        shard = ExpertShard(E, world, rank)
        b, e = shard_tokens(T, world, rank)
        lo, hi = shard.first, shard.first + shard.local
        if mode == "absent" and rank == 1:
            results[rank] = ("left", 0.0)  # this rank never joins the layer's collectives
            return
        ops = CorruptCountsOps() if (mode == "corrupt" and rank == 1) else OracleStepOps()
        t0 = time.monotonic()
        try:
            ep_moe_forward(torch.from_numpy(x[b:e]), torch.from_numpy(logits[b:e]), tuple(w[lo:hi] for w in ws),
                           shard=shard, top_k=k, inter=I, ops=ops)
            outcome = "ok"
        except ValueError:
            outcome = "ValueError"
        except Exception:  # the process group's timeout, or the peer's closed connection
            outcome = "error"
        results[rank] = (outcome, time.monotonic() - t0)
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run_fault(mode):
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_fault_rank_main, args=(2, _rendezvous(), mode, results), nprocs=2, start_method="spawn")
        return dict(results)


@pytest.mark.timeout(180)
def test_rank_that_never_joins_ends_in_an_error_not_a_hang():
    """Failure on the host: rank 1 leaves before the layer.  Rank 0's first
    collective of the layer ends in an error within the process group's
    timeout instead of waiting for ever."""
    res = _run_fault("absent")
    assert res[1][0] == "left"
    outcome, seconds = res[0]
    assert outcome == "error" and seconds < 60


@pytest.mark.timeout(180)
def test_corrupt_counts_are_rejected_before_rows_move():
    """A rank whose plan disagrees with its permuted rows raises ValueError
    after the count exchange, before the row exchange; its peer, waiting in the
    row exchange, ends in an error within the timeout."""
    res = _run_fault("corrupt")
    assert res[1][0] == "ValueError"
    outcome, seconds = res[0]
    assert outcome == "error" and seconds < 60


def test_check_counts():
    from mirai_b200.expert_parallel import check_counts
    M = np.ones((2, 2, 3, 4), np.int64)           # every rank sends 2 x 4 rows per chunk
    check_counts(M, 1, [8, 8, 8])
    with pytest.raises(ValueError, match="negative"):
        bad = M.copy()
        bad[0, 1, 2, 3] = -1
        check_counts(bad, 1, [8, 8, 8])
    with pytest.raises(ValueError, match="chunk 2"):
        check_counts(M, 1, [8, 8, 7])


def _bwd_rank_main(rank, world, rdv, cfg, results):
    dist.init_process_group("gloo", init_method=f"file://{rdv}", rank=rank, world_size=world)
    try:
        from mirai_b200.expert_parallel import ExpertShard, ep_moe_backward, ep_moe_forward, shard_tokens
        T, H, E, k, I, seed, token_split, chunks = cfg
        x, logits, ws = _problem(T, H, E, k, I, seed)
        g = oq.bf16_round(np.random.default_rng(seed + 100).standard_normal((T, H)).astype(np.float32))
        shard = ExpertShard(E, world, rank)
        b, e = token_split[rank] if token_split else shard_tokens(T, world, rank)
        local = tuple(w[shard.first:shard.first + shard.local] for w in ws)
        ops = OracleStepOps()
        out, st = ep_moe_forward(torch.from_numpy(x[b:e]), torch.from_numpy(logits[b:e]), local, shard=shard,
                                 top_k=k, inter=I, ops=ops, chunks=chunks, train=True)
        dx, dw = ep_moe_backward(torch.from_numpy(g[b:e]), st, local, shard=shard, inter=I, ops=ops)
        results[rank] = (b, e, out.numpy(), dx.numpy(), dw.numpy())
    finally:
        dist.destroy_process_group()


def _run_bwd(world, cfg):
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_bwd_rank_main, args=(world, _rendezvous(), cfg, results), nprocs=world,
                           start_method="spawn")
        return dict(results)


@pytest.mark.parametrize("world,cfg", [
    (2, (96, 64, 8, 2, 128, 3, None, 1)),
    (4, (150, 64, 8, 3, 64, 5, None, 2)),
    (2, (80, 32, 4, 2, 64, 7, [(0, 0), (0, 80)], 1)),  # rank 0 has no tokens
])
def test_expert_parallel_backward_equals_one_rank(world, cfg):
    """dX through the frozen experts across ranks (training forward keeps the
    owners' gate/up; gradient rows travel to the owners and dX rows back):
    the concatenated dX and route-weight gradients of world ranks equal the
    world-1 run of the same steps exactly, and the oracle's single-process
    backward within the bf16 tolerance (its un-permute sum rounds to bf16 after
    every route, as the reference's bf16 index_add does)."""
    res = _run_bwd(world, cfg)
    one = _run_bwd(1, cfg[:6] + (None, 1))
    T, H, E, k, I, seed = cfg[:6]
    dx = np.zeros((T, H), np.float32)
    dw = np.zeros((T, k), np.float32)
    out = np.zeros((T, H), np.float32)
    for r in range(world):
        b, e, o, d, w = res[r]
        out[b:e], dx[b:e], dw[b:e] = o, d, w
    np.testing.assert_array_equal(out, one[0][2])
    np.testing.assert_array_equal(dx, one[0][3])
    np.testing.assert_array_equal(dw, one[0][4])
    x, logits, ws = _problem(T, H, E, k, I, seed)
    g = oq.bf16_round(np.random.default_rng(seed + 100).standard_normal((T, H)).astype(np.float32))
    ridx, rw = om.route_topk(logits, k)
    rdx, rdw = om.moe_backward_dx(x, ridx, rw, *ws, g, bf16=True)
    assert om.rel_max_err(dx, rdx) < 2e-2
    assert om.rel_max_err(dw, rdw) < 1e-5


def test_owner_staging_helpers():
    """An owner's layer stages its keys through its step ops when they offer
    ``stage`` (the CUDA ops), keeps them as given otherwise (the oracle), and
    its backward reuses the forward's copies only for the same keys."""
    from mirai_b200.expert_parallel import _stage, _weights_for

    keys = (object(), object(), object())
    assert _stage(OracleStepOps(), keys, 10 ** 6, True) == (keys, None)

    class Staging:
        def stage(self, weights, rows, training):
            return tuple(("copy", w) for w in weights) if training else tuple(weights)

    copies, staged = _stage(Staging(), keys, 10 ** 6, True)
    assert copies == tuple(("copy", w) for w in keys) and staged == (keys, copies)
    assert _stage(Staging(), keys, 10 ** 6, False) == (keys, None)
    assert _weights_for(staged, keys) == copies
    other = (object(), keys[1], keys[2])
    assert _weights_for(staged, other) == other
    assert _weights_for(None, keys) == keys
