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
import socket
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


def _rank_main(rank, world, port, cfg, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, cfg):
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), cfg, results), nprocs=world, start_method="spawn")
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
