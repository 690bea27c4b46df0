"""Measure the expert-parallel exchange on this machine (one process per GPU).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m mirai_b200.ep_probe bandwidth
    python -m torch.distributed.run ... -m mirai_b200.ep_probe blocks
    python -m mirai_b200.ep_probe gemms          # one GPU
    python -m torch.distributed.run ... -m mirai_b200.ep_probe phases --config c2|c4 [--layout expert|source]

``bandwidth``: bytes that cross NVLink per rank per second for NCCL's
all_to_all_single and for copy-engine transfers into peer-mapped buffers (the
layer's ``ipc`` transport), on equal-sized blocks.  ``blocks``: the same
copy-engine exchange (128 MB per rank) split into 1 to 128 copies per peer, on
one or two streams — the cost of a copy.  ``gemms`` (one GPU): the owner's GEMMs on source-major rows against the same
rows contiguous per expert.  ``phases [--layout expert|source]
[--copy-streams S] [--regroup never|auto|always]``: CUDA-event times between the phases of one
``ExpertParallelMoE`` layer (1 chunk) on rank 0, averaged over 10 layers after
3 warm-up layers.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def _bandwidth(dev, world, rank):
    from . import _lib
    from .expert_parallel import PeerBuffers
    res = {}
    for name, rows, H in (("c2-sized", 65536, 2048), ("c4-sized", 131072, 4096)):
        n = rows * world
        x = torch.randn(n, H, device=dev).to(torch.bfloat16)
        y = torch.empty_like(x)
        remote = n * H * 2 * (world - 1) / world
        for _ in range(3):
            dist.all_to_all_single(y, x)
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            dist.all_to_all_single(y, x)
        b.record()
        torch.cuda.synchronize()
        nccl_ms = a.elapsed_time(b) / 10
        # copy engines: block j of this rank's buffer goes to rank j's buffer at slot `rank`
        pb = PeerBuffers()
        ptrs = pb.ensure(x.numel() * 2, dev)
        data = [p + PeerBuffers.FLAG_BYTES for p in ptrs]
        slots = (_lib.c_vp * world)(*[None if j == rank else ptrs[j] + 8 * rank for j in range(world)])
        blk = rows * H * 2
        stream = torch.cuda.current_stream()
        epoch = [0]

        def exchange():  # the layer's mechanism: copies (rotated schedule), then arrival flags
            for j in ((rank + i) % world for i in range(world)):
                _lib.call("mirai_copy_async", _lib.c_vp(data[j] + rank * blk), _lib.c_vp(x.data_ptr() + j * blk),
                          blk, _lib.c_vp(stream.cuda_stream))
            epoch[0] += 1
            _lib.call("mirai_ep_signal", slots, world, epoch[0], _lib.c_vp(stream.cuda_stream))
            _lib.call("mirai_ep_wait", _lib.c_vp(ptrs[rank]), world, rank, epoch[0], _lib.c_vp(stream.cuda_stream))

        for _ in range(3):
            exchange()
        torch.cuda.synchronize()
        dist.barrier()
        a.record()
        for _ in range(10):
            exchange()
        b.record()
        torch.cuda.synchronize()
        ce_ms = a.elapsed_time(b) / 10
        from .ops import check_device
        check_device()
        pb.release()
        res[name] = {"bytes_per_rank_remote": int(remote),
                     "nccl_all_to_all_ms": round(nccl_ms, 3), "nccl_GBps": round(remote / nccl_ms / 1e6, 1),
                     "copy_engine_ms": round(ce_ms, 3), "copy_engine_GBps": round(remote / ce_ms / 1e6, 1)}
        del x, y
    return res


def _blocks(dev, world, rank):
    """Copy-engine exchange of a fixed byte count per peer, split into n equal
    blocks per peer (one cudaMemcpyAsync each), on 1 or 2 streams."""
    import numpy as np
    from . import _lib
    from .expert_parallel import PeerBuffers
    res = {}
    blk = 134_217_728 // world          # bytes this rank sends each peer: 128 MB per rank in all
    pb = PeerBuffers()
    ptrs = pb.ensure(blk * world, dev)
    data = [p + PeerBuffers.FLAG_BYTES for p in ptrs]
    x = torch.empty(blk * world, dtype=torch.uint8, device=dev)
    slots = (_lib.c_vp * world)(*[None if j == rank else ptrs[j] + 8 * rank for j in range(world)])
    main = torch.cuda.current_stream()
    sides = [torch.cuda.Stream() for _ in range(2)]
    epoch = [0]
    for nb in (1, 16, 64, 128):
        piece = blk // nb
        peers = [(rank + i) % world for i in range(world)]  # rotated schedule, as the layer's
        dst = np.array([data[j] + rank * blk + i * piece for j in peers for i in range(nb)], np.uint64)
        src = np.array([x.data_ptr() + j * blk + i * piece for j in peers for i in range(nb)], np.uint64)
        nbytes = np.full(len(dst), piece, np.uint64)
        peer = np.repeat(np.array(peers), nb)
        for ns in (1, 2):
            def exchange():
                start = torch.cuda.Event()
                start.record(main)
                for i in range(ns):
                    sel = (peer % ns) == i
                    st = sides[i] if ns > 1 else main
                    if ns > 1:
                        st.wait_event(start)
                    d, s_, b = (np.ascontiguousarray(a[sel]) for a in (dst, src, nbytes))
                    _lib.call("mirai_copy_blocks", len(b), d.ctypes.data, s_.ctypes.data, b.ctypes.data,
                              _lib.c_vp(st.cuda_stream))
                    if ns > 1:
                        ev = torch.cuda.Event()
                        ev.record(st)
                        main.wait_event(ev)
                epoch[0] += 1
                _lib.call("mirai_ep_signal", slots, world, epoch[0], _lib.c_vp(main.cuda_stream))
                _lib.call("mirai_ep_wait", _lib.c_vp(ptrs[rank]), world, rank, epoch[0], _lib.c_vp(main.cuda_stream))

            for _ in range(3):
                exchange()
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(10):
                exchange()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / 10
            remote = blk * (world - 1)
            res[f"{nb} blocks/peer, {ns} stream(s)"] = {"block_bytes": piece, "ms": round(ms, 3),
                                                        "GBps": round(remote / ms / 1e6, 1)}
    from .ops import check_device
    check_device()
    pb.release()
    return res


def _phases(dev, world, rank, config, layout="source", copy_streams=1, regroup="auto"):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    from .expert_parallel import ExpertParallelMoE, ExpertShard, shard_tokens
    cfg = dict(bench.CONFIGS[config], layers=1)
    strong = bench.CONFIGS[config].get("ep") == "strong"
    T_total = cfg["T"] if strong else cfg["T"] * world
    b, e = shard_tokens(T_total, world, rank)
    shard = ExpertShard(cfg["E"], world, rank)
    x, logits, stack = bench.make_ep_workload(cfg, dev, rank, shard, e - b)
    layer = ExpertParallelMoE(shard, top_k=cfg["k"], inter=cfg["I"], chunks=1, layout=layout,
                              copy_streams=copy_streams, regroup=regroup)
    events = []

    def hook(name, stream):  # records at its point in the stream
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        events.append((name, ev))

    layer.on_phase = hook
    for _ in range(3):
        events.clear()
        layer.forward(x, logits, stack[0][1])
    torch.cuda.synchronize()
    dist.barrier()
    acc: dict[str, float] = {}
    for _ in range(10):
        events.clear()
        layer.forward(x, logits, stack[0][1])
        torch.cuda.synchronize()
        for i in range(1, len(events)):
            name = events[i][0]
            acc[name] = acc.get(name, 0.0) + events[i - 1][1].elapsed_time(events[i][1]) / 10
    layer.close()
    return {"config": config, "world": world, "tokens_rank0": e - b, "layout": layout, "copy_streams": copy_streams,
            "regroup": regroup,
            "phases_ms": {k: round(v, 3) for k, v in acc.items()}, "layer_ms": round(sum(acc.values()), 3)}


def _gemms(dev):
    """The owner's GEMMs on rows received source-major (``sources`` = G) against
    the same rows contiguous per expert, NF4, on one GPU: c2's segment sizes at 2
    GPUs (~2048 rows per source and expert) and c4's at 8 (~256), ragged.  Min
    and median of 7 alternating rounds of 20 launches each (ms)."""
    import statistics
    from . import ops, tables
    res = {}
    for case, (H, I, El, G, mean, spread) in {"c2 at 2 GPUs": (2048, 1408, 16, 2, 2048, 60),
                                             "c4 at 8 GPUs": (4096, 1536, 16, 8, 256, 16)}.items():
        g = torch.Generator(device=dev).manual_seed(1)
        ws = [ops.nf4_quantize((torch.randn(sh, generator=g, device=dev) * 0.02).to(torch.bfloat16),
                               tables.nf4_code(dev), tables.dynamic_map(dev))
              for sh in ((El, I, H), (El, I, H), (El, H, I))]
        cnt = mean + torch.randint(-spread, spread, (G * El,), generator=torch.Generator().manual_seed(5))
        S = int(cnt.sum())
        x = torch.randn(S, H, device=dev).to(torch.bfloat16)
        offs_src = torch.cumsum(cnt, 0).to(torch.int32).to(dev)
        offs_exp = torch.cumsum(cnt.view(G, El).sum(0), 0).to(torch.int32).to(dev)
        h = torch.empty(S, I, device=dev, dtype=torch.bfloat16)
        y = torch.empty(S, H, device=dev, dtype=torch.bfloat16)
        runs = {"gateup_sources": lambda: ops.gateup_swiglu(x, offs_src, ws[0], ws[1], inter=I, out=h, sources=G),
                "gateup_contiguous": lambda: ops.gateup_swiglu(x, offs_exp, ws[0], ws[1], inter=I, out=h),
                "down_sources": lambda: ops.down(h, offs_src, ws[2], hidden=H, out=y, sources=G),
                "down_contiguous": lambda: ops.down(h, offs_exp, ws[2], hidden=H, out=y)}
        acc = {k: [] for k in runs}
        for _ in range(7):
            for name, fn in runs.items():
                for _ in range(3):
                    fn()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(20):
                    fn()
                b.record()
                torch.cuda.synchronize()
                acc[name].append(a.elapsed_time(b) / 20)
        res[case] = {"rows": S, **{k: [round(min(v), 4), round(statistics.median(v), 4)] for k, v in acc.items()}}
    ops.check_device()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["bandwidth", "blocks", "phases", "gemms"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--layout", default="source", choices=["expert", "source"])
    ap.add_argument("--copy-streams", type=int, default=1)
    ap.add_argument("--regroup", default="auto", choices=["never", "auto", "always"])
    args = ap.parse_args()
    if args.what == "gemms":  # one GPU, no process group
        print(json.dumps(_gemms(torch.device("cuda", 0))), flush=True)
        return
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if args.what == "bandwidth":
            res = _bandwidth(dev, world, rank)
        elif args.what == "blocks":
            res = _blocks(dev, world, rank)
        else:
            res = _phases(dev, world, rank, args.config, args.layout, args.copy_streams, args.regroup)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
