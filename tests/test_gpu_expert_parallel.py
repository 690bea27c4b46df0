"""Expert-parallel layer on 2+ GPUs over NCCL against the single-GPU layer.

Each rank owns E/G experts (quantised separately; NF4 and INT8 buffers are
per expert, so a block quantised alone equals the same block of the whole
stack) and routes a contiguous shard of the tokens.  Rows of every expert
segment arrive in the single-GPU order, so the outputs must be bit-identical.
Skipped with fewer than two GPUs.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _weights(fmt, E, H, I, seed, dev):
    from mirai_b200 import ops, tables
    g = torch.Generator(device=dev).manual_seed(seed)
    raw = [(torch.randn(s, generator=g, device=dev) * 0.02).to(torch.bfloat16) for s in ((E, I, H), (E, I, H), (E, H, I))]
    return raw


def _quant(fmt, w, dev):
    from mirai_b200 import ops, tables
    if fmt == "nf4":
        return ops.nf4_quantize(w, tables.nf4_code(dev), tables.dynamic_map(dev))
    if fmt == "int8":
        return ops.int8_quantize(w.float())
    return w.contiguous()


def _rank_main(rank, world, rdv, cfg, results):
    import torch.distributed as dist
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"file://{rdv}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        from mirai_b200 import ops
        from mirai_b200.expert_parallel import ExpertShard, ep_moe_forward, shard_tokens
        T, H, E, k, I, fmt, chunks, transport, copy_streams, regroup, layout = cfg
        g = torch.Generator(device=dev).manual_seed(11)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=g, device=dev) * 1.5
        raw = _weights(fmt, E, H, I, 5, dev)
        shard = ExpertShard(E, world, rank)
        lo, hi = shard.first, shard.first + shard.local
        local = tuple(_quant(fmt, w[lo:hi].contiguous(), dev) for w in raw)
        b, e = shard_tokens(T, world, rank)
        xr, lr = x[b:e].contiguous(), logits[b:e].contiguous()
        if transport == "ipc":
            from mirai_b200.expert_parallel import ExpertParallelMoE
            layer = ExpertParallelMoE(shard, top_k=k, inter=I, chunks=chunks, copy_streams=copy_streams,
                                      regroup=regroup, layout=layout)
            # a quarter of the tokens first: the second call needs larger exchange buffers, so every
            # rank releases, re-exports and re-imports them (flags zeroed, the epoch still counting)
            q = max(1, (e - b) // 4)
            small = layer.forward(xr[:q].contiguous(), lr[:q].contiguous(), local)
            grown_from = layer.buffers.local.numel()
            out = layer.forward(xr, lr, local)
            grew = layer.buffers.local.numel() > grown_from
            out2 = layer.forward(xr, lr, local)  # buffers reused
            assert torch.equal(out, out2)
            layer.close()
        else:
            comm = torch.cuda.Stream() if chunks > 1 else None
            if chunks > 1:
                ops.set_gemm_sm_limit(torch.cuda.get_device_properties(dev).multi_processor_count - 16)
            out = ep_moe_forward(xr, lr, local, shard=shard, top_k=k, inter=I, chunks=chunks, comm_stream=comm)
            ops.set_gemm_sm_limit(0)
        code, info = ops.device_status()
        full = tuple(_quant(fmt, w, dev) for w in raw)
        idx, tw = ops.route_topk(logits, k)
        ref = ops.moe_forward(x, idx, tw, *full, num_experts=E, inter=I)[b:e]
        equal = bool(torch.equal(out, ref))
        if transport == "ipc":
            # the small call is the single-GPU layer on those tokens alone
            ridx, rtw = ops.route_topk(lr[:q].contiguous(), k)
            ours = ops.moe_forward(xr[:q].contiguous(), ridx, rtw, *full, num_experts=E, inter=I)
            equal = equal and bool(torch.equal(small, ours)) and grew
        results[rank] = (code, equal, float((out.float() - ref.float()).abs().max()))
    finally:
        dist.destroy_process_group()


def _rendezvous():
    """A fresh rendezvous file for one process group (file:// init: no TCP port
    to collide with another test's group)."""
    import tempfile
    fd, path = tempfile.mkstemp(prefix="mirai_pg_")
    os.close(fd)
    return path


@pytest.mark.parametrize("fmt,chunks,transport,copy_streams,world,regroup,layout", [
    ("nf4", 1, "nccl", 1, 2, "never", "source"), ("bf16", 1, "nccl", 1, 2, "never", "source"),
    ("int8", 1, "nccl", 1, 2, "never", "source"), ("nf4", 3, "nccl", 1, 2, "never", "source"),
    ("nf4", 1, "ipc", 1, 2, "never", "source"), ("nf4", 3, "ipc", 1, 2, "always", "source"),
    ("int8", 2, "ipc", 1, 2, "always", "source"), ("bf16", 2, "ipc", 3, 2, "auto", "source"),
    ("nf4", 2, "ipc", 1, 2, "never", "expert"), ("int8", 1, "ipc", 2, 2, "never", "expert"),
    ("nf4", 2, "ipc", 2, 4, "always", "source"), ("nf4", 2, "ipc", 1, 4, "never", "expert"),
    ("nf4", 2, "nccl", 1, 4, "never", "source"),
])
def test_expert_parallel_equals_single_gpu_layer(fmt, chunks, transport, copy_streams, world, regroup, layout):
    """nccl, chunks > 1: the pipelined all-to-all path (exchanges on a second
    stream, GEMMs capped below the SM count); ipc: copy-engine transfers into
    source-major peer-mapped buffers (owners regrouping received rows
    expert-major "always" or not "never") or into expert-major buffers (one
    copy per (peer, expert) block), on one stream or spread over side
    streams.  The ipc layer is first called on a quarter of the tokens, so its
    second call grows and re-shares the exchange buffers."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from mirai_b200.build import build
    build()
    # 1500 tokens per rank: the second ipc call outgrows the first call's 2 MiB-rounded buffers
    cfg = (1500 * world, 256, 8, 2, 384, fmt, chunks, transport, copy_streams, regroup, layout)
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _rendezvous(), cfg, results), nprocs=world, start_method="spawn")
        res = dict(results)
    for r in range(world):
        code, equal, maxdiff = res[r]
        assert code == 0
        assert equal, f"rank {r}: max |diff| {maxdiff}"


def _train_rank_main(rank, world, rdv, cfg, results):
    import torch.distributed as dist
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"file://{rdv}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        from mirai_b200 import ops
        from mirai_b200.expert_parallel import (ExpertParallelMoE, ExpertShard, ep_moe_backward, ep_moe_forward,
                                                shard_tokens)
        T, H, E, k, I, fmt, chunks, rotated, lora_rank, transport, regroup = cfg
        g = torch.Generator(device=dev).manual_seed(13)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=g, device=dev) * 1.5
        gout = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        raw = _weights(fmt, E, H, I, 5, dev)

        def quant(w, key_in):
            if fmt == "int8" and rotated:
                return ops.int8_quantize(w.float(), group_size=64 if key_in % 64 == 0 else 16)
            return _quant(fmt, w, dev)

        shard = ExpertShard(E, world, rank)
        lo, hi = shard.first, shard.first + shard.local
        local = tuple(quant(w[lo:hi].contiguous(), w.shape[2]) for w in raw)
        full = tuple(quant(w, w.shape[2]) for w in raw)
        b, e = shard_tokens(T, world, rank)
        lora = lora_full = None
        if lora_rank:
            la = torch.randn(E, lora_rank, I, generator=g, device=dev) * 0.05
            lb = torch.randn(E, H, lora_rank, generator=g, device=dev) * 0.05
            lora = ops.DownLoRA(la[lo:hi], lb[lo:hi], 2.0, compute_grads=True)
            lora_full = ops.DownLoRA(la, lb, 2.0, compute_grads=True)
        xr, lr_, gr = x[b:e].contiguous(), logits[b:e].contiguous(), gout[b:e].contiguous()
        stale_refused = True
        if transport == "ipc":
            layer = ExpertParallelMoE(shard, top_k=k, inter=I, chunks=chunks, regroup=regroup)
            try:
                # a training state is refused once another forward has used the layer's buffers
                _, old = layer.forward(xr, lr_, local, train=True, lora=lora)
                layer.forward(xr, lr_, local)
                try:
                    layer.backward(gr, old, local, lora=lora)
                    stale_refused = False
                except RuntimeError:
                    pass
                out, st = layer.forward(xr, lr_, local, train=True, lora=lora)
                dx, dw = layer.backward(gr, st, local, lora=lora)
                torch.cuda.synchronize()
            finally:
                layer.close()
        else:
            out, st = ep_moe_forward(xr, lr_, local, shard=shard, top_k=k, inter=I, chunks=chunks, train=True,
                                     lora=lora)
            dx, dw = ep_moe_backward(gr, st, local, shard=shard, inter=I, lora=lora)
        code, info = ops.device_status()
        idx, tw = ops.route_topk(logits, k)
        ref, rst = ops.moe_forward_train(x, idx, tw, *full, num_experts=E, inter=I, lora=lora_full)
        rdx, rdw = ops.moe_backward_dx(gout, rst, *full, inter=I, lora=lora_full)
        same = stale_refused and bool(torch.equal(out, ref[b:e])) and bool(torch.equal(dw, rdw[b:e]))
        if lora_rank:  # this rank's experts' factor gradients (partial sums per chunk: the bf16 tolerance)
            for got, want in ((lora.grad_a, lora_full.grad_a[lo:hi]), (lora.grad_b, lora_full.grad_b[lo:hi])):
                same = same and float((got - want).abs().max() / want.abs().max()) < 1e-3
        dx_exact = bool(torch.equal(dx, rdx[b:e]))
        rel = float((dx.float() - rdx[b:e].float()).abs().max() / rdx.float().abs().max())
        results[rank] = (code, same, dx_exact, rel)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,chunks,world,rotated,lora_rank,transport,regroup", [
    ("nf4", 1, 2, False, 0, "nccl", "never"), ("bf16", 2, 2, False, 0, "nccl", "never"),
    ("int8", 1, 2, False, 0, "nccl", "never"), ("int8", 2, 2, True, 0, "nccl", "never"),
    ("nf4", 2, 2, False, 16, "nccl", "never"), ("nf4", 2, 4, False, 16, "nccl", "never"),
    ("nf4", 2, 2, False, 16, "ipc", "never"), ("bf16", 1, 2, False, 0, "ipc", "always"),
    ("int8", 2, 2, True, 16, "ipc", "auto"), ("nf4", 2, 4, False, 16, "ipc", "always"),
])
def test_expert_parallel_backward_equals_single_gpu(fmt, chunks, world, rotated, lora_rank, transport, regroup):
    """Training through the expert-parallel layer (NCCL all-to-all, or the
    copy-engine exchange of ``ExpertParallelMoE`` with and without the
    owners' expert-major regrouping): the
    forward output and the route-weight gradients equal the single-GPU
    layer's exactly, and so does dX (the rows' products and each token's
    ascending-position sum are the single-GPU ones); the block-Hadamard INT8
    format rotates dX rows on the owners before the route sum, so there dX is
    held to the bf16 tolerance instead.  With a rank-16 LoRA on w2 the owners
    regroup their rows expert-major; the adapter's factor gradients of each
    rank's experts match the single-GPU ones (summed per chunk).  The
    copy-engine layer refuses a training state once another forward has
    reused its buffers."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from mirai_b200.build import build
    build()
    cfg = (2000, 256, 8, 2, 384, fmt, chunks, rotated, lora_rank, transport, regroup)
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_train_rank_main, args=(world, _rendezvous(), cfg, results), nprocs=world,
                           start_method="spawn")
        res = dict(results)
    for r in range(world):
        code, same, dx_exact, rel = res[r]
        assert code == 0 and same
        assert dx_exact or (rotated and rel < 3e-2), f"rank {r}: dx rel err {rel}"
