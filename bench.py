#!/usr/bin/env python
"""MoE-FFN tokens/s (NF4 experts) on B200 -- the routed expert FFN of the
seruva19/mirai denoiser, run through libmirai_b200.so.

Default workload: BASELINE config 2 as it is defined -- 32768 tokens, hidden
2048, 32 experts, top-2, SwiGLU intermediate 1408, NF4 blocksize-64 experts
with double-quantised absmax, forward plus the dX backward through the frozen
experts with a rank-16 LoRA on w2 (its factor gradients included).  One step
= one pass of the path over the batch: fp32 router top-k on precomputed gate
logits -> NF4 decode of the three keys into bf16 copies (with 2048 rows per
expert a training pass stages them; --nf4-staging never keeps the decode
inside the GEMMs) -> dispatch plan -> permute -> gate/up grouped GEMM + SwiGLU
-> LoRA rank projection -> down grouped GEMM with the rank block -> weighted
combine; then combine backward -> down dX (SwiGLU backward fused) -> gate/up
dX -> un-permute sum, and the LoRA factor gradients.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c0..c4] [--mode train|fwd]
                    [--int8-rotation] [--nf4-staging auto|always|never] [--tokens T]
                    [--impl ours|reference] [--ep-transport ipc|nccl] [--ep-chunks C]
                    [--ep-layout source|expert] [--ep-regroup never|auto|always] [--ep-copy-streams S]
                    [--probe bandwidth|blocks|phases|gemms|epilogue]

``--mode fwd`` times the forward layer alone (the line also carries the
forward rate of a train run under ``forward``).  ``--int8-rotation`` runs
c3 in the reference's default INT8 format (block-Hadamard groups of 256).
Under torchrun (N > 1) the layer runs expert-parallel
(mirai_b200.expert_parallel): each rank owns E/N experts and routes its own
tokens; rows move by copy engines into peer-mapped buffers (``ipc``, default)
or by NCCL all-to-all, in C chunks whose exchanges overlap the GEMMs.  c1-c3
keep their token count per rank (scaling "weak": per-GPU GEMM work is that of
one GPU); c4 is BASELINE config 4, a 16-layer stack over 65536 tokens in total
(scaling "strong", also runnable on one GPU).
``--impl reference`` times the CPU restatement of the reference's torch path
(``oracle/``) on the host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "c0": dict(T=512, H=256, E=8, k=2, I=512, fmt="nf4", zipf=None),
    "c1": dict(T=32768, H=2048, E=32, k=2, I=1408, fmt="bf16", zipf=None),
    "c2": dict(T=32768, H=2048, E=32, k=2, I=1408, fmt="nf4", zipf=None),
    "c3": dict(T=8192, H=3072, E=64, k=4, I=1024, fmt="int8", zipf=1.2),
    # expert-parallel stack: 16 layers, 65536 tokens split over the ranks, 128 experts
    # (16 per GPU at 8); strong scaling
    "c4": dict(T=65536, H=4096, E=128, k=8, I=1536, fmt="nf4", zipf=None, layers=16, ep="strong"),
}
METRIC = "MoE-FFN tokens/s (NF4 experts) + % TC/HBM roofline at 1/2/4/8 B200"
LORA_RANK = 16
# DRAM bytes (read + write) per launch of a grouped GEMM from an ncu capture of
# the same kernel on the same workload and mode (keyed config-mode-kernel), with
# the capture it came from (the summary and its command are under profiles/).
# A kernel changed since its capture, or not captured, reports null.
NCU_TRAFFIC = {
    "c2-train-gateup_dx_bf16 (NF4 staged)": (739_500_000 + 247_990_000, "profiles/grouped_gemm_traffic_c2.md"),
    "c2-train-down_dx_bf16 (NF4 staged)": (865_320_000 + 337_760_000, "profiles/grouped_gemm_traffic_c2.md"),
    "c2-train-gateup_swiglu_bf16 (NF4 staged)": (639_560_000 + 516_470_000,
                                                 "profiles/grouped_gemm_traffic_c2.md"),
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """Polls NVML (read-only) for SM clock and clock-event reasons.

    Every rank samples its own GPU; with several ranks the period grows with
    their number (5 ms x ranks), so that the processes' NVML queries stay few
    beside the driver calls of the copy-engine exchange (an 8-GPU train step
    timed 11.8 ms under eight 5 ms samplers, 4.7 ms with the period scaled)."""

    def __init__(self, index: int, period_s: float | None = None):
        world = int(os.environ.get("WORLD_SIZE", "1"))
        self.index, self.period = index, period_s if period_s is not None else 0.005 * max(1, world)
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.ok = False

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            names = {
                "hw_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwSlowdown", 0x8),
                "hw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                "sw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                "sw_power_cap": getattr(pynvml, "nvmlClocksEventReasonSwPowerCap", 0x4),
                "hw_power_brake_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
            }
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception as exc:  # NVML missing: report that, keep the run
            self.error = str(exc)
            return self

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    r = get_reasons(h)
                    for n, bit in names.items():
                        if r & bit:
                            self.reasons.add(n)
                except Exception:
                    pass
                time.sleep(self.period)

        self.ok = True
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=1)
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "error", "nvml")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- workload

def make_workload(cfg, dev, seed, rotation=False):
    import torch
    from mirai_b200 import ops, tables

    T, H, E, k, I = cfg["T"], cfg["H"], cfg["E"], cfg["k"], cfg["I"]
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    gate = torch.randn(E, H, generator=g, device=dev) * 0.02
    logits = x.float() @ gate.T
    if cfg["zipf"]:
        # Zipf(s) load over a seeded expert permutation: bias_e = c * log p_e,
        # c chosen so the top expert gets about a quarter of the routes.
        perm = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
        p = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** cfg["zipf"]
        p = (p / p.sum())[perm.argsort()].to(torch.float32).to(dev)
        logits = logits + 2.0 * torch.log(p)[None, :]
    ws = []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        if cfg["fmt"] == "nf4":
            w = ops.nf4_quantize(w, tables.nf4_code(dev), tables.dynamic_map(dev))
        elif cfg["fmt"] == "int8":
            # the reference's default format rotates groups of best_group_size(in) (quant.py:87-91)
            grp = (256 if shape[2] % 256 == 0 else 64 if shape[2] % 64 == 0 else 16) if rotation else 0
            w = ops.int8_quantize(w.float(), group_size=grp)
        ws.append(w)
    torch.cuda.synchronize()
    return x, logits, ws


def weight_bytes(cfg):
    E, H, I = cfg["E"], cfg["H"], cfg["I"]
    n = 3 * E * H * I
    if cfg["fmt"] == "nf4":
        return n // 2 + n // 64 + 4 * (n // 64 // 256 + E)
    if cfg["fmt"] == "int8":
        return n + 4 * E * (2 * I + H)
    return 2 * n


# ----------------------------------------------------------------------------- our arm

def measure_e2e(dev, host_in, n_out, out_shape, compute, args, barrier):
    """ms per step through the public API with host buffers.  Every step copies
    its inputs host -> device from pinned memory and its results device -> host.
    Two buffer slots and their own copy streams let step j's upload and step
    j-1's download overlap the neighbouring steps' compute, as a serving loop
    would; each direction's bytes are split by rows over ``--e2e-copy-streams``
    streams (copy engines)."""
    import torch

    comp = torch.cuda.current_stream()
    lanes = max(1, int(getattr(args, "e2e_copy_streams", 1)))
    ups = [torch.cuda.Stream() for _ in range(lanes)]
    downs = [torch.cuda.Stream() for _ in range(lanes)]

    def parts(t):  # the row blocks each lane copies
        return torch.tensor_split(t, lanes, dim=0) if t.dim() else (t,)

    slots = []
    for _ in range(2):
        slots.append({
            "din": [torch.empty_like(t, device=dev) for t in host_in],
            "dout": [torch.empty(out_shape, dtype=torch.bfloat16, device=dev) for _ in range(n_out)],
            "hout": [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(n_out)],
            "loaded": [torch.cuda.Event() for _ in range(lanes)], "computed": torch.cuda.Event(),
            "saved": [torch.cuda.Event() for _ in range(lanes)], "used": False,
        })

    def e2e_step(j):
        sl = slots[j % 2]
        for i, s in enumerate(ups):
            with torch.cuda.stream(s):
                if sl["used"]:
                    s.wait_event(sl["computed"])  # the slot's previous step has read its inputs
                for d, h in zip(sl["din"], host_in):
                    dp, hp = parts(d), parts(h)
                    if i < len(dp):
                        dp[i].copy_(hp[i], non_blocking=True)
                sl["loaded"][i].record(s)
        for ev in sl["loaded"]:
            comp.wait_event(ev)
        if sl["used"]:
            for ev in sl["saved"]:
                comp.wait_event(ev)  # the slot's previous result has been downloaded
        compute(sl["din"], sl["dout"])
        sl["computed"].record(comp)
        for i, s in enumerate(downs):
            with torch.cuda.stream(s):
                s.wait_event(sl["computed"])
                for h, d in zip(sl["hout"], sl["dout"]):
                    hp, dp = parts(h), parts(d)
                    if i < len(hp):
                        hp[i].copy_(dp[i], non_blocking=True)
                sl["saved"][i].record(s)
        sl["used"] = True

    def drain():
        for sl in slots:
            if sl["used"]:
                for ev in sl["saved"]:
                    comp.wait_event(ev)

    for j in range(max(1, min(3, args.warmup))):
        e2e_step(j)
    drain()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for s in ups + downs:
        s.wait_event(e0)
    for j in range(args.steps):
        e2e_step(j)
    drain()
    e1.record(comp)
    e1.synchronize()
    barrier()
    return e0.elapsed_time(e1) / args.steps


def make_weights_fmt(cfg, args):
    """Weight format label of the workload (INT8 with the rotation flag)."""
    if cfg["fmt"] == "int8" and args.int8_rotation:
        return "int8 block-Hadamard g=256"
    return cfg["fmt"]


def time_kernel(fn, reps):
    """Mean ms of ``fn`` over ``reps`` launches, CUDA events on the current stream."""
    import torch
    for _ in range(3):
        fn()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / reps


def run_ours(args, cfg, rank, world, dev):
    import torch
    import torch.distributed as dist
    from mirai_b200 import ops

    T, H, E, k, I = cfg["T"], cfg["H"], cfg["E"], cfg["k"], cfg["I"]
    x, logits, (w1, w3, w2) = make_workload(cfg, dev, seed=1234 + rank, rotation=args.int8_rotation)
    S = T * k
    train = args.mode == "train"
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    g_out = torch.randn(T, H, device=dev, generator=gen).to(torch.bfloat16) if train else None
    lora = None
    if train:
        # rank-16 LoRA on the down projection (alpha 16: scale alpha / rank = 1), lora_b perturbed
        # away from its zero init as the reference's adapter tests do
        la = torch.randn(E, LORA_RANK, I, device=dev, generator=gen) * (1.0 / I ** 0.5)
        lb = torch.randn(E, H, LORA_RANK, device=dev, generator=gen) * 0.02
        lora = ops.DownLoRA(la, lb, 16.0 / LORA_RANK, compute_grads=True)

    def forward(xin, lin, out=None):
        idx, tw = ops.route_topk(lin, k)
        o = ops.moe_forward(xin, idx, tw, w1, w3, w2, num_experts=E, inter=I)
        if out is not None:
            out.copy_(o)
        return o

    def step(xin, lin, out=None, gin=None, dx_out=None):
        if not train:
            return forward(xin, lin, out)
        idx, tw = ops.route_topk(lin, k)
        o, st = ops.moe_forward_train(xin, idx, tw, w1, w3, w2, num_experts=E, inter=I, lora=lora)
        if out is not None:
            out.copy_(o)
        dx, _ = ops.moe_backward_dx(g_out if gin is None else gin, st, w1, w3, w2, inter=I, lora=lora)
        if dx_out is not None:
            dx_out.copy_(dx)
        return o

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        ops.check_device()
        clocks = ClockSampler(torch.cuda.current_device()).start()
        barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = ops.launch_count()
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        n1 = ops.launch_count()
        t1.synchronize()
        barrier()
        torch.cuda.synchronize()
        clk = clocks.stop()
        ops.check_device()
        return t0.elapsed_time(t1) / steps, clk, n1 - n0

    # ---- device-resident throughput (value)
    ms, clk, launches = timed(lambda: step(x, logits), args.steps)
    fwd_ms = timed(lambda: forward(x, logits), args.steps)[0] if train else ms

    # ---- each grouped GEMM of the step alone (CUDA events on its stream)
    idx, tw = ops.route_topk(logits, k)
    _, st = ops.moe_forward_train(x, idx, tw, w1, w3, w2, num_experts=E, inter=I, lora=lora)
    plan = st.plan
    xs = ops.permute_rows(x, plan.sorted_token_indices)
    h = torch.empty((S, I), dtype=torch.bfloat16, device=dev)
    y = torch.empty((S, H), dtype=torch.bfloat16, device=dev)
    reps = max(5, min(50, args.steps))
    kclocks = ClockSampler(torch.cuda.current_device()).start()
    # the weights the step's GEMMs multiply: NF4 decoded once per pass to bf16 where staging pays
    sw1, sw3, sw2 = ops.stage_nf4((w1, w3, w2), S, E, training=train)
    staged = sw1 is not w1
    kernels = {"gateup_swiglu": (4.0 * S * H * I, lambda: ops.gateup_swiglu(xs, plan.offsets, sw1, sw3, inter=I,
                                                                             out=h)),
               "down": (2.0 * S * H * I, lambda: ops.down(h, plan.offsets, sw2, hidden=H, out=y))}
    if train and not args.int8_rotation:
        dgu = torch.empty((S, 2 * I), dtype=torch.bfloat16, device=dev)
        dxs = torch.empty((S, H), dtype=torch.bfloat16, device=dev)
        glow = ops.lora_project(y, plan.offsets, lora, forward=False)
        kernels["down_dx"] = (2.0 * S * H * I, lambda: ops.down_dx(y, plan.offsets, sw2, st.gate_up, inter=I,
                                                                   out=dgu, lora=lora, rank_a=glow))
        kernels["gateup_dx"] = (4.0 * S * H * I, lambda: ops.gateup_dx(dgu, plan.offsets, sw1, sw3, hidden=H,
                                                                       out=dxs))
    kernel_ms = {name: time_kernel(fn, reps) for name, (_, fn) in kernels.items()}
    if staged:  # the decode pass itself: HBM-bound, the three keys one after another
        kernel_ms["nf4_dequantize_x3"] = time_kernel(
            lambda: [ops.nf4_dequantize(w, out=o) for w, o in ((w1, sw1), (w3, sw3), (w2, sw2))], reps)
    kclk = kclocks.stop()
    top = max(kernels, key=kernel_ms.get)  # the step's dominant GEMM
    top_flops = kernels[top][0]
    del h, y

    # ---- end to end through the public API with host buffers
    host_in = [x.cpu().pin_memory(), logits.cpu().pin_memory()] + ([g_out.cpu().pin_memory()] if train else [])

    def compute(din, dout):
        if train:
            step(din[0], din[1], out=dout[0], gin=din[2], dx_out=dout[1])
        else:
            step(din[0], din[1], out=dout[0])

    e2e_ms = measure_e2e(dev, host_in, 2 if train else 1, (T, H), compute, args, barrier)
    ops.check_device()

    if world > 1:
        t = torch.tensor([ms, e2e_ms, fwd_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, fwd_ms = float(t[0]), float(t[1]), float(t[2])

    peaks = load_peaks()
    achieved = top_flops / (kernel_ms[top] * 1e-3) / 1e12
    fmt = make_weights_fmt(cfg, args)
    kname = f"{top}_{'bf16 (NF4 staged)' if staged else cfg['fmt']}"
    traffic = NCU_TRAFFIC.get(f"{args.config}-{args.mode}-{kname}") if not args.int8_rotation else None
    lora_flops = 6.0 * S * LORA_RANK * (H + I)  # rank projection + rank block, fwd and dX, and the factor grads
    step_flops = (12.0 * S * H * I + lora_flops) if train else 6.0 * S * H * I
    line = {
        "metric": METRIC,
        "value": world * T / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations x " + fmt + " weights, fp32 accumulate",
        "data": "synthetic (seeded torch.randn; random-init experts quantised on the GPU)",
        "config": {
            "workload": f"{args.config}: one routed expert FFN layer "
                        + (f"forward + dX backward with a rank-{LORA_RANK} LoRA on w2 (adapter grads included)"
                           if train else "forward") + f", T={T} H={H} E={E} k={k} I={I} "
                        f"{fmt} experts" + (f", Zipf({cfg['zipf']}) load" if cfg["zipf"] else ""),
            "tokens_per_gpu": T, "hidden": H, "experts": E, "top_k": k, "intermediate": I,
            "weights": fmt, "parallelism": f"dp{world} token-parallel replicas (experts replicated)",
            **({"nf4_decode": "once per pass into bf16 copies, then the bf16 GEMMs (staging "
                              f"{args.nf4_staging})" if staged else
                              f"inside the GEMMs' main loops (staging {args.nf4_staging})"}
               if cfg["fmt"] == "nf4" else {}),
            "l2": f"no flush: inputs {(T * H * 2 + weight_bytes(cfg)) / 1e6:.0f} MB per step exceed the 126 MB L2",
        },
        "tflops": world * step_flops / (ms * 1e-3) / 1e12,
        "forward": {"value": world * T / (fwd_ms * 1e-3), "unit": "tokens/s", "ms_per_step": fwd_ms,
                    "tflops": world * 6.0 * S * H * I / (fwd_ms * 1e-3) / 1e12},
        "kernel_ms": kernel_ms,
        "roofline": {
            "kernel": kname,
            "bound": "tensor",
            "achieved": achieved,
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_tflops"],
            "peak_source": f"{peaks['source']} bf16 dense (burst; kernel timed alone)",
            "algorithmic": f"{top_flops / (S * H * I):.0f}*S*H*I = {top_flops / 1e9:.1f} GFLOP per launch "
                           f"(the step's longest kernel)",
            "traffic": None if traffic is None else traffic[0],
            "traffic_source": None if traffic is None else f"ncu dram__bytes_read+write, {traffic[1]}",
            "clocks": kclk,
            "step_frac": (step_flops / (ms * 1e-3) / 1e12) / peaks["bf16_tflops"],
        },
        "e2e": {
            "value": world * T / (e2e_ms * 1e-3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": T * H * 2 * (2 if train else 1) + T * E * 4,
            "d2h_bytes_per_step": T * H * 2 * (2 if train else 1),
            "copies": f"pinned host buffers; 2 slots, uploads and downloads on their own streams overlap compute, "
                      f"each direction split over {args.e2e_copy_streams} stream(s)",
        },
        "gpu_launches": launches,
        "gpu_launches_source": "libmirai_b200's own count of the kernels its entry points enqueued in the timed "
                               "region (mirai_b200_launch_count)",
        "clocks": clk,
    }
    return line


# ----------------------------------------------------------------------------- expert-parallel arm

def make_ep_workload(cfg, dev, rank, shard, tokens_local):
    """This rank's tokens, layer-0 router logits and, per layer, the router gate
    (identical on every rank) and this rank's E/N experts (seeded per rank)."""
    import torch
    from mirai_b200 import ops, tables

    H, E, I = cfg["H"], cfg["E"], cfg["I"]
    El = shard.local
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(tokens_local, H, generator=g, device=dev).to(torch.bfloat16)
    stack = []
    for layer in range(cfg.get("layers", 1)):
        gate = (torch.randn(E, H, generator=torch.Generator(device=dev).manual_seed(77 + layer), device=dev)
                * 0.02).to(torch.bfloat16)
        wg = torch.Generator(device=dev).manual_seed(100003 * (layer + 1) + rank)
        ws = []
        for shape in ((El, I, H), (El, I, H), (El, H, I)):
            w = (torch.randn(shape, generator=wg, device=dev) * 0.02).to(torch.bfloat16)
            if cfg["fmt"] == "nf4":
                w = ops.nf4_quantize(w, tables.nf4_code(dev), tables.dynamic_map(dev))
            elif cfg["fmt"] == "int8":
                w = ops.int8_quantize(w.float())
            ws.append(w)
        stack.append((gate, tuple(ws)))
    x0 = x.float()
    u0 = (x0 * torch.rsqrt(x0.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    logits0 = ((u0 if cfg.get("layers", 1) > 1 else x) @ stack[0][0].T).float()
    torch.cuda.synchronize()
    return x, logits0, stack


def run_ep(args, cfg, rank, world, dev):
    import torch
    import torch.distributed as dist
    from mirai_b200 import ops
    from mirai_b200.expert_parallel import (CudaStepOps, ExpertParallelMoE, ExpertShard, ep_moe_backward,
                                            ep_moe_forward, shard_tokens)

    H, E, k, I = cfg["H"], cfg["E"], cfg["k"], cfg["I"]
    layers = cfg.get("layers", 1)
    strong = cfg.get("ep") == "strong"
    T_total = cfg["T"] if strong else cfg["T"] * world
    b, e = shard_tokens(T_total, world, rank)
    T_r = e - b
    shard = ExpertShard(E, world, rank)
    x, logits0, stack = make_ep_workload(cfg, dev, rank, shard, T_r)
    stepops = CudaStepOps()
    train = args.mode == "train"
    if train and layers > 1:
        raise SystemExit("--mode train runs single-layer workloads (c0-c3)")
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    g_out = torch.randn(T_r, cfg["H"], device=dev, generator=gen).to(torch.bfloat16) if train else None
    lora = None
    if train:  # the rank-16 LoRA on w2 of this rank's experts, as in the single-GPU step
        la = torch.randn(shard.local, LORA_RANK, cfg["I"], device=dev, generator=gen) * (1.0 / cfg["I"] ** 0.5)
        lb = torch.randn(shard.local, cfg["H"], LORA_RANK, device=dev, generator=gen) * 0.02
        lora = ops.DownLoRA(la, lb, 16.0 / LORA_RANK, compute_grads=True)
    chunks = args.ep_chunks if world > 1 else 1
    ipc = args.ep_transport == "ipc" and world > 1
    free_sms = args.ep_free_sms if args.ep_free_sms is not None else (2 if ipc else 16)
    if world > 1 and (chunks > 1 or ipc) and free_sms > 0:
        # leave SMs for the communication kernels (NCCL's all-to-all; with ipc only the
        # one-element arrival all-reduce) so the exchanges overlap the GEMMs
        ops.set_gemm_sm_limit(torch.cuda.get_device_properties(dev).multi_processor_count - free_sms)
    if ipc:
        layer = ExpertParallelMoE(shard, top_k=k, inter=I, chunks=chunks, ops=stepops,
                                  copy_streams=args.ep_copy_streams, layout=args.ep_layout,
                                  regroup=args.ep_regroup)
        ep = layer.forward
    else:
        layer = None
        comm = torch.cuda.Stream() if chunks > 1 else None
        ep = lambda u, lg, ws: ep_moe_forward(u, lg, ws, shard=shard, top_k=k, inter=I, ops=stepops, chunks=chunks,
                                              comm_stream=comm)

    def rms_norm(v):  # the block's pre-MoE norm (no learned scale): keeps the stack's activations bounded
        vf = v.float()
        return (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)

    def step(xin, l0, out=None, gin=None, dx_out=None):
        if train:  # one layer: forward keeping the owners' gate/up, then the dX exchange and GEMMs
            g = g_out if gin is None else gin
            if layer is not None:
                o, st = layer.forward(xin, l0, stack[0][1], train=True, lora=lora)
                dx, _ = layer.backward(g, st, stack[0][1], lora=lora)
            else:
                o, st = ep_moe_forward(xin, l0, stack[0][1], shard=shard, top_k=k, inter=I, ops=stepops,
                                       chunks=chunks, train=True, lora=lora)
                dx, _ = ep_moe_backward(g, st, stack[0][1], shard=shard, inter=I, ops=stepops, lora=lora)
            if out is not None:
                out.copy_(o)
            if dx_out is not None:
                dx_out.copy_(dx)
            return o
        h = xin
        for li, (gate, ws) in enumerate(stack):
            if layers == 1:
                h = ep(h, l0, ws)
                continue
            u = rms_norm(h)
            lg = l0 if li == 0 else (u @ gate.T).float()
            h = h + ep(u, lg, ws)  # residual
        if out is not None:
            out.copy_(h)
        return h

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step(x, logits0)
    ops.check_device()
    clocks = ClockSampler(torch.cuda.current_device()).start()
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = ops.launch_count()
    t0.record()
    for _ in range(args.steps):
        step(x, logits0)
    t1.record()
    launches = ops.launch_count() - n0
    t1.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    ops.check_device()

    # ---- dominant kernel alone: gate/up on this rank's expected share of rows
    # (T_total * k / N routed rows spread evenly over its E/N experts)
    R = T_total * k // world
    offs = torch.tensor([(R * (j + 1)) // shard.local for j in range(shard.local)], dtype=torch.int32, device=dev)
    xl = torch.randn(R, H, device=dev).to(torch.bfloat16)
    hl = torch.empty((R, I), dtype=torch.bfloat16, device=dev)
    # the weights the layer's GEMMs multiply (NF4 staged to bf16 copies where that pays)
    w1, w3, _ = ops.stage_nf4(stack[0][1], R, shard.local, training=train)
    staged = w1 is not stack[0][1][0]
    kclocks = ClockSampler(torch.cuda.current_device()).start()
    for _ in range(3):
        ops.gateup_swiglu(xl, offs, w1, w3, inter=I, out=hl)
    reps = max(5, min(20, args.steps))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, bb in evs:
        a.record()
        ops.gateup_swiglu(xl, offs, w1, w3, inter=I, out=hl)
        bb.record()
    torch.cuda.synchronize()
    gu_ms = sum(a.elapsed_time(bb) for a, bb in evs) / reps
    kclk = kclocks.stop()
    del xl, hl

    # ---- end to end with host buffers (each rank: its tokens and layer-0 logits up, its output down)
    host_in = [x.cpu().pin_memory(), logits0.cpu().pin_memory()] + ([g_out.cpu().pin_memory()] if train else [])
    e2e_ms = measure_e2e(dev, host_in, 2 if train else 1, (T_r, H),
                         lambda din, dout: step(din[0], din[1], out=dout[0], gin=din[2] if train else None,
                                                dx_out=dout[1] if train else None), args, barrier)

    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    if layer is not None:
        layer.close()
    ops.set_gemm_sm_limit(0)
    peaks = load_peaks()
    flops_gu = 4.0 * R * H * I
    achieved = flops_gu / (gu_ms * 1e-3) / 1e12
    S_total = T_total * k
    return {
        "metric": METRIC,
        "value": T_total / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations x " + cfg["fmt"] + " weights, fp32 accumulate",
        "data": "synthetic (seeded torch.randn tokens and router gates; random-init experts quantised on the GPU)",
        "config": {
            "workload": f"{args.config}: " + (f"a stack of {layers} routed expert FFN layers" if layers > 1 else
                                              "one routed expert FFN layer") +
                        (f" forward + dX backward with a rank-{LORA_RANK} LoRA on w2 (adapter grads included)"
                         if train else " forward") + f", expert-parallel over {world} GPU(s), T={T_total} tokens in total "
                        f"({T_r} on rank 0), H={H} E={E} ({shard.local} per GPU) k={k} I={I} {cfg['fmt']} experts",
            "tokens_total": T_total, "hidden": H, "experts": E, "experts_per_gpu": shard.local, "top_k": k,
            "intermediate": I, "layers": layers, "weights": cfg["fmt"],
            **({"nf4_decode": "once per layer into bf16 copies of the rank's experts, then the bf16 GEMMs "
                              f"(staging {args.nf4_staging})" if staged else
                              f"inside the GEMMs' main loops (staging {args.nf4_staging})"}
               if cfg["fmt"] == "nf4" else {}),
            "parallelism": f"ep{world}: experts sharded by contiguous blocks, tokens sharded by rank, " + (
                f"copy-engine transfers into {args.ep_layout}-major peer-mapped receive buffers (CUDA IPC over "
                f"NVLink, {args.ep_copy_streams} copy stream(s), regroup {args.ep_regroup}), arrival marked by "
                "epoch flags in the peers' buffers" if ipc else "NCCL all_to_all_single dispatch and return (source-major segments)")
                + (f"; {chunks} chunks per layer, exchanges on a second stream overlapping the GEMMs"
                   f" (GEMMs capped at {torch.cuda.get_device_properties(dev).multi_processor_count - free_sms} SMs)"
                   if chunks > 1 and world > 1 else ""),
            "l2": "no flush: each layer's routed activations exceed the 126 MB L2",
            **({"timed_outside_path": "per layer after the first: an RMS norm and the router logits "
                                      "(u @ gate.T) in torch/cuBLAS, and the residual add; they feed the "
                                      "next layer's routing and are not part of the routed expert FFN"}
               if layers > 1 else {}),
        },
        "tflops": (12.0 if train else 6.0) * S_total * H * I * layers / (ms * 1e-3) / 1e12,
        "roofline": {
            "kernel": f"gateup_swiglu_{'bf16 (NF4 staged)' if staged else cfg['fmt']}",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": achieved / peaks["bf16_tflops"],
            "peak_source": f"{peaks['source']} bf16 dense (burst; kernel timed alone)",
            "algorithmic": f"4*R*H*I = {flops_gu / 1e9:.1f} GFLOP per launch, R = {R} rows of rank 0's share",
            "traffic": None,
            "clocks": kclk,
        },
        "e2e": {
            "value": T_total / (e2e_ms * 1e-3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": T_r * H * 2 * (2 if train else 1) + T_r * E * 4,
            "d2h_bytes_per_step": T_r * H * 2 * (2 if train else 1),
            "copies": "per rank: pinned host buffers; 2 slots, uploads and downloads on their own streams, "
                      f"each direction split over {args.e2e_copy_streams} stream(s)",
        },
        "gpu_launches": launches,
        "gpu_launches_scope": "rank 0 (every rank launches its own)",
        "gpu_launches_source": "libmirai_b200's own count of the kernels its entry points enqueued in the timed "
                               "region (mirai_b200_launch_count)",
        "clocks": clk,
    }


# ----------------------------------------------------------------------------- CPU reference (oracle port)

class CpuReference:
    """The CPU restatement of the reference's torch path (oracle/), on host cores.

    The reference's ``chunked_dequant`` runner (the default) dequantises every
    expert chunk on every forward, and its frozen-linear autograd functions
    dequantise again in backward (linear.py:116-125, 191-203).  One step of the
    workload is therefore costed as: the full dequantisation of all experts
    (once for a forward, twice for forward + dX), plus the routed compute of
    all T tokens, measured on a ``sample``-token slice and scaled by
    T / sample (the compute is linear in the tokens; the dequantisation is
    not, so it is charged once per T tokens, never per sample)."""

    def __init__(self, cfg, sample_tokens, seed=1234, train=False, rotation=False):
        import numpy as np
        from oracle import quant as oq

        self.cfg = cfg
        self.train = train
        rng = np.random.default_rng(seed)
        T, H, E, k, I = sample_tokens, cfg["H"], cfg["E"], cfg["k"], cfg["I"]
        self.T = T
        self.x = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        gate = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
        self.logits = (self.x @ gate.T).astype(np.float32)
        if cfg["zipf"]:
            p = 1.0 / np.arange(1, E + 1) ** cfg["zipf"]
            p = p / p.sum()
            self.logits = (self.logits + 2.0 * np.log(p)[None, :]).astype(np.float32)
        self.g = oq.bf16_round(rng.standard_normal((T, H)).astype(np.float32)) if train else None
        self.lora = None
        if train:
            self.lora = {"a": oq.bf16_round((rng.standard_normal((E, LORA_RANK, I)) / I ** 0.5).astype(np.float32)),
                         "b": oq.bf16_round((rng.standard_normal((E, H, LORA_RANK)) * 0.02).astype(np.float32)),
                         "scale": 16.0 / LORA_RANK}
        raw = [(rng.standard_normal(s) * 0.02).astype(np.float32) for s in ((E, I, H), (E, I, H), (E, H, I))]
        self.threads = os.cpu_count() or 1
        if cfg["fmt"] == "nf4":
            from concurrent.futures import ThreadPoolExecutor
            with ThreadPoolExecutor(self.threads) as pool:
                per = list(pool.map(lambda a: oq.nf4_quantize_2d(raw[a[0]][a[1]]),
                                    [(key, e) for key in range(3) for e in range(E)]))
            self.store = []
            for key in range(3):
                p = per[key * E:(key + 1) * E]
                self.store.append({"nf4": np.stack([q["packed"] for q in p]),
                                   "absmax": np.stack([q["absmax"] for q in p]),
                                   "nabsmax": np.stack([q["nested_absmax"] for q in p]),
                                   "offset": np.stack([q["offset"] for q in p]),
                                   "code": p[0]["code"], "ncode": p[0]["nested_code"],
                                   "shape": raw[key].shape})
        elif cfg["fmt"] == "int8":
            self.store = [oq.int8_quantize(w, oq.best_group_size(w.shape[-1]) if rotation else 0) for w in raw]
        else:
            self.store = [oq.bf16_round(w) for w in raw]

    def dequant(self):
        from concurrent.futures import ThreadPoolExecutor
        import numpy as np
        from oracle import quant as oq

        fmt = self.cfg["fmt"]
        if fmt == "bf16":
            return self.store

        def one(args):
            key, e = args
            if fmt == "nf4":
                g = self.store[key]
                _, o, i = g["shape"]
                return oq.nf4_dequantize_2d({"packed": g["nf4"][e], "absmax": g["absmax"][e],
                                             "nested_absmax": g["nabsmax"][e], "offset": g["offset"][e],
                                             "code": g["code"], "nested_code": g["ncode"]}, (o, i))
            q, s, gs = self.store[key]
            return oq.bf16_round(oq.int8_dequantize(q[e], s[e], gs))

        E = self.cfg["E"]
        with ThreadPoolExecutor(self.threads) as pool:
            flat = list(pool.map(one, [(key, e) for key in range(3) for e in range(E)]))
        return [np.stack(flat[key * E:(key + 1) * E]) for key in range(3)]

    def compute(self, dense):
        """The routed compute on the sample: forward, or forward + dX (the
        oracle's dX pass recomputes the expert forward it needs)."""
        from oracle import moe as om
        idx, w = om.route_topk(self.logits, self.cfg["k"])
        if self.train:
            return om.moe_backward_dx(self.x, idx, w, *dense, self.g, bf16=True, lora=self.lora)
        return om.moe_forward(self.x, idx, w, *dense, bf16=True)

    def step_seconds(self):
        """(seconds for one full-T step, dequantisation seconds, sample compute seconds)."""
        t = time.perf_counter()
        dense = self.dequant()
        t_deq = time.perf_counter() - t
        t = time.perf_counter()
        self.compute(dense)
        t_cmp = time.perf_counter() - t
        passes = 2 if self.train else 1
        return passes * t_deq + t_cmp * self.cfg["T"] / self.T, t_deq, t_cmp

    def describe(self, n):
        what = "forward + dX with a rank-16 LoRA on w2" if self.train else "forward"
        passes = "twice (forward and backward)" if self.train else "once"
        return (f"{n} step(s); each: the full dequantisation of all {self.cfg['E']} x 3 experts, charged {passes} "
                f"per {self.cfg['T']}-token step, plus the routed {what} of a {self.T}-token sample scaled by "
                f"{self.cfg['T']}/{self.T}; oracle/ numpy restatement of the reference torch path")


def cpu_sample_tokens(cfg):
    return min(cfg["T"], 4096 if not cfg.get("layers") else 1024)


def cpu_sample_cfg(cfg):
    """The CPU restatement runs one layer; for the expert-parallel stack it takes
    one GPU's share of the experts (16 of 128) so the host holds a few GB, and
    the rate is divided by the number of layers."""
    if cfg.get("layers"):
        return dict(cfg, E=16, layers=1), cfg["layers"], (f"one layer with 16 of {cfg['E']} experts, "
                                                         f"rate divided by {cfg['layers']} layers")
    return cfg, 1, ""


def run_reference(args, cfg):
    cfg, per, note = cpu_sample_cfg(cfg)
    train = args.mode == "train" and not cfg.get("layers")
    ref = CpuReference(cfg, cpu_sample_tokens(cfg), train=train, rotation=args.int8_rotation)
    for _ in range(args.warmup):
        ref.step_seconds()
    total = 0.0
    for _ in range(args.steps):
        total += ref.step_seconds()[0]
    sec = total / args.steps
    value = cfg["T"] / sec / per
    sample = ref.describe(args.steps) + (f"; {note}" if note else "")
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 numpy with bf16 rounding points",
        "data": "synthetic (seeded numpy)",
        "config": {"workload": f"{args.config} " + ("forward + dX" if train else "forward") + " (CPU, projected "
                   "to the full token count)", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def cpu_baseline(cfg, args):
    cfg, per, note = cpu_sample_cfg(cfg)
    train = args.mode == "train" and not cfg.get("layers")
    ref = CpuReference(cfg, cpu_sample_tokens(cfg), train=train, rotation=args.int8_rotation)
    ref.step_seconds()  # warm
    t = time.perf_counter()
    n, total = 0, 0.0
    while True:
        total += ref.step_seconds()[0]
        n += 1
        if time.perf_counter() - t > 10.0 or n >= 3:
            break
    sec = total / n
    return {"value": cfg["T"] / sec / per, "unit": "tokens/s", "cores": ref.threads, "kind": "port",
            "sample": ref.describe(n) + (f"; {note}" if note else "")}


# ----------------------------------------------------------------------------- probes (--probe)
# Measurements behind the profiles/ summaries, run as `bench.py --probe ...`
# (one process per GPU under torchrun, except gemms and epilogue):
#   bandwidth  bytes crossing NVLink per rank per second: NCCL all_to_all_single
#              vs copy-engine transfers into peer-mapped buffers (the ipc transport)
#   blocks     that copy-engine exchange (128 MB per rank) split into 1-128 copies
#              per peer on one or two streams: the cost of a copy
#   gemms      (one GPU) the owner's GEMMs on source-major rows vs the same rows
#              contiguous per expert
#   epilogue   (one GPU) c2's down dX with and without its SwiGLU-backward epilogue,
#              and the NF4 decode of one key
#   phases     CUDA-event times between the phases of one ExpertParallelMoE layer
#              (1 chunk) on rank 0, over 10 layers after 3 warm-up layers
#              (--config, --ep-layout, --ep-copy-streams, --ep-regroup)

def probe_bandwidth(dev, world, rank):
    import torch
    import torch.distributed as dist
    from mirai_b200 import _lib
    from mirai_b200.expert_parallel import PeerBuffers
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
        from mirai_b200.ops import check_device
        check_device()
        pb.release()
        res[name] = {"bytes_per_rank_remote": int(remote),
                     "nccl_all_to_all_ms": round(nccl_ms, 3), "nccl_GBps": round(remote / nccl_ms / 1e6, 1),
                     "copy_engine_ms": round(ce_ms, 3), "copy_engine_GBps": round(remote / ce_ms / 1e6, 1)}
        del x, y
    return res


def probe_blocks(dev, world, rank):
    """Copy-engine exchange of a fixed byte count per peer, split into n equal
    blocks per peer (one cudaMemcpyAsync each), on 1 or 2 streams."""
    import torch
    import torch.distributed as dist
    import numpy as np
    from mirai_b200 import _lib
    from mirai_b200.expert_parallel import PeerBuffers
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
    from mirai_b200.ops import check_device
    check_device()
    pb.release()
    return res


def probe_phases(dev, world, rank, config, layout="source", copy_streams=1, regroup="auto", train=False,
                 chunks=1):
    import torch
    import torch.distributed as dist
    from mirai_b200 import ops
    from mirai_b200.expert_parallel import ExpertParallelMoE, ExpertShard, shard_tokens
    cfg = dict(CONFIGS[config], layers=1)
    strong = CONFIGS[config].get("ep") == "strong"
    T_total = cfg["T"] if strong else cfg["T"] * world
    b, e = shard_tokens(T_total, world, rank)
    shard = ExpertShard(cfg["E"], world, rank)
    x, logits, stack = make_ep_workload(cfg, dev, rank, shard, e - b)
    layer = ExpertParallelMoE(shard, top_k=cfg["k"], inter=cfg["I"], chunks=chunks, layout=layout,
                              copy_streams=copy_streams, regroup=regroup)
    lora = g_out = None
    if train:
        gen = torch.Generator(device=dev).manual_seed(99 + rank)
        g_out = torch.randn(e - b, cfg["H"], device=dev, generator=gen).to(torch.bfloat16)
        lora = ops.DownLoRA(torch.randn(shard.local, LORA_RANK, cfg["I"], device=dev, generator=gen) * 0.03,
                            torch.randn(shard.local, cfg["H"], LORA_RANK, device=dev, generator=gen) * 0.02,
                            16.0 / LORA_RANK, compute_grads=True)

    def step():
        if not train:
            return layer.forward(x, logits, stack[0][1])
        _, st = layer.forward(x, logits, stack[0][1], train=True, lora=lora)
        return layer.backward(g_out, st, stack[0][1], lora=lora)

    events = []

    def hook(name, stream):  # records at its point in the stream
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        events.append((name, ev))

    layer.on_phase = hook
    for _ in range(3):
        events.clear()
        step()
    torch.cuda.synchronize()
    dist.barrier()
    acc: dict[str, float] = {}
    step_ms = 0.0
    for _ in range(10):
        events.clear()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        step()
        t1.record()
        torch.cuda.synchronize()
        step_ms += t0.elapsed_time(t1) / 10
        for i in range(1, len(events)):
            name = events[i][0]
            acc[name] = acc.get(name, 0.0) + events[i - 1][1].elapsed_time(events[i][1]) / 10
    layer.close()
    return {"config": config, "world": world, "tokens_rank0": e - b, "layout": layout, "copy_streams": copy_streams,
            "regroup": regroup, "train": train, "chunks": chunks,
            "phases_ms": {k: round(v, 3) for k, v in acc.items()}, "layer_ms": round(sum(acc.values()), 3),
            "step_ms": round(step_ms, 3)}


def probe_gemms(dev):
    """The owner's GEMMs on rows received source-major (``sources`` = G) against
    the same rows contiguous per expert, NF4, on one GPU: c2's segment sizes at 2
    GPUs (~2048 rows per source and expert) and c4's at 8 (~256), ragged.  Min
    and median of 7 alternating rounds of 20 launches each (ms)."""
    import torch
    import statistics
    from mirai_b200 import ops, tables
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



def probe_epilogue(dev):
    """c2's down dX on bf16 copies of NF4 weights with its full epilogue (saved
    gate/up read, SwiGLU backward, two outputs) against the same GEMM writing dh
    alone (``gate_up`` NULL), and the NF4 decode of one key (ms, CUDA events,
    mean of 30 launches after 3)."""
    import torch
    from mirai_b200 import _lib, ops, tables
    cfg = CONFIGS["c2"]
    T, H, E, k, I = cfg["T"], cfg["H"], cfg["E"], cfg["k"], cfg["I"]
    S = T * k
    g = torch.Generator(device=dev).manual_seed(0)
    w2q = ops.nf4_quantize((torch.randn(E, H, I, device=dev, generator=g) * 0.02).to(torch.bfloat16),
                           tables.nf4_code(dev), tables.dynamic_map(dev))
    w2 = ops.nf4_dequantize(w2q)
    offs = torch.tensor([(S * (j + 1)) // E for j in range(E)], dtype=torch.int32, device=dev)
    gy = torch.randn(S, H, device=dev, generator=g).to(torch.bfloat16)
    gu = torch.randn(S, 2 * I, device=dev, generator=g).to(torch.bfloat16)
    dgu = torch.empty(S, 2 * I, dtype=torch.bfloat16, device=dev)
    dh = torch.empty(S, I, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    res = {
        "down_dx_full_ms": time_kernel(lambda: ops.down_dx(gy, offs, w2, gu, inter=I, out=dgu), 30),
        "down_dx_dh_only_ms": time_kernel(lambda: _lib.call("mirai_moe_down_dx_src_bf16", gy.data_ptr(),
                                                            offs.data_ptr(), 1, E, S, H, I, w2.data_ptr(), None,
                                                            dh.data_ptr(), stream), 30),
        "nf4_dequantize_one_key_ms": time_kernel(lambda: ops.nf4_dequantize(w2q, out=w2), 30),
    }
    ops.check_device()
    return res


def run_probe(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if args.probe in ("gemms", "epilogue"):  # one GPU, no process group
        dev = torch.device("cuda", 0)
        print(json.dumps(probe_gemms(dev) if args.probe == "gemms" else probe_epilogue(dev)), flush=True)
        return
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if args.probe == "bandwidth":
            res = probe_bandwidth(dev, world, rank)
        elif args.probe == "blocks":
            res = probe_blocks(dev, world, rank)
        else:
            res = probe_phases(dev, world, rank, args.config, args.ep_layout, args.ep_copy_streams, args.ep_regroup,
                               train=args.mode == "train", chunks=args.ep_chunks)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default=None, choices=["fwd", "train"],
                    help="train (default for c0-c3, at every GPU count: BASELINE config 2's step): forward + dX "
                         "backward through the frozen experts with a rank-16 LoRA on w2; fwd: forward only (the "
                         "default for the c4 stack)")
    ap.add_argument("--int8-rotation", action="store_true",
                    help="c3: INT8 in the reference's default block-Hadamard format (groups of 256)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-copy-streams", type=int, default=1,
                    help="end-to-end timing: streams (copy engines) each direction's host copies are split over")
    ap.add_argument("--nf4-staging", default="auto", choices=["auto", "always", "never"],
                    help="NF4 experts: decode each key once per pass into bf16 copies for the bf16 GEMMs "
                         "(always), decode inside the GEMMs (never), or stage training passes with many rows "
                         "per expert (auto)")
    ap.add_argument("--ep-chunks", type=int, default=2,
                    help="N > 1: token chunks per layer whose exchanges overlap the other chunks' GEMMs")
    ap.add_argument("--ep-free-sms", type=int, default=None,
                    help="N > 1: SMs the GEMMs leave free for communication kernels (default 2 ipc, 16 nccl)")
    ap.add_argument("--ep-layout", default="source", choices=["expert", "source"],
                    help="ipc transport: receive rows expert-major (a copy per (peer, expert) block) or "
                         "source-major (a copy per peer; G segments per expert in the GEMMs)")
    ap.add_argument("--ep-regroup", default="auto", choices=["never", "auto", "always"],
                    help="ipc transport, source-major layout: owners regroup received rows expert-major before "
                         "the GEMMs where that saves more GEMM time than the two row gathers cost")
    ap.add_argument("--ep-copy-streams", type=int, default=1,
                    help="ipc transport: side streams a chunk's copy blocks are spread over (by peer)")
    ap.add_argument("--ep-transport", default="ipc", choices=["ipc", "nccl"],
                    help="N > 1: copy-engine transfers into peer-mapped buffers, or NCCL all_to_all_single")
    ap.add_argument("--tokens", type=int, default=None,
                    help="override the workload's token count (small cases for profiler captures)")
    ap.add_argument("--probe", default=None, choices=["bandwidth", "blocks", "phases", "gemms", "epilogue"],
                    help="run one expert-parallel measurement instead of the benchmark (see the probes section)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.probe:
        run_probe(args)
        return
    cfg = CONFIGS[args.config] if args.tokens is None else dict(CONFIGS[args.config], T=int(args.tokens))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.mode is None:  # BASELINE config 2's step at every GPU count; the c4 stack runs forward
        args.mode = "fwd" if cfg.get("layers") else "train"
    if args.mode == "train" and cfg.get("layers"):
        raise SystemExit("--mode train runs single-layer workloads (c0-c3)")
    if args.int8_rotation and cfg["fmt"] != "int8":
        raise SystemExit("--int8-rotation applies to the INT8 workload (c3)")

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, cfg)), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        from mirai_b200 import _lib, ops
        _lib.load()
        ops.set_nf4_staging(args.nf4_staging)
        line = run_ep(args, cfg, rank, world, dev) if (world > 1 or cfg.get("layers")) else \
            run_ours(args, cfg, rank, world, dev)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:  # the host-core baseline, N = 1 only
            line["cpu_baseline"] = cpu_baseline(cfg, args)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
