#!/usr/bin/env python
"""Benchmark of the quantized-expert MoE decode path on B200s.

A step decodes one token (per rank) through a chain of L distinct MoE layers of configuration 2: hidden 2048,
512 experts of SwiGLU inner 512 as GGUF blocks, top-10 softmax router (float16 weights), a shared expert of
inner 512 with its sigmoid gate, bfloat16 activations. Experts alternate Q2_0 / IQ3_S layer by layer. Weights
are seeded synthetic blocks made in HBM (no model files exist); each layer's weights are distinct, so a step
reads ~0.6 GB of routed expert blocks from HBM, far more than the 126 MB L2, with a fresh token every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0. `value` is tokens/s with the token already in HBM (the chain replayed as a CUDA graph);
`e2e` is the same through the public API (strata_mlx_b200.fused.DecodeGraph) from pinned host memory, copies in
the timed region. `roofline` times the dominant kernel (the routed experts' fused gate/up matvec) alone, 48
launches in a graph, against the measured HBM copy bandwidth. `cpu_baseline` is the C oracle on the host cores.
`--impl reference` times the C oracle (strata-mlx's block decode and MoE block restated in C: the reference's own
implementation is Metal, which has no CPU form) on all host cores, for the same config and metric.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, I, E, K, IS = 2048, 512, 512, 10, 512
METRIC = "decode tok/s and expert-matvec HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
BLOCK = {"Q2_0": (64, 18), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98)}


def row_bytes(kind: str, cols: int) -> int:
    pb, bb = BLOCK[kind]
    return cols // pb * bb


def kind_of(layer: int, mode: str) -> str:
    return ("Q2_0" if layer % 2 == 0 else "IQ3_S") if mode == "mixed" else mode


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "source": "fallback"}


# ---- distributed plumbing


def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def reduce_max(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---- clocks during the timed region


class Clocks:
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(device_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---- the workload


def build_layers(n_layers: int, mode: str, rank: int, device, first: int = 0):
    """The chain's layers on one device, every expert: the same model as build_ep_layers makes (seeds of the layer
    index only, EP_SIGMA scales), layers [first, first + n_layers)."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as F
    from strata_mlx_b200.synthetic import blocks_cuda

    layers = []
    for l in range(first, first + n_layers):
        kind = kind_of(l, mode)
        seed = 10 * l
        sig = EP_SIGMA.get(kind, 0.02)
        g = torch.Generator(device=device)
        g.manual_seed(seed + 7)
        lin = {
            "gate": B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, seed + 1, device, sigma=sig), kind, (E, I, H)),
            "up": B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, seed + 2, device, sigma=sig), kind, (E, I, H)),
            "down": B.BlockSwitchLinear(blocks_cuda(kind, E, H, I, seed + 3, device, sigma=sig), kind, (E, H, I)),
            "sgate": B.BlockSwitchLinear(blocks_cuda(kind, 1, IS, H, seed + 4, device, sigma=sig), kind, (1, IS, H)),
            "sup": B.BlockSwitchLinear(blocks_cuda(kind, 1, IS, H, seed + 5, device, sigma=sig), kind, (1, IS, H)),
            "sdown": B.BlockSwitchLinear(blocks_cuda(kind, 1, H, IS, seed + 6, device, sigma=sig), kind, (1, H, IS)),
        }
        router = (torch.randn((E, H), generator=g, device=device) * 0.02).half()
        sgw = (torch.randn((H,), generator=g, device=device) * 0.02).half()
        layer = F.MoEDecodeLayer(router, lin["gate"], lin["up"], lin["down"], K,
                                 shared=(lin["sgate"], lin["sup"], lin["sdown"]), shared_gate=sgw, dtype=torch.bfloat16)
        layer.kind, layer.lin = kind, lin
        layers.append(layer)
    return layers


# Expert scales of the expert-parallel chain, whose layers take the previous layer's outputs: N(0, sigma) block
# scales that keep a layer's outputs O(1) for O(1) inputs (measured with the oracle on one expert: output std 0.43 at
# Q2_0's 0.02, 663 at IQ3_S's 0.002, growing as sigma^3). At 0.02 the IQ3 layers' outputs reach ~1e6 and overflow to
# inf / NaN within four layers, and NaN logits send the top-k to its slow path.
EP_SIGMA = {"Q2_0": 0.025, "IQ3_S": 2.4e-4, "IQ3_XXS": 2.4e-4}
EP_REFEED = 2  # the token is fed again every two layers (EPDecodeChain refeed): the chain stays finite


def build_ep_layers(n_layers: int, mode: str, rank: int, world: int, device):
    """The chain's layers, expert parallel: every rank makes the same model (the seeds do not depend on the rank)
    and keeps its share of each layer's routed experts; the router and shared expert are replicated."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import ep as EP
    from strata_mlx_b200.synthetic import blocks_cuda

    e0, e1 = EP.expert_range(rank, world, E)
    layers = []
    for l in range(n_layers):
        kind = kind_of(l, mode)
        seed = 10 * l
        g = torch.Generator(device=device)
        g.manual_seed(seed + 7)
        mine = {}
        sig = EP_SIGMA.get(kind, 0.02)
        for name, shp, sd in (("gate", (E, I, H), 1), ("up", (E, I, H), 2), ("down", (E, H, I), 3)):
            full = blocks_cuda(kind, *shp, seed + sd, device, sigma=sig)
            mine[name] = B.BlockSwitchLinear(EP.local_experts(full, E, rank, world), kind, (e1 - e0,) + shp[1:])
            del full
        shared = tuple(B.BlockSwitchLinear(blocks_cuda(kind, 1, r, c, seed + sd, device, sigma=sig), kind, (1, r, c))
                       for r, c, sd in ((IS, H, 4), (IS, H, 5), (H, IS, 6)))
        router = (torch.randn((E, H), generator=g, device=device) * 0.02).half()
        sgw = (torch.randn((H,), generator=g, device=device) * 0.02).half()
        layer = EP.EPMoEDecodeLayer(router, mine["gate"], mine["up"], mine["down"], K, E, shared=shared,
                                    shared_gate=sgw, dtype=torch.bfloat16)
        layer.kind = kind
        layers.append(layer)
    torch.cuda.empty_cache()
    return layers


def ep_parity(layers, eager, x_in, refeed: int, args, world: int, rank: int, device, cs) -> bool | None:
    """Bit-identity of the expert-parallel chain with one device, checked on every rank before anything is timed:
    for 3 steps, this rank's output of the chain (eager) against the single-device MoEDecodeLayer (every expert) on
    the window of all ranks' tokens. With refeed r the chain's output depends only on its last r layers (each
    segment starts again from the step's token), so those are built on one device. Returns the AND over ranks."""
    import torch.distributed as dist

    if not refeed:
        return None
    ref = build_layers(refeed, args.kinds, rank, device, first=len(layers) - refeed)
    windows = []
    for r in range(world):  # every rank's tokens, made as that rank makes them
        g = torch.Generator(device=device)
        g.manual_seed(99 + r)
        windows.append(torch.randn((3, H), generator=g, device=device).to(torch.bfloat16))
    ok = True
    with torch.cuda.stream(cs):
        for i in range(3):
            x_in.copy_(windows[rank][i : i + 1])
            got = eager().clone()
            X = torch.cat([w[i : i + 1] for w in windows])
            y = X
            for l in ref:
                y = l(y)
            ok = ok and bool(torch.equal(got.reshape(1, H), y[rank : rank + 1]))
    torch.cuda.synchronize()
    for l in ref:
        l.check_errors()
    del ref
    torch.cuda.empty_cache()
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def run_ep(args, world, rank, local) -> None:
    """N > 1: expert parallel decode, one token per rank per step through the chain; the exchange of each layer is
    an NCCL all-gather and all-reduce (strata_mlx_b200/ep.py)."""
    import torch.distributed as dist
    from strata_mlx_b200 import _lib

    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    layers = build_ep_layers(args.layers, args.kinds, rank, world, device)
    gen = torch.Generator(device=device)
    gen.manual_seed(99 + rank)
    n_tok = args.steps + args.warmup
    xs = torch.randn((n_tok, H), generator=gen, device=device).to(torch.bfloat16)
    x_in = torch.empty((1, H), dtype=torch.bfloat16, device=device)
    torch.cuda.synchronize()

    chain = None
    if len(layers) % 2 == 0 and os.environ.get("SC_EP_NCCL") != "1":
        from strata_mlx_b200 import ep as EP

        chain = EP.EPDecodeChain(layers, 1, device)  # the exchange in the kernels, over peer memory

    refeed = EP_REFEED if len(layers) % EP_REFEED == 0 else 0

    def eager():
        if chain is not None:
            return chain(x_in, refeed=refeed)
        y = x_in
        for i, l in enumerate(layers):
            y = l(x_in if refeed and i % refeed == 0 else y)
        return y

    # the chain with its collectives captured as one CUDA graph (released before the process group ends)
    cs = torch.cuda.Stream(device=device)
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        for i in range(3):
            x_in.copy_(xs[i : i + 1])
            eager()
    torch.cuda.current_stream().wait_stream(cs)
    torch.cuda.synchronize()
    barrier(world)
    bits_same = ep_parity(layers, eager, x_in, refeed, args, world, rank, device, cs)
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cs):
            y_out = eager()
        torch.cuda.synchronize()
    barrier(world)

    def step():
        if graph is None:
            return eager()
        graph.replay()
        return y_out

    s = torch.cuda.current_stream()
    for i in range(args.warmup):
        x_in.copy_(xs[i : i + 1])
        step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(args.steps):
        x_in.copy_(xs[args.warmup + i : args.warmup + i + 1])
        step()
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = reduce_max(e0.elapsed_time(e1) / args.steps, world)
    barrier(world)
    _lib.check_device_errors(device)
    last = eager() if graph is None else y_out  # (every rank runs the extra eager step: the exchange needs all)
    finite = bool(torch.isfinite(last.float()).all().item())

    # e2e: the public call per layer, the rank's token from pinned host memory, its result back to the host
    host_x = xs.cpu().pin_memory()
    e2e_steps = min(args.steps, 200)
    for i in range(3):
        x_in.copy_(host_x[i : i + 1], non_blocking=True)
        step().cpu()
    barrier(world)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        x_in.copy_(host_x[(args.warmup + i) % n_tok : (args.warmup + i) % n_tok + 1], non_blocking=True)
        step().cpu()
    e2e_ms = reduce_max((time.perf_counter() - t0) / e2e_steps * 1000.0, world)

    # bytes a rank must read per step: its experts' share of the window's pairs (world tokens x K pairs spread over
    # world ranks: K pairs per rank on average) plus the replicated router and shared expert
    per_rank = sum(stage_bytes(l.kind)["gate_up"] + stage_bytes(l.kind)["down"] + stage_bytes(l.kind)["route"]
                   for l in layers)
    pk = peaks()
    achieved = per_rank / (ms * 1e-3) / 1e9
    cfg = workload_config(args, world)
    cfg["refeed"] = refeed
    cfg["expert_sigma"] = EP_SIGMA
    cfg["outputs_finite"] = finite
    cfg["ep_bits_same"] = bits_same
    cfg["ep_bits_same_how"] = (f"before timing, 3 steps of the chain on every rank against the single-device decode "
                               f"block (all 512 experts) on the window of every rank's tokens, through the last "
                               f"{refeed}-layer segment the chain's output depends on")
    cfg["parallelism"] = (f"ep{world}: experts sharded over ranks, the exchange in the kernels over peer memory "
                          "(NVLink stores, release/acquire counts)" if chain is not None else
                          f"ep{world}: experts sharded over ranks, NCCL all-gather + all-reduce per layer")
    line = {"metric": METRIC, "value": world * 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded GGUF blocks and float16 router made in HBM",
            "config": cfg,
            "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": H * 2,
                    "d2h_bytes_per_step": H * 2,
                    "api": "strata_mlx_b200.ep.EPDecodeChain.__call__" if chain is not None else
                           "strata_mlx_b200.ep.EPMoEDecodeLayer.__call__ per layer"},
            "roofline": {"bound": "hbm", "kernel": "the whole expert-parallel step of a rank (kernels + exchange)",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": pk["source"], "traffic": None},
            "gpu_launches": (4 * args.layers + (1 if chain is not None else 0)) * args.steps,
            "gpu_launches_per_step": 4 * args.layers + (1 if chain is not None else 0), "clocks": clk}
    line["graph"] = graph is not None
    del graph
    torch.cuda.synchronize()
    barrier(world)
    if chain is not None:
        chain.check_errors()
        chain.close()
    del layers, chain
    torch.cuda.empty_cache()
    if not args.no_extra:
        line["config4"] = config4_result(world, rank, device, group=dist.group.WORLD)
        barrier(world)
        line["config5"] = config5_result(world, rank, device, group=dist.group.WORLD, steps=args.config5_steps)
        barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    barrier(world)
    dist.destroy_process_group()


# ---- configuration 3: the prefill grouped expert GEMM (--workload prefill)

PREFILL_KIND = "IQ3_XXS"


def prefill_result(steps: int, warmup: int, cpu_seconds: float | None) -> dict:
    """Configuration 3 on one GPU: a prefill chunk's 20,480 (token, expert) pairs through switch_glu's tiled
    path (tiles_of, the gate / up / down tile products on tcgen05, swiglu), IQ3_XXS experts, bf16 in, fp32 sums.
    `value`: TFLOP/s on the pairs' 6 * pairs * H * I flops; roofline: the gate product's kernel alone against the
    measured bf16 tensor peak (burst: the kernel is timed alone). cpu_seconds None: no CPU baseline."""
    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200.synthetic import PREFILL_TOKENS, ZIPF_S, blocks_cuda, prefill_routes

    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    kind = PREFILL_KIND
    gate = B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, 31, device), kind, (E, I, H))
    up = B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, 32, device), kind, (E, I, H))
    down = B.BlockSwitchLinear(blocks_cuda(kind, E, H, I, 33, device), kind, (E, H, I))
    idx_np = prefill_routes()
    counts = np.bincount(idx_np.reshape(-1), minlength=E)
    idx = torch.from_numpy(idx_np).to(device).reshape(1, PREFILL_TOKENS, K)
    gen = torch.Generator(device=device)
    gen.manual_seed(4)
    x = torch.randn((1, PREFILL_TOKENS, H), generator=gen, device=device).to(torch.bfloat16)
    pairs = PREFILL_TOKENS * K
    flops = 6.0 * pairs * H * I
    s = torch.cuda.current_stream()
    for _ in range(warmup):
        B.switch_glu(x, idx, up, gate, down)
    torch.cuda.synchronize()
    clocks = Clocks(device.index)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        B.switch_glu(x, idx, up, gate, down)
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    _lib.check_device_errors(device)

    # the gate product's kernel alone (the dominant kernel: the three products are alike in flops)
    te, token, where = B.tiles_of(idx, E)
    a = x.reshape(-1, H).index_select(0, token.to(torch.int64))
    for _ in range(3):
        B.tile_matmul(gate.blocks, kind, (E, I, H), a, te)
    torch.cuda.synchronize()
    reps = 20
    e0.record(s)
    for _ in range(reps):
        B.tile_matmul(gate.blocks, kind, (E, I, H), a, te)
    e1.record(s)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / reps
    k_tflops = 2.0 * pairs * I * H / (k_ms * 1e-3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk, src = float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        tpk, src = 1590.0, "fallback"

    # e2e: the reference's call (switch_glu) from pinned host activations, the pairs' outputs back to the host
    # (pinned host buffers both ways)
    host_x = x.cpu().pin_memory()
    e2e_steps = min(steps, 10)
    out = B.switch_glu(host_x.to(device, non_blocking=True), idx, up, gate, down)
    host_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    host_out.copy_(out, non_blocking=True)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_out.copy_(B.switch_glu(host_x.to(device, non_blocking=True), idx, up, gate, down), non_blocking=True)
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) / e2e_steps * 1000.0
    res = {"metric": "prefill grouped expert GEMM TFLOP/s (config 3)", "value": flops / (ms * 1e-3) / 1e12,
           "unit": "TFLOP/s", "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
           "dtype": "bf16", "data": "synthetic: seeded IQ3_XXS blocks made in HBM, seeded Zipf-skewed routes",
           "config": {"workload": "config3: prefill grouped expert GEMM, 2048-token chunk, top-10 of 512 experts "
                                  "(hidden 2048, SwiGLU inter 512), IQ3_XXS, bf16 in / fp32 accumulate",
                      "pairs": pairs, "experts_used": int((counts > 0).sum()), "max_pairs_per_expert": int(counts.max()),
                      "median_pairs_per_used_expert": float(np.median(counts[counts > 0])), "zipf_s": ZIPF_S,
                      "flops_per_step": flops,
                      "l2": "inputs larger than L2: 3 x 401 MB of expert blocks, ~360 experts' share read per step"},
           "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                   "h2d_bytes_per_step": PREFILL_TOKENS * H * 2, "d2h_bytes_per_step": int(host_out.numel()) * 2,
                   "api": "strata_mlx_b200.blocks.switch_glu"},
           "roofline": {"bound": "tensor", "kernel": "tile_mma_kernel (the gate product, 512 x 2048)",
                        "achieved": k_tflops, "peak": tpk, "unit": "TFLOP/s", "frac": k_tflops / tpk,
                        "peak_source": src, "traffic": None, "us_per_launch": k_ms * 1e3},
           # per step: tiles_of, slot_pairs, the gate / up products, swiglu, the down product
           "gpu_launches": 6 * steps, "gpu_launches_per_step": 6, "clocks": clk}
    if cpu_seconds:
        res["cpu_baseline"] = prefill_cpu_sample(pairs, flops, cpu_seconds)
    del gate, up, down
    torch.cuda.empty_cache()
    return res


def run_prefill(args, world, rank) -> None:
    """--workload prefill: configuration 3 as a line of its own."""
    res = prefill_result(args.steps, args.warmup, None if args.no_cpu_baseline else 10.0)
    line = {"metric": res.pop("metric"), "value": res.pop("value"), "unit": res.pop("unit"), "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "scaling": "weak", "vs_baseline": None, **res}
    print(json.dumps(line), flush=True)


# ---- configuration 1: one IQ3_S SwiGLU expert, float32 activations, batch 1

C1_KIND, C1_COPIES = "IQ3_S", 256


def config1_result(reps: int = 20, cpu_seconds: float = 5.0) -> dict:
    """One SwiGLU expert (gate / up 2048 -> 512, down 512 -> 2048) as IQ3_S blocks, x float32 N(0, 1), batch 1,
    through the reference's call (switch_glu of one token and one expert: gate and up products, swiglu, down).
    C1_COPIES distinct copies of the expert (346 MB, more than L2) are called in turn, the calls replayed as a CUDA
    graph. Bytes per call: the expert's 1,351,680 B of blocks."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200.synthetic import blocks_cuda

    device = torch.device("cuda", torch.cuda.current_device())
    gate = B.BlockSwitchLinear(blocks_cuda(C1_KIND, C1_COPIES, I, H, 41, device), C1_KIND, (C1_COPIES, I, H))
    up = B.BlockSwitchLinear(blocks_cuda(C1_KIND, C1_COPIES, I, H, 42, device), C1_KIND, (C1_COPIES, I, H))
    down = B.BlockSwitchLinear(blocks_cuda(C1_KIND, C1_COPIES, H, I, 43, device), C1_KIND, (C1_COPIES, H, I))
    gen = torch.Generator(device=device)
    gen.manual_seed(1)
    x = torch.randn((1, H), generator=gen, device=device)
    ids = [torch.tensor([[e]], dtype=torch.int32, device=device) for e in range(C1_COPIES)]
    nbytes = 2 * I * row_bytes(C1_KIND, H) + H * row_bytes(C1_KIND, I)
    st = torch.cuda.Stream(device=device)
    with torch.cuda.stream(st):
        for e in range(C1_COPIES):
            B.switch_glu(x, ids[e], up, gate, down)
    st.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for e in range(C1_COPIES):
            out = B.switch_glu(x, ids[e], up, gate, down)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        g.replay()
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * C1_COPIES)
    # e2e: the token from pinned host memory, the call, the result back to pinned host memory
    hx = x.cpu().pin_memory()
    ho = torch.empty((1, H), dtype=torch.float32).pin_memory()
    for e in range(3):
        ho.copy_(B.switch_glu(hx.to(device, non_blocking=True), ids[e], up, gate, down).reshape(1, H), non_blocking=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n_e2e = 200
    for i in range(n_e2e):
        ho.copy_(B.switch_glu(hx.to(device, non_blocking=True), ids[i % C1_COPIES], up, gate, down).reshape(1, H),
                 non_blocking=True)
    torch.cuda.synchronize()
    e2e_us = (time.perf_counter() - t0) / n_e2e * 1e6
    pk = peaks()
    res = {"workload": "config1: one SwiGLU expert (gate/up 2048->512, down 512->2048) as IQ3_S blocks, x float32 "
                       "N(0,1), batch 1, through blocks.switch_glu",
           "bytes_per_call": nbytes, "us_per_call": us, "gbs": nbytes / (us * 1e-6) / 1e9,
           "roofline": {"bound": "hbm", "achieved": nbytes / (us * 1e-6) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                        "frac": nbytes / (us * 1e-6) / 1e9 / pk["hbm_gbs"], "peak_source": pk["source"]},
           "e2e": {"us_per_call": e2e_us, "gbs": nbytes / (e2e_us * 1e-6) / 1e9, "h2d_bytes_per_step": H * 4,
                   "d2h_bytes_per_step": H * 4, "api": "strata_mlx_b200.blocks.switch_glu"},
           "l2": f"{C1_COPIES} distinct copies of the expert called in turn ({C1_COPIES * nbytes / 1e6:.0f} MB > L2)",
           "gpu_launches_per_call": 4}
    if cpu_seconds:
        from oracle import cref
        from strata_mlx_b200.synthetic import blocks_numpy

        threads = cref.threads(os.cpu_count() or 1)
        rng = np.random.default_rng(0)
        k = cref.KINDS[C1_KIND]
        wg, wu = blocks_numpy(C1_KIND, 1, I, H, rng), blocks_numpy(C1_KIND, 1, I, H, rng)
        wd = blocks_numpy(C1_KIND, 1, H, I, rng)
        xx = rng.standard_normal(H).astype(np.float32)
        og, ou, od = np.empty(I, np.float32), np.empty(I, np.float32), np.empty(H, np.float32)
        lib = cref.lib()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < cpu_seconds or n < 3:
            lib.ref_matvec(k, wg.ctypes.data, I, H, xx.ctypes.data, og.ctypes.data)
            lib.ref_matvec(k, wu.ctypes.data, I, H, xx.ctypes.data, ou.ctypes.data)
            with np.errstate(over="ignore"):
                h = (og / (1 + np.exp(-og)) * ou).astype(np.float32)
            lib.ref_matvec(k, wd.ctypes.data, H, I, h.ctypes.data, od.ctypes.data)
            n += 1
        cus = (time.perf_counter() - t0) / n * 1e6
        res["cpu_baseline"] = {"value": nbytes / (cus * 1e-6) / 1e9, "unit": "GB/s", "us_per_call": cus,
                               "cores": threads, "kind": "port",
                               "sample": f"{n} calls of the C oracle (decode + float32 matvec, OpenMP) in ~{cpu_seconds:.0f} s"}
    del gate, up, down, g
    torch.cuda.empty_cache()
    return res


def prefill_cpu_sample(pairs: int, flops: float, seconds: float = 10.0) -> dict:
    """The C oracle (decode + float32 matvec per pair, all host cores) on a bounded sample of pairs of the same
    shapes, scaled to the step's pairs."""
    from oracle import cref
    from strata_mlx_b200.synthetic import blocks_numpy

    threads = cref.threads(os.cpu_count() or 1)
    rng = np.random.default_rng(3)
    lib = cref.lib()
    k = cref.KINDS[PREFILL_KIND]
    w_gu = blocks_numpy(PREFILL_KIND, 1, I, H, rng)
    w_d = blocks_numpy(PREFILL_KIND, 1, H, I, rng)
    x = rng.standard_normal(H).astype(np.float32)
    h = rng.standard_normal(I).astype(np.float32)
    og, od = np.empty(I, np.float32), np.empty(H, np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 3:
        for w, xin, o, r, c in ((w_gu, x, og, I, H), (w_gu, x, og, I, H), (w_d, h, od, H, I)):
            lib.ref_matvec(k, w.ctypes.data, r, c, xin.ctypes.data, o.ctypes.data)
        n += 1
    per_pair = (time.perf_counter() - t0) / n
    return {"value": flops / (per_pair * pairs) / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n} pairs' gate, up and down products timed (~{seconds:.0f} s), scaled to {pairs} pairs"}


# ---- the reference's unfused call at a mid-size batch

MB_TOKENS, MB_LAYERS = 64, 3


def mid_batch_result(reps: int = 10, layers: int = MB_LAYERS) -> dict:
    """The reference's unfused expert call for a mid-size batch: blocks.switch_glu of 64 tokens x top-10 of 512
    experts (config-2 shapes: gate / up 2048 -> 512, down 512 -> 2048), bfloat16 x -- the gate/up product with
    swiglu (sc_expert_gate_up) and the down product (sc_expert_matvec), both on the grouped fragment kernel. Three
    layers' stacks of each block type with seeded uniform routes are called in turn from a CUDA graph (a call's
    distinct experts are ~0.4-0.5 GB of blocks: more than L2). Bytes per call: the distinct experts' gate, up and
    down rows."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200.synthetic import blocks_cuda

    device = torch.device("cuda", torch.cuda.current_device())
    pk = peaks()
    out = {"workload": f"{MB_TOKENS} tokens x top-{K} of {E} experts (gate/up {H}->{I}, down {I}->{H}), bfloat16 x, "
                       "through blocks.switch_glu (BlockSwitchLinear products)", "api": "strata_mlx_b200.blocks.switch_glu",
           "gpu_launches_per_call": 2}
    for kind in ("Q2_0", "IQ3_S"):
        rng = np.random.default_rng(5)
        calls, nbytes = [], []
        for l in range(layers):
            gate = B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, 60 + 3 * l, device), kind, (E, I, H))
            up = B.BlockSwitchLinear(blocks_cuda(kind, E, I, H, 61 + 3 * l, device), kind, (E, I, H))
            down = B.BlockSwitchLinear(blocks_cuda(kind, E, H, I, 62 + 3 * l, device), kind, (E, H, I))
            idx = np.stack([rng.choice(E, K, replace=False) for _ in range(MB_TOKENS)]).astype(np.int32)
            x = torch.from_numpy(rng.standard_normal((MB_TOKENS, H)).astype(np.float32)).to(device, torch.bfloat16)
            calls.append((x, torch.from_numpy(idx).to(device), up, gate, down))
            used = len(np.unique(idx))
            nbytes.append(used * (2 * I * row_bytes(kind, H) + H * row_bytes(kind, I)))
        g, _ = graph_of(lambda: [B.switch_glu(*c) for c in calls], device)
        st = torch.cuda.Stream(device=device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            g.replay()
            e0.record(st)
            for _ in range(reps):
                g.replay()
            e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * layers)
        gbs = float(np.mean(nbytes)) / (us * 1e-6) / 1e9
        out[kind] = {"us_per_call": us, "bytes_per_call": float(np.mean(nbytes)), "gbs": gbs,
                     "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                  "frac": gbs / pk["hbm_gbs"], "peak_source": pk["source"]}}
        del g, calls
        torch.cuda.synchronize()
    return out


# ---- configurations 4 and 5: the synthetic decoder around the MoE blocks


def decoder_bytes(dec, routes_per_layer: list, ctx: int, world: int) -> float:
    """Bytes a rank reads in one pass: its share of the window's distinct experts (routes counted per layer), the
    shared expert, the router, the dense projections and the key/value cache up to `ctx` (all replicated)."""
    total = dec.dense_bytes + 2 * dec.vocab * dec.hidden  # projections; output head (bf16) and embedding rows
    for (per_expert, shared), used in zip(dec.expert_bytes, routes_per_layer):
        total += used * per_expert / world + shared + E * H * 2
    total += dec.n_layers * ctx * dec.kv_heads * 256 * 2 * 2
    return float(total)


def graph_of(fn, device):
    """fn captured as a CUDA graph on a side stream (after one warm call); returns (graph, its output)."""
    st = torch.cuda.Stream(device=device)
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        out = fn()
    torch.cuda.synchronize()
    return g, out


def config4_result(world: int, rank: int, device, group=None, passes: int = 20) -> dict:
    """Configuration 4: a verify pass of 1 + 4 tokens through 48 layers (attention 16 q / 2 kv heads of 256 over an
    8K context in 16-token pages, then the configuration-2 MoE block, experts Q2_0 / IQ3_S by layer), the experts
    sharded over the ranks (every rank holds the window; an NCCL all-reduce of the pairs' outputs a layer). The cache
    is filled with random keys and values (standing in for the prefill of an 8K prompt of random tokens). tok/s =
    5 / pass time; the pass replays from a CUDA graph at the same position."""
    from strata_mlx_b200 import decoder as D

    T, CTX = 5, 8192
    dec = D.SyntheticDecoder(48, ["Q2_0", "IQ3_S"], dense="bf16", device=device, group=group, mode="replicated",
                             max_pos=CTX + 64)
    cache = dec.cache(CTX + 16)
    cache.fill_random(CTX - T)
    g = torch.Generator(device=device)
    g.manual_seed(44)
    toks = torch.randint(0, dec.vocab, (T,), generator=g, device=device)
    graph, logits = graph_of(lambda: dec.forward(toks, cache), device)
    s = torch.cuda.current_stream()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(device.index)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(passes):
        graph.replay()
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = reduce_max(e0.elapsed_time(e1) / passes, world)
    dec.check_errors()
    used = [int(torch.unique(L["base"].routes(T, device)[0].view(torch.int32)).numel()) for L in dec.layers]
    nbytes = decoder_bytes(dec, used, CTX, world)
    pk = peaks()
    top1 = logits.argmax(-1).tolist()
    res = {"workload": "config4: speculative verify pass of 1 + 4 tokens, 48-layer synthetic MoE decoder (per layer "
                       "GQA attention 16 q / 2 kv heads of 256 with RoPE over a paged 8K cache, 16-token pages, bf16 "
                       "projections; the config-2 MoE block, experts Q2_0 / IQ3_S by layer)",
           "tok_per_s": T / (ms * 1e-3), "ms_per_pass": ms, "tokens_per_pass": T, "context": CTX,
           "parallelism": f"ep{world}: experts sharded, attention and dense replicated, NCCL all-reduce of the "
                          "pairs' outputs per layer" if world > 1 else "single",
           "roofline": {"bound": "hbm", "bytes_per_pass_per_rank": nbytes, "achieved": nbytes / (ms * 1e-3) / 1e9,
                        "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                        "what": "a rank's share of the window's distinct experts + shared expert + router + dense "
                                "projections + KV cache read, per pass"},
           "distinct_experts_per_layer_mean": float(np.mean(used)), "top1": top1,
           "kv_prefill": "random keys and values stand in for the prefill of the random-token prompt",
           "graph": True, "clocks": clk}
    del graph, dec, cache
    torch.cuda.empty_cache()
    return res


def config5_result(world: int, rank: int, device, group=None, steps: int = 256, ctx: int = 131072) -> dict:
    """Configuration 5: greedy decode of `steps` tokens for a batch of `world` sequences (one a rank) at a 128K
    context, 48 layers cycling Q2_0 / IQ3_S / IQ3_XXS experts, Q8_0 dense projections (through the library's window
    matvec). The MoE block's window is every rank's token (expert parallel: all-gather, all-reduce). Each step --
    every layer, the head, the argmax, the next token and the position -- replays from a CUDA graph. The caches are
    filled with random keys and values (standing in for the prefill of 128K-token random prompts)."""
    from strata_mlx_b200 import decoder as D

    dec = D.SyntheticDecoder(48, ["Q2_0", "IQ3_S", "IQ3_XXS"], dense="Q8_0", device=device, group=group,
                             mode="per_rank", max_pos=ctx + steps + 64, seed=5)
    cache = dec.cache(ctx + steps + 16, seed=rank)
    cache.fill_random(ctx, seed=100 + rank)
    g = torch.Generator(device=device)
    g.manual_seed(55 + rank)
    tok = torch.randint(0, dec.vocab, (1,), generator=g, device=device)
    out = torch.zeros(steps, dtype=torch.int64, device=device)
    step_i = torch.zeros(1, dtype=torch.int64, device=device)

    def step():
        logits = dec.forward(tok, cache)
        nxt = logits.argmax(-1)
        out.index_copy_(0, step_i, nxt)
        tok.copy_(nxt)
        cache.pos.add_(1)
        step_i.add_(1)
        return nxt

    graph, _ = graph_of(step, device)
    # the warm call and the capture moved nothing on the device that the replays depend on except pos and step_i
    cache.pos.fill_(ctx)
    step_i.zero_()
    torch.cuda.synchronize()
    barrier(world)
    s = torch.cuda.current_stream()
    clocks = Clocks(device.index)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        graph.replay()
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = reduce_max(e0.elapsed_time(e1) / steps, world)
    dec.check_errors()
    pk = peaks()
    used = [world * 10] * dec.n_layers  # at most 10 distinct experts a token
    nbytes = decoder_bytes(dec, used, ctx + steps // 2, world)
    res = {"workload": "config5: greedy decode of 256 tokens at a 128K context, batch = one sequence a rank, 48-layer "
                       "synthetic MoE decoder (GQA 16 q / 2 kv heads of 256, paged cache of 16-token pages, Q8_0 "
                       "projections), experts cycling Q2_0 / IQ3_S / IQ3_XXS by layer",
           "tok_per_s": world / (ms * 1e-3), "ms_per_step": ms, "steps": steps, "context": ctx, "batch": world,
           "parallelism": f"ep{world}: experts sharded, the MoE window is every rank's token (NCCL all-gather + "
                          "all-reduce), attention per rank" if world > 1 else "single",
           "roofline": {"bound": "hbm", "bytes_per_step_per_rank": nbytes, "achieved": nbytes / (ms * 1e-3) / 1e9,
                        "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                        "what": "KV cache read (12.9 GB a step) + Q8_0 projections + the rank's share of at most "
                                "10 experts a token + shared expert + router, per step"},
           "first_tokens": out[:8].tolist(),
           "kv_prefill": "random keys and values stand in for the prefill of 128K-token random prompts",
           "graph": True, "clocks": clk}
    del graph, dec, cache
    torch.cuda.empty_cache()
    return res


def paged_result(steps: int = 200, warmup: int = 20, budget_experts: int = 128) -> dict:
    """The paged expert store (strata_mlx_b200/paged.py, strata_mlx/paged.py:105-419): one configuration-2 layer
    of IQ3_S experts (512 x gate/up 2048 -> 512, down 512 -> 2048) written to a GGUF file, served by
    PagedSwitchGLU within a budget of `budget_experts` experts, one token a call with seeded uniform top-10 routes:
    each call waits for its routes on the host, reads the experts the store lacks (the file is in the page cache,
    having just been written) and runs the separate-expert kernels. Beside it, the same layer resident
    (BlockSwitchGLU)."""
    import tempfile

    import gguf
    from gguf import GGMLQuantizationType as Q

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import gguf as G
    from strata_mlx_b200 import paged as P
    from strata_mlx_b200.synthetic import blocks_numpy

    device = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(21)
    kind = "IQ3_S"
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "layer.gguf")
        w = gguf.GGUFWriter(path, "bench")
        for name, (rows, cols) in (("up", (I, H)), ("gate", (I, H)), ("down", (H, I))):
            a = blocks_numpy(kind, E, rows, cols, rng, sigma=EP_SIGMA[kind]).reshape(E, rows, -1)
            w.add_tensor(f"blk.0.ffn_{name}_exps.weight", a, raw_dtype=Q.IQ3_S)
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
        f = G.GGUF(path)
        gate, up, down = (f[f"blk.0.ffn_{n}_exps.weight"] for n in ("gate", "up", "down"))
        size = sum(t.data.nbytes // t.shape[0] for t in (gate, up, down))
        store = P.ExpertStore(budget_experts * size, device=device)
        layer = P.PagedSwitchGLU(0, store, gate, up, down)
        resident = B.BlockSwitchGLU(*(B.BlockSwitchLinear(G.to_device(t, device), t.type, t.shape)
                                      for t in (gate, up, down)))
        xs = torch.randn((steps + warmup, 1, H), device=device).to(torch.bfloat16)
        idx = torch.from_numpy(np.stack([rng.choice(E, K, replace=False) for _ in range(steps + warmup)])
                               .astype(np.int32)).to(device).reshape(steps + warmup, 1, K)

        def run(fn, first, n):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(first, first + n):
                fn(xs[i], idx[i])
            torch.cuda.synchronize()
            return (time.perf_counter() - t0) / n

        run(layer, 0, warmup)
        store.reset_stats()
        paged_s = run(layer, warmup, steps)
        stats = {"hits": store.hits, "misses": store.misses, "bytes_read": store.bytes_read, "read_s": store.read_s}
        run(resident, 0, warmup)
        resident_s = run(resident, warmup, steps)
        del store, layer, resident, f
    torch.cuda.empty_cache()
    return {"api": "strata_mlx_b200.paged.PagedSwitchGLU.__call__ (ExpertStore, budget of "
                   f"{budget_experts} of {E} experts)",
            "workload": "one configuration-2 layer of IQ3_S experts from a GGUF file, one token a call, uniform "
                        "random top-10 routes; the file in the page cache",
            "calls": steps, "ms_per_call": paged_s * 1e3, "calls_per_s": 1.0 / paged_s,
            "hit_rate": stats["hits"] / max(1, stats["hits"] + stats["misses"]),
            "read_bytes_per_call": stats["bytes_read"] / steps,
            "read_gbs": stats["bytes_read"] / max(stats["read_s"], 1e-9) / 1e9,
            "resident_ms_per_call": resident_s * 1e3,
            "note": "each call waits on the host for its routes (as the reference does); reads are file -> pinned "
                    "host memory -> device"}


def stage_bytes(kind: str) -> dict:
    """Algorithmic bytes of each of the three kernels of one layer, one token: every byte a kernel must read or
    write once (routed experts: 10 distinct, one token)."""
    rb_h, rb_i = row_bytes(kind, H), row_bytes(kind, I)
    units = K + 1  # the routed experts and the shared one
    h_bytes = units * (I + 32) * 2
    return {
        "route": E * H * 2 + H * 2 + H * 2 + E * 4,
        "gate_up": K * 2 * I * rb_h + 2 * IS * rb_h + H * 2 + h_bytes,
        "down": K * H * rb_i + H * row_bytes(kind, IS) + h_bytes + H * 2 + K * 8,
    }


def window_stream(layers, device, tokens: int = 8, reps: int = 20) -> dict:
    """The fused decode block over a window of `tokens` tokens (its largest; a decode batch of 8 sequences), the 48
    layers replayed as a CUDA graph: each layer reads every distinct routed expert of the window once (~60-80 of
    512), so a step streams a few GB. Algorithmic bytes: per layer the distinct experts' gate, up and down blocks
    (counted from the routes the layers chose), the shared expert, the router. Shows the decode kernels' rate once
    a layer carries enough bytes; one-token layers are latency-bound."""
    from strata_mlx_b200 import fused as F

    # every layer in one launch of the persistent chain kernel (each layer reads the window: refeed 1)
    g = F.DecodeGraph(layers, tokens=tokens, device=device, capture=True, persistent=True)
    gen = torch.Generator(device=device)
    gen.manual_seed(8)
    xs = torch.randn((reps + 3, tokens, H), generator=gen, device=device).to(torch.bfloat16)
    for i in range(3):
        g.x.copy_(xs[i])
        g.replay()
    torch.cuda.synchronize()
    s = g.stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nbytes = 0.0
    total_us = 0.0
    for i in range(reps):
        with torch.cuda.stream(s):
            g.x.copy_(xs[3 + i])
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        total_us += e0.elapsed_time(e1) * 1e3
        routes = g.persistent.routes(tokens, device)[0]
        for i, l in enumerate(layers):  # the routes this step chose: the distinct experts each layer read
            used = int(torch.unique(routes[i].view(torch.int32)).numel())
            per_expert = 2 * I * row_bytes(l.kind, H) + H * row_bytes(l.kind, I)
            shared = 2 * IS * row_bytes(l.kind, H) + H * row_bytes(l.kind, IS)
            nbytes += used * per_expert + shared + E * H * 2
    us = total_us / reps
    nbytes /= reps
    return {"api": "strata_mlx_b200.fused.DecodeGraph(persistent=True): sc_moe_decode_chain, 48 layers in one "
                   "launch, graph replay", "tokens": tokens,
            "bytes_per_step": nbytes, "us_per_step": us, "gbs": nbytes / (us * 1e-6) / 1e9,
            "tok_per_s": tokens / (us * 1e-6)}


def dense_stream(device, n_layers: int = 24, rows: int = 4096, cols: int = 4096, reps: int = 20) -> dict:
    """The Q6_K dense layer (dense.ScaledLinear, strata_mlx/dense.py:109-167) of a one-token window through
    `n_layers` distinct 4096 x 4096 layers in turn, replayed as a CUDA graph (codes 16 MB a layer: the step reads
    HBM, not L2). Synthetic parts (codes in [-32, 31], scales, d) made on the device. Algorithmic bytes: codes,
    scales and d of every layer, the activations and outputs."""
    from strata_mlx_b200.dense import ScaledLinear

    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    lins = []
    for _ in range(n_layers):
        codes = torch.randint(-32, 32, (rows, cols), generator=gen, device=device, dtype=torch.int8)
        scales = torch.randint(-128, 128, (rows, cols // 16), generator=gen, device=device, dtype=torch.int8)
        d = (torch.randn((rows, cols // 256), generator=gen, device=device) * 1e-3).half()
        lins.append(ScaledLinear(codes, scales, d))
    x = torch.randn((1, cols), generator=gen, device=device).to(torch.bfloat16)
    s = torch.cuda.Stream(device=device)
    with torch.cuda.stream(s):
        for lin in lins:
            lin(x)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()  # the layers replayed as a graph: host launches would set the pace otherwise
    with torch.cuda.graph(graph, stream=s):
        for lin in lins:
            lin(x)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        graph.replay()
        e0.record(s)
        for _ in range(reps):
            graph.replay()
        e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n_layers)
    nbytes = lins[0].nbytes + cols * 2 + rows * 2
    return {"api": "strata_mlx_b200.dense.ScaledLinear.__call__ (Q6_K parts, one token, 24 layers in turn, graph)",
            "rows": rows, "cols": cols, "bytes_per_launch": nbytes, "us_per_launch": us,
            "gbs": nbytes / (us * 1e-6) / 1e9}


def time_stages(layers, graph, device, reps: int, capture: bool) -> dict:
    """Each of the fused path's three kernels alone: one launch per layer on the workspace the last step left,
    48 launches (with their programmatic dependencies) replayed as a graph, timed with CUDA events on its stream."""
    s = torch.cuda.Stream(device=device)
    outs = [torch.empty((1, H), dtype=torch.bfloat16, device=device) for _ in layers]
    result = {}
    for stage, name in enumerate(("route", "gate_up", "down")):
        def launch_all():
            for l, o in zip(layers, outs):
                l.stage(graph.x, o, stage)

        with torch.cuda.stream(s):
            launch_all()
        s.synchronize()
        cg = None
        if capture:
            cg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(cg, stream=s):
                launch_all()
        with torch.cuda.stream(s):
            for _ in range(3):
                cg.replay() if cg else launch_all()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                cg.replay() if cg else launch_all()
            e1.record(s)
        s.synchronize()
        ms = e0.elapsed_time(e1) / (reps * len(layers))
        nbytes = sum(stage_bytes(l.kind)[name] for l in layers) / len(layers)
        result[name] = {"us_per_launch": ms * 1e3, "bytes_per_launch": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}
    return result


def read_traffic(kinds: list) -> float | None:
    """Per-launch DRAM bytes (read + write) of the gate/up kernel from the committed ncu summary
    (profiles/traffic.txt, one line per block type), averaged over the chain's layers; None unless every block
    type of the chain was captured."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    got = {}
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) == 2 and parts[0].startswith("gate_up_") and parts[0].endswith("_bytes_per_launch"):
                got[parts[0][len("gate_up_"):-len("_bytes_per_launch")]] = float(parts[1])
    except OSError:
        return None
    if not all(k in got for k in kinds):
        return None
    return sum(got[k] for k in kinds) / len(kinds)


def cpu_sample(mode: str, seconds: float, all_threads: bool) -> dict:
    """The C oracle on the host cores: one layer of each block type (the same shapes), timed for about
    `seconds`, scaled to the 48-layer step."""
    from oracle import cref
    from strata_mlx_b200.synthetic import layer_numpy

    threads = cref.threads(os.cpu_count() or 1)
    rng = np.random.default_rng(12345)
    kinds = ["Q2_0", "IQ3_S"] if mode == "mixed" else [mode]
    per_layer = {}
    for kind in kinds:
        L = layer_numpy(rng, H, I, E, (kind, kind, kind), shared_inter=IS)
        layer = cref.Layer(L, H, I, E, K, "bfloat16", shared_inter=IS)
        x = rng.standard_normal((1, H)).astype(np.float32)
        layer(x)  # warm
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / len(kinds) or n < 2:
            layer(rng.standard_normal((1, H)).astype(np.float32))
            n += 1
        per_layer[kind] = (time.perf_counter() - t0) / n
    return {"per_layer_s": per_layer, "threads": threads}


def step_seconds(per_layer: dict, n_layers: int, mode: str) -> float:
    return sum(per_layer[kind_of(l, mode)] for l in range(n_layers))


def run_chain(args) -> None:
    """--workload chain: the persistent chain kernel alone (sc_moe_decode_chain over --layers layers at --tokens
    tokens, each layer taking the previous one's output, the window fed again every two layers), for timing and
    profiling it; one JSON line. With --no-graph the launches are eager, as a profiler wants them."""
    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import fused as F

    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    layers = build_layers(args.layers, args.kinds, 0, device)
    chain = F.DecodeChain(layers, EP_REFEED if args.layers % EP_REFEED == 0 else 0)
    x = torch.randn((args.tokens, H), device=device).to(torch.bfloat16)
    for _ in range(args.warmup):
        chain(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        chain(x)
    e1.record()
    torch.cuda.synchronize()
    chain.check_errors()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"workload": "the persistent chain kernel alone", "layers": args.layers, "tokens": args.tokens,
                      "ms_per_launch": ms, "us_per_layer": ms * 1000 / args.layers,
                      "tok_per_s": args.tokens / (ms * 1e-3)}), flush=True)


def run_reference(args, world, rank) -> None:
    """--impl reference: the C oracle (the reference's block decode and MoE block restated in C) on all host
    cores, rank 0 only; each step a bounded sample of the 48-layer chain."""
    if rank != 0:
        return
    from oracle import cref
    from strata_mlx_b200.synthetic import layer_numpy

    threads = cref.threads(os.cpu_count() or 1)
    rng = np.random.default_rng(777)
    kinds = ["Q2_0", "IQ3_S"] if args.kinds == "mixed" else [args.kinds]
    host = {k: cref.Layer(layer_numpy(rng, H, I, E, (k, k, k), shared_inter=IS), H, I, E, K, "bfloat16", shared_inter=IS)
            for k in kinds}
    # one probe layer of each kind sizes the sample: (steps + warmup) samples within about two minutes
    probe = {}
    for k in kinds:
        host[k](rng.standard_normal((1, H)).astype(np.float32))
        t0 = time.perf_counter()
        host[k](rng.standard_normal((1, H)).astype(np.float32))
        probe[k] = time.perf_counter() - t0
    full = step_seconds(probe, args.layers, args.kinds)
    budget = 120.0 / max(1, args.steps + args.warmup)
    sample_layers = max(len(kinds), min(args.layers, int(args.layers * budget / max(full, 1e-9))))
    sample_layers -= sample_layers % len(kinds)

    def step():
        t0 = time.perf_counter()
        for l in range(sample_layers):
            host[kind_of(l, args.kinds)](rng.standard_normal((1, H)).astype(np.float32))
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step()
    total = sum(step() for _ in range(args.steps))
    ms = total / args.steps * args.layers / sample_layers * 1000.0
    value = 1000.0 / ms
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": workload_config(args, world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{sample_layers} of {args.layers} layers per step, one token, scaled to the chain"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args, world) -> dict:
    return {"workload": "config2: one MoE layer decode, batch 1 per rank (hidden 2048, 512 experts x SwiGLU inter 512, "
                        "top-10 softmax router, shared expert inter 512), experts "
                        + ("Q2_0 / IQ3_S alternating" if args.kinds == "mixed" else args.kinds)
                        + f", chained over {args.layers} distinct layers (a layer takes the previous one's output; "
                        f"the step's token is fed again every {EP_REFEED} layers)",
            "layers": args.layers, "tokens_per_rank_per_step": 1, "hidden": H, "experts": E, "inter": I, "top_k": K,
            "shared_inter": IS, "global_batch": world, "parallelism": "replicas" if world > 1 else "single",
            "l2": "inputs larger than L2: ~0.6 GB of distinct routed-expert blocks per step, a fresh token each step"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--kinds", default="mixed", choices=["mixed", "Q2_0", "IQ3_S"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "chain", "mid", "dense"],
                    help="decode: configuration 2, the headline line; prefill: configuration 3 (one GPU); chain: the "
                         "persistent chain kernel alone (one GPU, for profiling); mid: the mid_batch sub-line alone "
                         "(--steps replays, min(--layers, 3) layers a block type); dense: the Q6_K dense_stream "
                         "sub-line alone (--layers layers, --steps replays)")
    ap.add_argument("--tokens", type=int, default=1, help="--workload chain: the window's tokens")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config5-steps", type=int, default=256, help="greedy decode steps of the configuration-5 line")
    ap.add_argument("--no-extra", action="store_true",
                    help="leave out the configuration-1 and configuration-3 sub-lines of the one-GPU decode line")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the layers one by one instead of replaying a CUDA graph (for profilers that cannot "
                         "follow a stream capture); the same kernels run")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    if args.workload == "dense":  # one GPU: the Q6_K layers alone, for timing and profiling them
        from strata_mlx_b200 import _lib

        _lib.load()
        device = torch.device("cuda", torch.cuda.current_device())
        ds = dense_stream(device, n_layers=args.layers, reps=args.steps)
        ds["frac"] = ds["gbs"] / peaks()["hbm_gbs"]
        print(json.dumps({"workload": "dense", **ds}), flush=True)
        return
    if args.workload == "mid":
        if rank == 0:
            from strata_mlx_b200 import _lib

            _lib.load()
            print(json.dumps({"workload": "mid", **mid_batch_result(reps=args.steps, layers=min(args.layers, MB_LAYERS))}),
                  flush=True)
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()
        return
    if args.workload == "chain":
        if rank == 0:
            run_chain(args)
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()
        return
    if args.workload == "prefill":
        if rank == 0:
            run_prefill(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            barrier(world)
            dist.destroy_process_group()
        return
    if world > 1:
        run_ep(args, world, rank, local)
        return

    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import fused as F

    _lib.load()
    device = torch.device("cuda", torch.cuda.current_device())
    layers = build_layers(args.layers, args.kinds, rank, device)
    refeed = EP_REFEED if args.layers % EP_REFEED == 0 else 0
    graph = F.DecodeGraph(layers, tokens=1, device=device, capture=not args.no_graph, chain=True, refeed=refeed)
    gen = torch.Generator(device=device)
    gen.manual_seed(99 + rank)
    n_tok = args.steps + args.warmup
    xs = torch.randn((n_tok, H), generator=gen, device=device).to(torch.bfloat16)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()

    # ---- value: the chain replayed from HBM-resident tokens
    for i in range(args.warmup):
        graph.x.copy_(xs[i : i + 1])
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(args.steps):
        graph.x.copy_(xs[args.warmup + i : args.warmup + i + 1])
        graph.replay()
    e1.record(s)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = reduce_max(e0.elapsed_time(e1) / args.steps, world)
    barrier(world)
    _lib.check_device_errors(device)

    # ---- e2e: the public call, pinned host token in, host result out, every step
    host_x = xs.cpu().pin_memory()
    for i in range(args.warmup):
        graph(host_x[i])
    barrier(world)
    e2e_steps = min(args.steps, 500)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        graph(host_x[(args.warmup + i) % n_tok])
    e2e_ms = reduce_max((time.perf_counter() - t0) / e2e_steps * 1000.0, world)

    # ---- the three kernels alone; the dominant one (gate/up: two thirds of the expert bytes) is the roofline's
    st = time_stages(layers, graph, device, reps=20 if args.no_graph else 50, capture=not args.no_graph)
    gu = st["gate_up"]
    pk = peaks()
    achieved = gu["gbs"]
    traffic = read_traffic([l.kind for l in layers])

    finite = bool(torch.isfinite(graph.outs[-1].float()).all().item())
    cfg = workload_config(args, world)
    cfg.update(refeed=refeed, expert_sigma=EP_SIGMA, outputs_finite=finite)
    line = {"metric": METRIC, "value": world * 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded GGUF blocks and float16 router made in HBM",
            "config": cfg,
            "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2,
                    "api": "strata_mlx_b200.fused.DecodeGraph.__call__"},
            "roofline": {"bound": "hbm", "kernel": "gate_up_kernel (routed + shared experts' gate/up/swiglu)",
                         "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": pk["source"], "traffic": traffic,
                         "bytes_per_launch": gu["bytes_per_launch"], "us_per_launch": gu["us_per_launch"]},
            "kernels": st,
            "expert_bytes_per_step": sum(stage_bytes(l.kind)["gate_up"] + stage_bytes(l.kind)["down"] for l in layers),
            "expert_matvec_gbs": achieved, "expert_matvec_frac_of_8tbs": achieved / 8000.0,
            "gpu_launches": 3 * args.layers * args.steps, "gpu_launches_per_step": 3 * args.layers, "clocks": clk}
    line["chain_gbs"] = (line["expert_bytes_per_step"] + sum(stage_bytes(l.kind)["route"] for l in layers)) / (ms * 1e-3) / 1e9
    if world == 1:
        st = window_stream(layers, device)
        st["frac"] = st["gbs"] / pk["hbm_gbs"]
        st["peak"] = pk["hbm_gbs"]
        line["window8_stream"] = st
        ds = dense_stream(device)
        ds["frac"] = ds["gbs"] / pk["hbm_gbs"]
        ds["peak"] = pk["hbm_gbs"]
        line["dense_stream"] = ds
    if world == 1 and not args.no_extra:
        del graph
        torch.cuda.synchronize()
        line["config1"] = config1_result(cpu_seconds=None if args.no_cpu_baseline else 5.0)
        line["mid_batch"] = mid_batch_result()
        line["paged"] = paged_result()
        line["prefill"] = prefill_result(20, 5, None if args.no_cpu_baseline else 6.0)
        line["config4"] = config4_result(world, rank, device)
        line["config5"] = config5_result(world, rank, device, steps=args.config5_steps)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cb = cpu_sample(args.kinds, 12.0, True)
        cpu_ms = step_seconds(cb["per_layer_s"], args.layers, args.kinds) * 1000.0
        line["cpu_baseline"] = {"value": 1000.0 / cpu_ms, "unit": "tok/s", "cores": cb["threads"], "kind": "port",
                                "sample": "one layer of each block type timed for ~12 s, scaled to the 48-layer step"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
