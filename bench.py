"""Benchmark of the NVFP4 MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2|reference]
                    [--workload decode|prefill|ep_prefill|qmm] [--qmm-m M] [--blocks B]
                    [--no-cpu-baseline]

Default workload: the B=1 MoE decode block --
hidden 2048, 128 NVFP4 experts, top-8 softmax router (fp32 router weight),
SwiGLU experts with ffn 768.  One step = one token through one block (one
launch of the fused decode kernel).  The timed region replays a CUDA graph of
a 16-block chain (block l+1 consumes block l's output, like a layer stack)
whose distinct weights (5.4 GB of MLX-layout banks) exceed the 126 MB L2, so
every step streams its experts from HBM.  With N GPUs each rank runs its own
replica (the decode path does not shard); `value` is the sum.

--workload prefill: the 2048-token MoE prefill
block on the tensor-core grouped GEMMs; one step = one block forward over
2048 tokens (router, top-k, expert sort, gate/up + SwiGLU GEMM, down GEMM,
ordered combine); roofline against the measured dense bf16 tensor peak.

--workload qmm: one NVFP4 quantized_matmul,
x bf16 [M, 4096] (M = 1, or 32 with --qmm-m 32) times a 4096 x 4096 NVFP4
weight (transpose=True); one step = one call.  The graph chains 24 distinct
weights (226 MB, beyond L2); roofline against the measured copy bandwidth.

Prints ONE JSON line on rank 0 (see the keys in `report`).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mlxfast-challenge_senpai_b200")
sys.path.insert(0, PKG)

H, E, F, TOPK = 2048, 128, 768, 8
DECODE_BYTES = (E * H * 4) + TOPK * (2 * F) * (H // 2 + H // 16) + TOPK * H * (F // 2 + F // 16) + 2 * H * 2
GATEUP_BYTES = TOPK * (2 * F) * (H // 2 + H // 16)
N_BLOCKS = 16
PREFILL_T = 2048
# 2 * rows * (gate/up + down) multiply-adds of the expert GEMMs (config 3)
PREFILL_FLOP = 2 * PREFILL_T * TOPK * (H * 2 * F + F * H)
# DRAM bytes (read + write) of one decode-kernel launch from the committed
# ncu summary profiles/decode_block_tma_config2.txt; None when not captured
DECODE_TRAFFIC_BYTES = 22_420_000
# same for the prefill's dominant kernel (gate/up grouped GEMM, read 293.7 MB +
# write 20.7 MB) from profiles/prefill_block_config3.txt
PREFILL_GEMM_TRAFFIC_BYTES = 314_410_000
# MLX-layout expert bank of one block (codes + scales of gate, up, down)
BLOCK_BANK_MB = E * (3 * F * H) * (1 / 2 + 1 / 16) / 1e6
METRIC = "NVFP4 MoE decode tok/s + HBM GB/s %peak; prefill tok/s at 1/2/4/8 B200"
# one quantized_matmul, 4096 x 4096 NVFP4 weight; 24 distinct
# weights chained per graph replay (226 MB, beyond L2)
QMM_N = QMM_K = 4096
QMM_WEIGHTS = 24
QMM_WEIGHT_BYTES = QMM_N * (QMM_K // 2 + QMM_K // 16)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- setup
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def make_decode_blocks(dev, n_blocks, seed=0):
    import torch

    import b2moe

    gen = torch.Generator(device=dev).manual_seed(seed)
    blocks = []
    for b in range(n_blocks):
        t = {}
        for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
            w = torch.randn(shp, generator=gen, device=dev, dtype=torch.float32) * 0.02
            t[nm + "_codes"], t[nm + "_scales"] = b2moe.quantize(w)
            del w
        wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
        blocks.append(b2moe.MoEBlock(b2moe.ExpertBank(**t), wr, top_k=TOPK, prepare_decode=True))
    torch.cuda.synchronize()
    return blocks


# --------------------------------------------------------------------------- timing helpers
def time_graph(graph, reps, stream, world):
    import torch

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end)


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- decode workload
def bench_decode(args, world, rank, local):
    import torch

    dev = torch.device("cuda", local)
    nblk = args.blocks
    blocks = make_decode_blocks(dev, nblk, seed=1234 + rank)
    x0 = torch.randn(1, H, device=dev, dtype=torch.float32).to(torch.bfloat16)
    bufs = [x0] + [torch.empty(1, H, device=dev, dtype=torch.bfloat16) for _ in range(nblk)]
    for b in blocks:
        b._workspace(1, dev)  # allocate before capture

    def chain():
        for i, b in enumerate(blocks):
            b(bufs[i], out=bufs[i + 1])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            chain()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    reps_w = max(1, -(-args.warmup // nblk))
    reps = max(1, -(-args.steps // nblk))
    steps = reps * nblk
    with torch.cuda.stream(stream):
        for _ in range(reps_w):
            g.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = time_graph(g, reps, stream, world)
    ms = max_over_ranks(ms, world)
    per_step_ms = ms / steps

    # the block is one launch of the fused decode kernel: per-launch time =
    # graph time / steps (launch gaps included), algorithmic bytes = router +
    # the 8 experts' gate/up and down tiles + x and y
    hbm, _, peak_kind = peaks()
    achieved_gbs = DECODE_BYTES / (per_step_ms * 1e-3) / 1e9

    # end to end through the public API with host buffers
    e2e = bench_decode_e2e(blocks, dev, args, world)

    value = world * 1e3 / per_step_ms
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": reps_w * nblk, "ms_per_step": round(per_step_ms, 6), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 weights (e2m1+e4m3), bf16 activations, f32 accum",
        "data": "synthetic: N(0,0.02) weights quantized to nvfp4 on device, N(0,1) bf16 tokens, seeded",
        "config": {"workload": "moe_decode_block (BASELINE configs[1])", "hidden": H, "experts": E, "top_k": TOPK,
                   "ffn": F, "router": "softmax top-8 renormalised, fp32 router weight", "tokens_per_step": 1,
                   "blocks_rotated": nblk,
                   "l2": f"inputs larger than L2 ({nblk} distinct blocks, {nblk * BLOCK_BANK_MB:.0f} MB of expert weights)",
                   "parallelism": f"replicas x{world}"},
        "hbm_gbs": round(achieved_gbs, 1), "hbm_frac_of_peak": round(achieved_gbs / hbm, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved_gbs / hbm, 4), "traffic": DECODE_TRAFFIC_BYTES,
                     "kernel": "decode_block_tma_kernel (fused router, top-k, gate/up+SwiGLU, down, combine)",
                     "algorithmic_bytes_per_launch": DECODE_BYTES, "peak_source": peak_kind + " (of measured copy bw)"},
        "e2e": e2e,
        "gpu_launches": steps,
        "clocks": clk.summary(),
    }
    return out


def bench_decode_e2e(blocks, dev, args, world):
    import torch

    xh = torch.randn(1, H).to(torch.bfloat16).pin_memory()
    yh = torch.empty(1, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    nblk = len(blocks)
    steps = max(nblk, (args.steps // nblk) * nblk)
    for i in range(nblk):
        xd.copy_(xh, non_blocking=True)
        y = blocks[i](xd)
        yh.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    start.record(stream)
    for i in range(steps):
        xd.copy_(xh, non_blocking=True)
        y = blocks[i % nblk](xd)
        yh.copy_(y, non_blocking=True)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    return {"value": round(world * steps / (ms * 1e-3), 2), "unit": "tok/s", "h2d_bytes_per_step": H * 2,
            "d2h_bytes_per_step": H * 2}


# --------------------------------------------------------------------------- prefill workload
def make_prefill_block(dev, seed=0):
    import torch

    import b2moe

    gen = torch.Generator(device=dev).manual_seed(seed)
    t = {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        w = torch.randn(shp, generator=gen, device=dev, dtype=torch.float32) * 0.02
        t[nm + "_codes"], t[nm + "_scales"] = b2moe.quantize(w)
        del w
    # N(0, 0.02) router rows over N(0, 1) tokens: near-uniform expert load
    wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
    blk = b2moe.MoEBlock(b2moe.ExpertBank(**t), wr, top_k=TOPK, prepare_prefill=True)
    torch.cuda.synchronize()
    return blk, gen


def bench_prefill(args, world, rank, local):
    import torch

    dev = torch.device("cuda", local)
    blk, gen = make_prefill_block(dev, seed=4321 + rank)
    x = torch.randn(PREFILL_T, H, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty_like(x)
    blk._workspace(PREFILL_T, dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            blk(x, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        blk(x, out=out)
    steps, warm = args.steps, args.warmup
    with torch.cuda.stream(stream):
        for _ in range(warm):
            g.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = time_graph(g, steps, stream, world)
    ms = max_over_ranks(ms, world)
    per_step_ms = ms / steps
    _, tflops_peak, peak_kind = peaks()
    achieved = PREFILL_FLOP / (per_step_ms * 1e-3) / 1e12
    # end to end through the public API: x from pinned host memory, output back
    xh = x.cpu().pin_memory()
    yh = torch.empty(PREFILL_T, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x)
    cur = torch.cuda.current_stream(dev)
    for _ in range(2):
        xd.copy_(xh, non_blocking=True)
        blk(xd, out=out)
        yh.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, steps // 4)
    barrier(world)
    e0.record(cur)
    for _ in range(n_e2e):
        xd.copy_(xh, non_blocking=True)
        blk(xd, out=out)
        yh.copy_(out, non_blocking=True)
    e1.record(cur)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), world)
    value = world * PREFILL_T * 1e3 / per_step_ms
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": round(per_step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "nvfp4 weights dequantized exactly to bf16 in TMEM (tcgen05 A operand), "
                                    "bf16 activations, f32 accumulate",
        "data": "synthetic: N(0,0.02) weights quantized to nvfp4 on device, N(0,1) bf16 tokens, seeded",
        "config": {"workload": "moe_prefill_block (BASELINE configs[2])", "tokens": PREFILL_T, "hidden": H,
                   "experts": E, "top_k": TOPK, "ffn": F, "router": "softmax top-8, near-uniform load",
                   "l2": "inputs larger than L2 (340 MB expert bank per step)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tflops_peak, 4), "traffic": PREFILL_GEMM_TRAFFIC_BYTES,
                     "kernel": "whole prefill block step (expert GEMM flops / step time); traffic of the "
                               "gate/up grouped GEMM launch",
                     "algorithmic_flop_per_step": PREFILL_FLOP, "peak_source": peak_kind + " (of measured bf16 "
                                                                                            "cuBLAS burst)"},
        "e2e": {"value": round(world * n_e2e * PREFILL_T / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": PREFILL_T * H * 2, "d2h_bytes_per_step": PREFILL_T * H * 2},
        # router logits, top-k, sort histogram + scatter, token tiles, row
        # gather, gate/up GEMM, down GEMM, combine
        "gpu_launches": 9 * steps,
        "clocks": clk.summary(),
    }


# --------------------------------------------------------------------------- single qmm workload
def cpu_qmm_sample(M, threads, target_s=10.0, seed=11):
    """MLX's own fp_qmm_t (oracle/_ref; the restatement when that was not
    built) on the host cores for the configs[0] shape: independent calls on
    `threads` threads over a bounded sample.  Returns (rows/s, kind, threads,
    seconds, calls)."""
    import concurrent.futures as cf

    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    O.build()
    kind = "reference" if O.ref_available() else "port"
    qmm = O.ref_qmm_bf16 if kind == "reference" else O.qmm_bf16
    rng = np.random.default_rng(seed)
    w, sc = O.fp_quantize((rng.standard_normal((QMM_N, QMM_K), dtype=np.float32) * np.float32(0.02)))
    x = O.f32_to_bf16(rng.standard_normal((M, QMM_K), dtype=np.float32))
    t0 = time.perf_counter()
    qmm(x, w, sc)
    one = max(time.perf_counter() - t0, 1e-4)
    n = max(threads, int(target_s * threads / one) // threads * threads)
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda _: qmm(x, w, sc), range(n)))
    dt = time.perf_counter() - t0
    return n * M / dt, kind, threads, dt, n


def bench_qmm(args, world, rank, local):
    import torch

    import b2moe

    dev = torch.device("cuda", local)
    M = args.qmm_m
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    ws = []
    for _ in range(QMM_WEIGHTS):
        w = torch.randn(QMM_N, QMM_K, generator=gen, device=dev, dtype=torch.float32) * 0.02
        ws.append(b2moe.quantize(w))
        del w
    x0 = torch.randn(M, QMM_K, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    bufs = [x0] + [torch.empty(M, QMM_N, device=dev, dtype=torch.bfloat16) for _ in range(QMM_WEIGHTS)]

    def chain():
        for i, (c, sc) in enumerate(ws):
            y = b2moe.quantized_matmul(bufs[i], c, sc)
            bufs[i + 1] = y

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            chain()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    reps_w = max(1, -(-args.warmup // QMM_WEIGHTS))
    reps = max(1, -(-args.steps // QMM_WEIGHTS))
    steps = reps * QMM_WEIGHTS
    with torch.cuda.stream(stream):
        for _ in range(reps_w):
            g.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = time_graph(g, reps, stream, world)
    ms = max_over_ranks(ms, world)
    per_step_ms = ms / steps
    hbm, _, peak_kind = peaks()
    algo = QMM_WEIGHT_BYTES + 2 * M * QMM_K * 2
    achieved = algo / (per_step_ms * 1e-3) / 1e9

    # end to end: x from pinned host memory, y back, through the public call
    xh = x0.cpu().pin_memory()
    yh = torch.empty(M, QMM_N, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x0)
    cur = torch.cuda.current_stream(dev)
    for i in range(QMM_WEIGHTS):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(b2moe.quantized_matmul(xd, *ws[i]), non_blocking=True)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    e0.record(cur)
    for i in range(steps):
        xd.copy_(xh, non_blocking=True)
        yh.copy_(b2moe.quantized_matmul(xd, *ws[i % QMM_WEIGHTS]), non_blocking=True)
    e1.record(cur)
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), world)
    kern = "qmv_mma_kernel (tensor-core GEMV, bf16 x, M <= 32)"
    return {
        "metric": METRIC, "value": round(world * M * 1e3 / per_step_ms, 2), "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": reps_w * QMM_WEIGHTS, "ms_per_step": round(per_step_ms, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "nvfp4 weights (e2m1+e4m3), bf16 activations, f32 accum",
        "data": "synthetic: N(0,0.02) weights quantized to nvfp4 on device, N(0,1) bf16 x, seeded",
        "config": {"workload": f"quantized_matmul nvfp4 (BASELINE configs[0]), M={M}", "M": M, "N": QMM_N,
                   "K": QMM_K, "weights_rotated": QMM_WEIGHTS,
                   "l2": f"inputs larger than L2 ({QMM_WEIGHTS} distinct weights, "
                         f"{QMM_WEIGHTS * QMM_WEIGHT_BYTES / 1e6:.0f} MB)",
                   "parallelism": f"replicas x{world}"},
        "hbm_gbs": round(achieved, 1), "hbm_frac_of_peak": round(achieved / hbm, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None, "kernel": kern,
                     "algorithmic_bytes_per_launch": algo, "peak_source": peak_kind + " (of measured copy bw)"},
        "e2e": {"value": round(world * steps * M / (ms_e2e * 1e-3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": M * QMM_K * 2, "d2h_bytes_per_step": M * QMM_N * 2},
        "gpu_launches": steps,
        "clocks": clk.summary(),
    }


# --------------------------------------------------------------------------- EP prefill workload
EP_TOKENS = 8192
NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per GPU on this pool


def bench_ep_prefill(args, world, rank, local):
    """8192 tokens over `world` ranks (strong scaling), 128
    experts sharded E/world per rank, top-8, Zipf(1.1)-skewed routing logits;
    all_to_all dispatch and return over NCCL around the grouped GEMMs."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import b2moe
    import ep

    dev = torch.device("cuda", local)
    if not dist.is_initialized():
        import socket

        with socket.socket() as so:
            so.bind(("127.0.0.1", 0))
            port = so.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
    gen = torch.Generator(device=dev).manual_seed(777)  # same weights on every rank
    t = {}
    for nm, shp in (("gate", (E, F, H)), ("up", (E, F, H)), ("down", (E, H, F))):
        w = torch.randn(shp, generator=gen, device=dev, dtype=torch.float32) * 0.02
        t[nm + "_codes"], t[nm + "_scales"] = b2moe.quantize(w)
        del w
    wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
    blk = ep.make_gpu_block(b2moe.ExpertBank(**t), wr, TOPK)
    del t
    T_l = EP_TOKENS // world
    gx = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(T_l, H, generator=gx, device=dev, dtype=torch.float32).to(torch.bfloat16)
    # Zipf(1.1) expert popularity over a seeded rank -> expert permutation,
    # added to the router logits as log-popularity (computed once: an input)
    rs = np.random.default_rng(5)
    perm = rs.permutation(E)
    pop = np.empty(E, np.float32)
    pop[perm] = (1.0 / np.arange(1, E + 1) ** 1.1).astype(np.float32)
    bias = torch.from_numpy(np.log(pop)).to(dev)
    logits = b2moe.router_logits(x, wr) + bias
    for _ in range(max(2, args.warmup)):
        out, inds, _, (ss, rsz) = blk(x, logits=logits, return_routing=True)
    torch.cuda.synchronize()
    steps = args.steps
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(steps):
            blk(x, logits=logits)
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    # lower bound of this configuration: the busiest rank's expert flops at the
    # bf16 peak vs its exchanged bytes (dispatch + return) at the NVLink rate
    _, tflops_peak, peak_kind = peaks()
    rows_recv = float(sum(rsz))
    flop_rank = 2.0 * rows_recv * (H * 2 * F + F * H)
    # rows leaving this GPU: dispatched to peers plus expert outputs returned
    # to peers (rows a rank keeps do not cross NVLink); the same enter it
    remote_rows = (sum(ss) - ss[rank]) + (sum(rsz) - rsz[rank])
    bytes_rank = float(remote_rows) * H * 2
    lb_ms = max(flop_rank / (tflops_peak * 1e12), bytes_rank / (NVLINK_GBS * 1e9)) * 1e3
    lb_ms = max_over_ranks(lb_ms, world)
    total_flop = 2.0 * EP_TOKENS * TOPK * (H * 2 * F + F * H)
    value = EP_TOKENS * 1e3 / ms
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": max(2, args.warmup), "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "nvfp4 weights dequantized exactly to bf16 in TMEM (tcgen05 A operand), "
                                    "bf16 activations, f32 accumulate",
        "data": "synthetic: N(0,0.02) weights quantized on device, N(0,1) bf16 tokens, Zipf(1.1) expert popularity",
        "config": {"workload": "ep_moe_prefill (BASELINE configs[4])", "tokens": EP_TOKENS, "tokens_per_rank": T_l,
                   "hidden": H, "experts": E, "experts_per_rank": E // world, "top_k": TOPK, "ffn": F,
                   "parallelism": f"ep{world}", "exchange": "NCCL all_to_all_single (dispatch + return)"},
        "roofline": {"bound": "max(tensor, nvlink) of the busiest rank", "achieved": round(lb_ms / ms, 4),
                     "peak": 1.0, "unit": "fraction of the lower-bound time", "frac": round(lb_ms / ms, 4),
                     "traffic": None, "lower_bound_ms": round(lb_ms, 4),
                     "expert_tflops_per_gpu": round(total_flop / (ms * 1e-3) / 1e12 / world, 1),
                     "peak_source": peak_kind + f" bf16 {tflops_peak} TFLOP/s, NVLink {NVLINK_GBS} GB/s"},
        "gpu_launches": None,
        "clocks": clk.summary(),
    }


# --------------------------------------------------------------------------- CPU baseline
def cpu_decode_sample(n_tokens, threads, seed=7):
    """The reference's CPU path for the decode block on a bounded sample of
    tokens: MLX's own fp_qmm_t (bf16 activations, the stock path) from
    oracle/_ref when present, else the restatement; router, SwiGLU and combine
    from the restatement.  Returns (tokens/s, kind, threads)."""
    import concurrent.futures as cf

    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    O.build()
    kind = "reference" if O.ref_available() else "port"
    rng = np.random.default_rng(seed)

    def q(shape):
        w = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        return O.fp_quantize(w)

    # only the experts a token routes to are touched; build a bank of 16
    # experts and route within it (same shapes and arithmetic per expert)
    Es = 16
    gw, gs = q((Es, F, H))
    uw, us = q((Es, F, H))
    dw, ds = q((Es, H, F))
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    qmm = O.ref_qmm_bf16 if kind == "reference" else O.qmm_bf16
    xs = [O.f32_to_bf16(rng.standard_normal((1, H), dtype=np.float32)) for _ in range(n_tokens)]

    def one(x):
        logits = O.router_logits(x, wr)
        inds, wts = O.topk_softmax(logits, TOPK)
        d = np.zeros((1, TOPK, H), np.uint16)
        for s in range(TOPK):
            e = int(inds[0, s]) % Es
            g = qmm(x, gw[e], gs[e])
            u = qmm(x, uw[e], us[e])
            a = O.swiglu_bf16(g, u)
            d[0, s] = qmm(a, dw[e], ds[e])[0]
        return O.combine_bf16(d, wts)

    one(xs[0])
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, xs))
    dt = time.perf_counter() - t0
    return n_tokens / dt, kind, threads, dt


def cpu_baseline(threads, target_s=15.0):
    """The CPU path timed on a bounded sample sized to about target_s seconds
    (a calibration run of one token per thread picks the sample size)."""
    _, _, _, dt0 = cpu_decode_sample(threads, threads)
    per_token = max(dt0 / threads, 1e-4)
    n = max(threads, int(target_s / per_token) // threads * threads)
    v, kind, thr, dt = cpu_decode_sample(n, threads)
    return v, kind, thr, dt, n


def run_reference_arm(args, world, rank):
    """The reference's CPU path (MLX's own fp_qmm_t from oracle/_ref when it
    was built here, else the restatement) on the host cores.  The CPU path
    runs the same per-token expert GEMVs for decode and prefill (MLX's CPU
    gather_qmm is a loop over (token, slot) pairs), so both workloads report
    tokens/s of that loop."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    if args.workload == "qmm":
        v, kind, thr, dt, n = cpu_qmm_sample(args.qmm_m, threads)
        return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
                "steps": n, "warmup": 1, "ms_per_step": round(1e3 * args.qmm_m / v, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 weights, bf16 activations (MLX CPU path)",
                "data": "synthetic seeded",
                "config": {"workload": f"quantized_matmul nvfp4 (BASELINE configs[0]), M={args.qmm_m}",
                           "M": args.qmm_m, "N": QMM_N, "K": QMM_K},
                "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": thr, "kind": kind,
                                 "sample": f"{n} calls of M={args.qmm_m} on {thr} host threads, {dt:.1f} s"},
                "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    v, kind, thr, dt, n = cpu_baseline(threads)
    wl = "moe_prefill_block (BASELINE configs[2])" if args.workload == "prefill" else \
        "moe_decode_block (BASELINE configs[1])"
    return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
            "steps": n, "warmup": 1, "ms_per_step": round(1e3 / v, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4 weights, bf16 activations (MLX CPU path)",
            "data": "synthetic seeded", "config": {"workload": wl, "hidden": H, "experts": E, "top_k": TOPK,
                                                     "ffn": F},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": thr, "kind": kind,
                             "sample": f"{n} tokens through one block on {thr} host threads, {dt:.1f} s"},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--impl", default="b2", choices=["b2", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "ep_prefill", "qmm"])
    ap.add_argument("--qmm-m", type=int, default=1, choices=[1, 32], help="rows of x for --workload qmm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--blocks", type=int, default=N_BLOCKS,
                    help="distinct blocks chained per graph replay (default 16: weights exceed L2)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        r = run_reference_arm(args, world, rank)
        if r is not None:
            print(json.dumps(r), flush=True)
        return

    world, rank, local = dist_setup(args)
    if args.workload == "prefill":
        res = bench_prefill(args, world, rank, local)
    elif args.workload == "ep_prefill":
        res = bench_ep_prefill(args, world, rank, local)
    elif args.workload == "qmm":
        res = bench_qmm(args, world, rank, local)
    else:
        res = bench_decode(args, world, rank, local)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline and args.workload == "qmm":
            threads = os.cpu_count() or 1
            v, kind, thr, dt, n = cpu_qmm_sample(args.qmm_m, threads)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": thr, "kind": kind,
                                   "sample": f"{n} calls of M={args.qmm_m} on {thr} host threads ({dt:.1f} s)"}
        elif world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            v, kind, thr, dt, n = cpu_baseline(threads)
            res["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": thr, "kind": kind,
                                   "sample": f"{n} tokens through one block on {thr} host threads ({dt:.1f} s); "
                                             "the CPU path does the same per-token work for decode and prefill"}
        print(json.dumps(res), flush=True)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
