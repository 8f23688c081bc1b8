"""Benchmark of the NVFP4 MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2|reference]
                    [--workload all|ep_prefill|decode|prefill|qmm|decode_step] [--qmm-m M]
                    [--blocks B]
                    [--no-cpu-baseline] [--ep-impl peer|nccl]

Default (`--workload all`): the headline line is BASELINE.json configs[4],
the expert-parallel MoE prefill block: 8192 tokens split over the N ranks
(strong scaling), hidden 2048, 128 NVFP4 experts (E/N per rank), top-8
softmax router over Zipf(1.1)-skewed logits, SwiGLU experts with ffn 768.
One step = one block forward over all 8192 tokens (router logits, top-k,
dispatch, grouped GEMMs, return, ordered combine) on every rank; `value` =
8192 tokens / the step time (max over ranks).  The path is
b2_moe_ep_prefill: NVLink peer loads and stores into CUDA-IPC-mapped
buffers, flag barriers in peer memory, no host round trip.  At N = 1 the
line also carries `configs`: one record per single-GPU configuration, each
with its own roofline, e2e and CPU baseline --
  qmm_m1 / qmm_m32  configs[0]: one quantized_matmul, x bf16 [M, 4096] times
                    a 4096 x 4096 NVFP4 weight; 24 distinct weights rotated
                    (226 MB, beyond L2);
  decode            configs[1]: the B=1 MoE decode block (one token, one
                    launch of the fused decode kernel); 16 distinct blocks
                    chained like a layer stack (5.4 GB, beyond L2);
  prefill           configs[2]: the 2048-token prefill block on the
                    tensor-core grouped GEMMs (340 MB bank per step);
  decode_step       configs[3]: one token through a 4-layer stack (attention
                    over a 4096-long bf16 KV cache + the MoE block per
                    layer), two stacks alternating (330 MB, beyond L2).
`--workload X` runs one of them alone as the line.

Every timed region is exactly K steps, after W untimed warm-up steps,
bracketed by a barrier and a device synchronize, timed with CUDA events on
the launching stream, max over ranks.  nvidia-smi clocks are sampled while
it runs.
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
N_BLOCKS = 16
PREFILL_T = 2048
EXPERT_FLOP_PER_ROW = 2 * (H * 2 * F + F * H)
# 2 * rows * (gate/up + down) multiply-adds of the expert GEMMs (config 3)
PREFILL_FLOP = PREFILL_T * TOPK * EXPERT_FLOP_PER_ROW
# DRAM bytes (read + write) of one launch of each workload's dominant kernel,
# from the committed ncu summaries under profiles/
DECODE_TRAFFIC_BYTES = 22_420_000      # decode_block_tma_config2.txt
PREFILL_GEMM_TRAFFIC_BYTES = 314_410_000  # prefill_block_config3.txt (gate/up GEMM)
QMM_M1_TRAFFIC_BYTES = 9_470_000       # qmv_mma_config1.txt
# MLX-layout expert bank of one block (codes + scales of gate, up, down)
BLOCK_BANK_MB = E * (3 * F * H) * (1 / 2 + 1 / 16) / 1e6
METRIC = "NVFP4 MoE decode tok/s + HBM GB/s %peak; prefill tok/s at 1/2/4/8 B200"
QMM_N = QMM_K = 4096
QMM_WEIGHTS = 24
QMM_WEIGHT_BYTES = QMM_N * (QMM_K // 2 + QMM_K // 16)
EP_TOKENS = 8192
ZIPF_S = 1.1
NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per GPU on this pool
DATA = "synthetic: N(0,0.02) weights quantized to nvfp4 on device, N(0,1) bf16 tokens, seeded"
DTYPE = "nvfp4 weights (e2m1 + e4m3 per 16), bf16 activations, f32 accumulate"


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
            time.sleep(0.2)
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


def timed_events(fn, stream, world):
    """Device time (ms) of fn() between two events on `stream`, bracketed by a
    barrier and a synchronize on both sides; max over ranks."""
    import torch

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1), world)


def pipelined_e2e(run_step, xh, yh, xd_bufs, out_bufs, stream, n):
    """n end-to-end steps through the public API, double-buffered the way a
    serving loop runs them: step i copies its inputs from pinned host memory
    (xh) into xd_bufs[i % 2] on a copy-in stream, runs run_step(xd, out) on
    `stream`, and copies out_bufs[i % 2] back to pinned host memory (yh) on a
    copy-out stream, so its copies overlap the compute of steps i - 1 and
    i + 1.  Every step's copies are issued; `stream` waits for the last
    copy-out before returning, so events on `stream` around the call cover
    them all."""
    import torch

    dev = xd_bufs[0].device
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    start = torch.cuda.Event()
    start.record(stream)
    s_in.wait_event(start)
    s_out.wait_event(start)
    ev_in = [torch.cuda.Event() for _ in range(n)]
    ev_comp = [torch.cuda.Event() for _ in range(n)]
    ev_out = [torch.cuda.Event() for _ in range(n)]
    for i in range(n):
        b = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_comp[i - 2])  # step i - 2 has read this input buffer
            xd_bufs[b].copy_(xh, non_blocking=True)
            ev_in[i].record(s_in)
        with torch.cuda.stream(stream):
            stream.wait_event(ev_in[i])
            if i >= 2:
                stream.wait_event(ev_out[i - 2])  # step i - 2's output has been copied out
            run_step(xd_bufs[b], out_bufs[b])
            ev_comp[i].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[i])
            yh.copy_(out_bufs[b], non_blocking=True)
            ev_out[i].record(s_out)
    stream.wait_event(ev_out[n - 1])


E2E_PIPELINE = ("double-buffered: inputs copied in and outputs copied out on two copy streams, each step's copies "
                "overlapping the neighbouring steps' compute")


def capture(fn, stream):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def quantized(shape, seed, dev):
    import torch

    import b2moe

    gen = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * 0.02
    return b2moe.quantize(w)


def make_bank(dev, seed, experts=None):
    """MLX-layout expert bank; expert e's matrices come from seed + e, so a
    rank's slice is the same bytes whatever the number of ranks."""
    import torch

    import b2moe

    experts = range(E) if experts is None else experts
    parts = {nm: ([], []) for nm in ("gate", "up", "down")}
    for e in experts:
        for j, (nm, shp) in enumerate((("gate", (F, H)), ("up", (F, H)), ("down", (H, F)))):
            c, s = quantized(shp, seed * 1000 + e * 3 + j, dev)
            parts[nm][0].append(c)
            parts[nm][1].append(s)
    t = {}
    for nm, (cs, ss) in parts.items():
        t[nm + "_codes"] = torch.stack(cs)
        t[nm + "_scales"] = torch.stack(ss)
    return b2moe.ExpertBank(**t)


# --------------------------------------------------------------------------- CPU baselines
def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    O.build()
    return O


def cpu_block_sample(n_tokens, threads, seed=7):
    """The reference's CPU path for the MoE block on `n_tokens` tokens: MLX's
    own fp_qmm_t (bf16 activations: the stock path, compiled from the
    reference into oracle/_ref; the restatement when that library is absent)
    for the 8 routed experts' gate, up and down GEMVs of every token -- MLX's
    CPU gather_qmm is a loop over (token, expert) pairs, so decode and
    prefill cost the same per token -- with router, top-k, SwiGLU and the
    ordered combine from the restatement.  All 128 experts exist (random
    NVFP4 codes and in-range scale bytes, 340 MB), so the routed experts'
    weights come from DRAM as on the GPU.  Returns (tokens/s, kind, threads,
    seconds)."""
    import concurrent.futures as cf

    import numpy as np

    O = _oracle()
    kind = "reference" if O.ref_available() else "port"
    rng = np.random.default_rng(seed)

    def bank(rows, K):
        codes = rng.integers(0, 2 ** 32, size=(E, rows, K // 8), dtype=np.uint64).astype(np.uint32)
        scales = rng.integers(0x28, 0x38, size=(E, rows, K // 16), dtype=np.uint8)
        return codes, scales

    gw, gs = bank(F, H)
    uw, us = bank(F, H)
    dw, ds = bank(H, F)
    wr = (rng.standard_normal((E, H), dtype=np.float32) * 0.02).astype(np.float32)
    qmm = O.ref_qmm_bf16 if kind == "reference" else O.qmm_bf16
    xs = [O.f32_to_bf16(rng.standard_normal((1, H), dtype=np.float32)) for _ in range(n_tokens)]

    def one(x):
        inds, wts = O.topk_softmax(O.router_logits(x, wr), TOPK)
        d = np.zeros((1, TOPK, H), np.uint16)
        for s in range(TOPK):
            e = int(inds[0, s])
            a = O.swiglu_bf16(qmm(x, gw[e], gs[e]), qmm(x, uw[e], us[e]))
            d[0, s] = qmm(a, dw[e], ds[e])[0]
        return O.combine_bf16(d, wts)

    one(xs[0])
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, xs))
    dt = time.perf_counter() - t0
    return n_tokens / dt, kind, threads, dt


def cpu_block_baseline(threads, target_s=12.0):
    """cpu_block_sample sized to about target_s seconds by a calibration run."""
    _, _, _, dt0 = cpu_block_sample(threads, threads)
    per_token = max(dt0 / threads, 1e-4)
    n = max(threads, int(target_s / per_token) // threads * threads)
    v, kind, thr, dt = cpu_block_sample(n, threads)
    return {"value": round(v, 3), "unit": "tok/s", "cores": thr, "kind": kind,
            "sample": f"{n} tokens through one block (router, top-8 of 128 experts, SwiGLU, combine) on {thr} host "
                      f"threads, {dt:.1f} s; expert GEMVs = MLX fp_qmm_t on bf16 x"}


def cpu_qmm_baseline(M, threads, target_s=8.0, seed=11):
    """MLX's own fp_qmm_t (oracle/_ref; the restatement when absent) on the
    host cores for the configs[0] shape: independent calls on `threads`
    threads over a bounded sample."""
    import concurrent.futures as cf

    import numpy as np

    O = _oracle()
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
    return {"value": round(n * M / dt, 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"{n} calls of M={M} on {threads} host threads, {dt:.1f} s (MLX fp_qmm_t, bf16 x)"}


# --------------------------------------------------------------------------- decode
def bench_decode(args, world, rank, local, cpu):
    import torch

    import b2moe

    dev = torch.device("cuda", local)
    nblk = args.blocks
    blocks = []
    for b in range(nblk):
        bank = make_bank(dev, seed=11 + 100 * b + 1000 * rank)
        gen = torch.Generator(device=dev).manual_seed(5000 + b)
        wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
        blocks.append(b2moe.MoEBlock(bank, wr, top_k=TOPK, prepare_decode=True))
    bufs = [torch.randn(1, H, device=dev).to(torch.bfloat16)] + \
           [torch.empty(1, H, device=dev, dtype=torch.bfloat16) for _ in range(nblk)]
    K, W = args.steps, args.warmup

    def run(n):
        # block i % nblk consumes the previous block's output (a layer stack)
        for i in range(n):
            j = i % nblk
            blocks[j](bufs[j], out=bufs[j + 1])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for b in blocks:
            b._workspace(1, dev)  # this stream's workspace, allocated before capture
        run(W)
        torch.cuda.synchronize()
        g = capture(lambda: run(K), stream)
        g.replay()  # untimed: first replay of the graph
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = timed_events(g.replay, stream, world)
    per_step_ms = ms / K
    hbm, _, peak_kind = peaks()
    achieved = DECODE_BYTES / (per_step_ms * 1e-3) / 1e9

    # end to end through the public API: the token from pinned host memory,
    # the block's output back to pinned host memory, every step
    xh = torch.randn(1, H).to(torch.bfloat16).pin_memory()
    yh = torch.empty(1, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    yd = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    cur = torch.cuda.current_stream(dev)

    def e2e(n):
        for i in range(n):
            xd.copy_(xh, non_blocking=True)
            blocks[i % nblk](xd, out=yd)
            yh.copy_(yd, non_blocking=True)

    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), cur, world)
    rec = {
        "value": round(world * 1e3 / per_step_ms, 2), "unit": "tok/s", "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 6), "higher_is_better": True, "scaling": "weak", "dtype": DTYPE,
        "data": DATA,
        "config": {"workload": "moe_decode_block (BASELINE configs[1])", "hidden": H, "experts": E, "top_k": TOPK,
                   "ffn": F, "router": "softmax top-8 renormalised, fp32 router weight", "tokens_per_step": 1,
                   "blocks_rotated": nblk,
                   "l2": f"inputs larger than L2 ({nblk} distinct blocks chained, "
                         f"{nblk * BLOCK_BANK_MB:.0f} MB of expert weights)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": DECODE_TRAFFIC_BYTES,
                     "kernel": "decode_block_tma_kernel (fused router, top-k, gate/up+SwiGLU, down, combine)",
                     "algorithmic_bytes_per_launch": DECODE_BYTES,
                     "peak_source": peak_kind + " copy bandwidth (of measured)"},
        "e2e": {"value": round(world * K / (ms_e2e * 1e-3), 2), "unit": "tok/s", "h2d_bytes_per_step": H * 2,
                "d2h_bytes_per_step": H * 2},
        "gpu_launches": K,
        "clocks": clk.summary(),
    }
    if cpu:
        rec["cpu_baseline"] = cpu_block_baseline(os.cpu_count() or 1)
    del blocks
    torch.cuda.empty_cache()
    if world == 1:
        rec["e2e_c_abi"] = capi_decode_e2e(K, W, local)
    return rec


def capi_decode_e2e(steps, warmup, local):
    """The same end-to-end measurement through the bare C ABI with no Python
    in the loop (lib/capi_decode_e2e, built with the library): per step the
    token from pinned host memory, b2_moe_block_forward, the output back to
    pinned host memory, 16 rotated config-2 blocks of synthetic NVFP4 bytes."""
    exe = os.path.join(ROOT, "mlxfast-challenge_senpai_b200", "lib", "capi_decode_e2e")
    if not os.path.exists(exe):
        return {"unavailable": "lib/capi_decode_e2e not built"}
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(local)) if "CUDA_VISIBLE_DEVICES" not in os.environ else None
    try:
        r = subprocess.run([exe, str(max(steps, 100)), str(max(warmup, 3)), "16"], capture_output=True, text=True,
                           timeout=600, env=env)
        d = json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as e:  # noqa: BLE001 -- reported, the record stands without it
        return {"unavailable": f"{type(e).__name__}: {str(e)[:120]}"}
    us = d["us_per_step"]
    return {"value": round(1e6 / us, 2), "unit": "tok/s", "us_per_step": us, "h2d_bytes_per_step": H * 2,
            "d2h_bytes_per_step": H * 2, "steps": d["steps"], "device_status": d["device_status"],
            "via": "lib/capi_decode_e2e: cudaMemcpyAsync H2D, b2_moe_block_forward, cudaMemcpyAsync D2H per step, "
                   "CUDA events around the steps"}


# --------------------------------------------------------------------------- prefill
def bench_prefill(args, world, rank, local, cpu):
    import torch

    import b2moe

    dev = torch.device("cuda", local)
    bank = make_bank(dev, seed=21 + 1000 * rank)
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    # N(0, 0.02) router rows over N(0, 1) tokens: near-uniform expert load
    wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
    blk = b2moe.MoEBlock(bank, wr, top_k=TOPK, prepare_prefill=True)
    x = torch.randn(PREFILL_T, H, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty_like(x)
    K, W = args.steps, args.warmup
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        blk._workspace(PREFILL_T, dev)  # this stream's workspace, allocated before capture
        for _ in range(W):
            blk(x, out=out)
        torch.cuda.synchronize()
        g = capture(lambda: blk(x, out=out), stream)

        def run():
            for _ in range(K):
                g.replay()

        with ClockSampler(local) as clk:
            ms = timed_events(run, stream, world)
    per_step_ms = ms / K
    _, tflops_peak, peak_kind = peaks()
    achieved = PREFILL_FLOP / (per_step_ms * 1e-3) / 1e12
    xh = x.cpu().pin_memory()
    yh = torch.empty(PREFILL_T, H, dtype=torch.bfloat16).pin_memory()
    xds = [torch.empty_like(x) for _ in range(2)]
    outs = [out, torch.empty_like(out)]
    cur = torch.cuda.current_stream(dev)

    def e2e(n):
        pipelined_e2e(lambda xd, o: blk(xd, out=o), xh, yh, xds, outs, cur, n)

    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), cur, world)
    rec = {
        "value": round(world * PREFILL_T * 1e3 / per_step_ms, 1), "unit": "tok/s", "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "dtype": "nvfp4 weights dequantized exactly to bf16 in TMEM (tcgen05 A operand), bf16 activations, "
                 "f32 accumulate", "data": DATA,
        "config": {"workload": "moe_prefill_block (BASELINE configs[2])", "tokens": PREFILL_T, "hidden": H,
                   "experts": E, "top_k": TOPK, "ffn": F, "router": "softmax top-8, near-uniform load",
                   "l2": "inputs larger than L2 (340 MB expert bank per step)", "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / tflops_peak, 4), "traffic": PREFILL_GEMM_TRAFFIC_BYTES,
                     "kernel": "whole block step (expert GEMM flops / step time); traffic of the gate/up "
                               "grouped GEMM launch", "algorithmic_flop_per_step": PREFILL_FLOP,
                     "peak_source": peak_kind + " bf16 cuBLAS burst (of measured)"},
        "e2e": {"value": round(world * K * PREFILL_T / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": PREFILL_T * H * 2, "d2h_bytes_per_step": PREFILL_T * H * 2,
                "pipeline": E2E_PIPELINE},
        # router logits, top-k, sort histogram + scatter, token tiles, row
        # gather, gate/up GEMM, down GEMM, combine
        "gpu_launches": 9 * K,
        "clocks": clk.summary(),
    }
    if cpu:
        rec["cpu_baseline"] = cpu_block_baseline(os.cpu_count() or 1)
    del blk, bank
    torch.cuda.empty_cache()
    return rec


# --------------------------------------------------------------------------- decode step
STEP_LAYERS, STEP_NQ, STEP_NKV, STEP_HD, STEP_SEQ = 4, 32, 4, 128, 4096
STEP_LAYER_BYTES = ((STEP_NQ + 2 * STEP_NKV) * STEP_HD * H + H * STEP_NQ * STEP_HD) * 9 // 16 + \
    2 * STEP_SEQ * STEP_NKV * STEP_HD * 2 + DECODE_BYTES
STEP_BYTES = STEP_LAYERS * STEP_LAYER_BYTES


def make_decode_stack(dev, seed, layers=STEP_LAYERS):
    import torch

    import b2moe

    attn, moe = [], []
    gen = torch.Generator(device=dev).manual_seed(seed)
    for li in range(layers):
        qkv = quantized(((STEP_NQ + 2 * STEP_NKV) * STEP_HD, H), seed * 100 + 10 * li + 1, dev)
        o = quantized((H, STEP_NQ * STEP_HD), seed * 100 + 10 * li + 2, dev)
        norm = lambda: (1.0 + 0.1 * torch.randn(H, generator=gen, device=dev)).to(torch.bfloat16)
        attn.append(b2moe.AttentionWeights(attn_norm_w=norm(), qkv_codes=qkv[0], qkv_scales=qkv[1], o_codes=o[0],
                                           o_scales=o[1], mlp_norm_w=norm()))
        bank = make_bank(dev, seed=seed * 100 + 10 * li + 3)
        wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
        moe.append(b2moe.MoEBlock(bank, wr, top_k=TOPK, prepare_decode=True))
    fn = (1.0 + 0.1 * torch.randn(H, generator=gen, device=dev)).to(torch.bfloat16)
    stack = b2moe.DecoderStack(attn, moe, fn, STEP_NQ, STEP_NKV, STEP_SEQ, STEP_HD, rope_theta=1e6)
    for kc, vc in zip(stack.k_cache, stack.v_cache):  # a full 4096-position context
        kc.copy_(torch.randn(kc.shape, generator=gen, device=dev).to(torch.bfloat16))
        vc.copy_(torch.randn(vc.shape, generator=gen, device=dev).to(torch.bfloat16))
    return stack


def bench_decode_step(args, world, rank, local, cpu):
    """one token through a 4-layer stack (attention with
    a 4096-long bf16 KV cache + the 128-expert MoE block per layer) at the
    last cache position; two stacks alternate (330 MB of weights and caches,
    beyond L2)."""
    import torch

    dev = torch.device("cuda", local)
    nst, nl = args.stacks, args.layers
    stacks = [make_decode_stack(dev, 61 + 7 * j + 1000 * rank, nl) for j in range(nst)]
    pos = STEP_SEQ - 1
    x0 = torch.randn(1, H, device=dev).to(torch.bfloat16)
    outs = [torch.empty(1, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    K, W = args.steps, args.warmup

    def run(n):
        # step i feeds step i+1 (greedy decoding feeds the sampled token's
        # embedding; with no LM head the hidden state stands in for it)
        prev = x0
        for i in range(n):
            prev = stacks[i % nst].step(prev, pos, out=outs[i % 2])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for st_ in stacks:  # this stream's MoE workspaces before capture
            for m in st_.moe:
                m._workspace(1, dev)
        run(W)
        torch.cuda.synchronize()
        g = capture(lambda: run(K), stream)
        g.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = timed_events(g.replay, stream, world)
    per_step_ms = ms / K
    hbm, _, peak_kind = peaks()
    step_bytes = nl * STEP_LAYER_BYTES
    achieved = step_bytes / (per_step_ms * 1e-3) / 1e9
    xh = x0.cpu().pin_memory()
    yh = torch.empty(1, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x0)
    cur = torch.cuda.current_stream(dev)

    def e2e(n):
        for i in range(n):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(stacks[i % nst].step(xd, pos, out=outs[i % 2]), non_blocking=True)

    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), cur, world)
    rec = {
        "value": round(world * 1e3 / per_step_ms, 2), "unit": "tok/s", "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 6), "higher_is_better": True, "scaling": "weak", "dtype": DTYPE,
        "data": DATA + ", N(0,1) bf16 KV caches",
        "config": {"workload": f"decode_step {nl}-layer stack (BASELINE configs[3])", "layers": nl,
                   "hidden": H, "q_heads": STEP_NQ, "kv_heads": STEP_NKV, "head_dim": STEP_HD, "rope_theta": 1e6,
                   "kv_cache_len": STEP_SEQ, "position": pos, "experts": E, "top_k": TOPK, "ffn": F,
                   "lm_head": "none (not specified)", "stacks_rotated": nst,
                   "l2": f"inputs larger than L2 ({nst} stacks, {nst * step_bytes / 1e6:.0f} MB of weights and "
                         "caches)" if nst * step_bytes > 126e6 else "working set fits in L2 (profiling case)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "kernel": "whole step (weights + KV cache bytes / step time)",
                     "algorithmic_bytes_per_step": step_bytes,
                     "peak_source": peak_kind + " copy bandwidth (of measured)"},
        "e2e": {"value": round(world * K / (ms_e2e * 1e-3), 2), "unit": "tok/s", "h2d_bytes_per_step": H * 2,
                "d2h_bytes_per_step": H * 2},
        # per layer: 2 norms, qkv GEMV, attention, o GEMV, MoE; + final norm
        "gpu_launches": K * (6 * nl + 1),
        "clocks": clk.summary(),
    }
    if cpu:
        rec["cpu_baseline"] = cpu_step_baseline(os.cpu_count() or 1)
    del stacks
    torch.cuda.empty_cache()
    return rec


def cpu_step_baseline(threads, target_s=10.0):
    """The CPU path for the decode step, per token: the MoE blocks as
    cpu_block_sample (MLX's fp_qmm_t for the expert GEMVs) plus the attention
    projections through the same fp_qmm_t and the attention over a
    4096-long cache in numpy, on `threads` host threads (one token each)."""
    import concurrent.futures as cf

    import numpy as np

    O = _oracle()
    kind = "reference" if O.ref_available() else "port"
    qmm = O.ref_qmm_bf16 if kind == "reference" else O.qmm_bf16
    rng = np.random.default_rng(3)

    def rand_q(rows, K):
        return (rng.integers(0, 2 ** 32, size=(rows, K // 8), dtype=np.uint64).astype(np.uint32),
                rng.integers(0x28, 0x38, size=(rows, K // 16), dtype=np.uint8))

    qkv = rand_q((STEP_NQ + 2 * STEP_NKV) * STEP_HD, H)
    o = rand_q(H, STEP_NQ * STEP_HD)
    kc = O.f32_to_bf16(rng.standard_normal((STEP_NKV, STEP_SEQ, STEP_HD), dtype=np.float32))
    vc = O.f32_to_bf16(rng.standard_normal((STEP_NKV, STEP_SEQ, STEP_HD), dtype=np.float32))

    def attn_layer(x):
        y = qmm(x, *qkv)
        q = y[0, : STEP_NQ * STEP_HD].reshape(STEP_NQ, STEP_HD)
        a = O.attention_bf16(q, kc, vc).reshape(1, -1)
        return qmm(a, *o)

    x = O.f32_to_bf16(rng.standard_normal((1, H), dtype=np.float32))
    t0 = time.perf_counter()
    attn_layer(x)
    one = max(time.perf_counter() - t0, 1e-4)
    n = max(threads, int(target_s * threads / (one * STEP_LAYERS)) // threads * threads)
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda _: [attn_layer(x) for _ in range(STEP_LAYERS)], range(n)))
    dt_attn = (time.perf_counter() - t0) / n  # wall seconds per token of the attention halves, all threads busy
    blk = cpu_block_baseline(threads, target_s=target_s)
    per_token = dt_attn + STEP_LAYERS / blk["value"]
    return {"value": round(1.0 / per_token, 3), "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"{n} tokens of 4 attention halves ({dt_attn * n:.1f} s) + the MoE block sample "
                      f"({blk['value']} tok/s per block) on {threads} host threads"}


# --------------------------------------------------------------------------- W4A4 (north_star (c))
W4_M, W4_N, W4_K, W4_SETS = 2048, 4096, 4096, 16
W4_FLOP = 2 * W4_M * W4_N * W4_K


def _to_blocked(sc):
    """Scale bytes [rows, cols] -> cuBLASLt's VEC16 block layout (128 x 4
    tiles, element (r, c) of a tile at (r % 32) * 16 + (r // 32) * 4 + c)."""
    import torch

    rows, cols = sc.shape
    rb, cb = -(-rows // 128), -(-cols // 4)
    pad = torch.zeros(rb * 128, cb * 4, dtype=sc.dtype, device=sc.device)
    pad[:rows, :cols] = sc
    blocks = pad.view(rb, 128, cb, 4).permute(0, 2, 1, 3)
    return blocks.reshape(-1, 4, 32, 4).transpose(1, 2).reshape(-1, 32, 16).flatten()


def bench_w4a4(args, world, rank, local, cpu):
    """The W4A4 product (qqmm nvfp4: activations quantized on the fly) for a
    2048-token block through a 4096 x 4096 NVFP4 weight, on the block-scaled
    tcgen05 kernels, with the reference's own sm_100 path -- cuBLASLt with
    CUDA_R_4F_E2M1 operands and VEC16_UE4M3 scales (reached here through
    torch._scaled_mm) -- timed on the same operands."""
    import torch

    import b2moe

    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(17 + rank)
    ws = [quantized((W4_N, W4_K), 300 + i + 1000 * rank, dev) for i in range(W4_SETS)]
    xs = [(torch.randn(W4_M, W4_K, generator=gen, device=dev)).to(torch.bfloat16) for _ in range(W4_SETS)]
    wk = torch.empty(W4_M * W4_K, dtype=torch.uint8, device=dev)  # >= b2_qqmm_workspace_size
    ys = [torch.empty(W4_M, W4_N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    K, W = args.steps, args.warmup
    # every timed loop is a CUDA graph replay (device time, no host gaps)
    stream = torch.cuda.Stream(device=dev)

    def run(n):
        for i in range(n):
            ys[i % 2] = b2moe.qqmm(xs[i % W4_SETS], *ws[i % W4_SETS], workspace=wk)

    with torch.cuda.stream(stream):
        run(W)
        torch.cuda.synchronize()
        g_q = capture(lambda: run(K), stream)
        g_q.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = timed_events(g_q.replay, stream, world) / K
    _, tflops_peak, peak_kind = peaks()
    fp4_peak = 4 * tflops_peak
    achieved = W4_FLOP / (ms * 1e-3) / 1e12
    # the GEMM alone (activations already quantized)
    qx = [b2moe.quantize_activations(x) for x in xs]

    def run_g(n):  # outputs are dropped at once, so the allocator reuses one buffer
        for i in range(n):
            b2moe.nvfp4_gemm(*qx[i % W4_SETS], *ws[i % W4_SETS])

    with torch.cuda.stream(stream):
        run_g(W)
        torch.cuda.synchronize()
        g_g = capture(lambda: run_g(K), stream)
        g_g.replay()
        torch.cuda.synchronize()
        ms_gemm = timed_events(g_g.replay, stream, world) / K
    # the reference's sm_100 path on the same operands
    cublas = {"unavailable": None}
    try:
        fp4 = torch.float4_e2m1fn_x2
        a = [q[0].view(torch.uint8).view(fp4) for q in qx]
        sa = [_to_blocked(q[1]).view(torch.float8_e4m3fn) for q in qx]
        b = [w[0].view(torch.uint8).view(fp4) for w in ws]
        sb = [_to_blocked(w[1]).view(torch.float8_e4m3fn) for w in ws]
        def mm_c(i):
            return torch._scaled_mm(a[i % W4_SETS], b[i % W4_SETS].t(), sa[i % W4_SETS], sb[i % W4_SETS],
                                    out_dtype=torch.bfloat16)

        def run_c(n):
            for i in range(n):
                mm_c(i)

        yc = mm_c(0)
        yo = b2moe.nvfp4_gemm(*qx[0], *ws[0])
        diff = (yc.float() - yo.float()).abs()
        with torch.cuda.stream(stream):
            run_c(W)
            torch.cuda.synchronize()
            g_c = capture(lambda: run_c(K), stream)
            g_c.replay()
            torch.cuda.synchronize()
            ms_c = timed_events(g_c.replay, stream, world) / K
        cublas = {"ms_per_gemm": round(ms_c, 5), "tflops": round(W4_FLOP / (ms_c * 1e-3) / 1e12, 1),
                  "speed_ratio_b2_over_cublaslt": round(ms_c / ms_gemm, 3),
                  "max_abs_diff_vs_b2": round(float(diff.max()), 5),
                  "mean_rel_diff_vs_b2": round(float(diff.sum() / yc.float().abs().sum()), 7),
                  "via": "torch._scaled_mm (cuBLASLt, NVFP4 VEC16_UE4M3)"}
    except Exception as e:  # noqa: BLE001 -- reported, the line stands without it
        cublas = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    rec = {
        "value": round(world * W4_M * 1e3 / ms, 1), "unit": "tok/s", "steps": K, "warmup": W,
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "dtype": "nvfp4 activations and weights (e2m1 + ue4m3 per 16), f32 accumulate, bf16 out",
        "data": "synthetic: N(0,0.02) weights quantized on device, N(0,1) bf16 activations, seeded",
        "config": {"workload": "w4a4 qqmm nvfp4 (north_star (c))", "M": W4_M, "N": W4_N, "K": W4_K,
                   "sets_rotated": W4_SETS, "l2": f"inputs larger than L2 ({W4_SETS} weight + activation sets)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": fp4_peak, "unit": "TFLOP/s",
                     "frac": round(achieved / fp4_peak, 4), "traffic": None,
                     "kernel": "activation quantizer + w4a4_gemm_kernel (tcgen05 kind::mxf4nvf4)",
                     "gemm_only_ms": round(ms_gemm, 5),
                     "gemm_only_tflops": round(W4_FLOP / (ms_gemm * 1e-3) / 1e12, 1),
                     "peak_source": f"4 x {peak_kind} bf16 cuBLAS burst (dense fp4 = 4 x dense bf16 nominally)"},
        "cublaslt_reference_path": cublas,
        "e2e": None,
        "gpu_launches": 2 * K,
        "clocks": clk.summary(),
    }
    xh = xs[0].cpu().pin_memory()
    yh = torch.empty(W4_M, W4_N, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(xs[0])

    def e2e(n):
        for i in range(n):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(b2moe.qqmm(xd, *ws[i % W4_SETS], workspace=wk), non_blocking=True)

    cur = torch.cuda.current_stream(dev)
    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), cur, world) / K
    rec["e2e"] = {"value": round(world * W4_M * 1e3 / ms_e2e, 1), "unit": "tok/s",
                  "h2d_bytes_per_step": W4_M * W4_K * 2, "d2h_bytes_per_step": W4_M * W4_N * 2}
    del ws, xs, qx, g_q, g_g
    torch.cuda.empty_cache()
    return rec


# --------------------------------------------------------------------------- single qmm
def bench_qmm(args, world, rank, local, cpu, M):
    import torch

    import b2moe

    dev = torch.device("cuda", local)
    ws = [quantized((QMM_N, QMM_K), 99 + 31 * i + 1000 * rank, dev) for i in range(QMM_WEIGHTS)]
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    x0 = torch.randn(M, QMM_K, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    K, W = args.steps, args.warmup

    def run(n):
        # call i multiplies the previous call's output by weight i % 24
        prev = x0
        for i in range(n):
            prev = b2moe.quantized_matmul(prev, *ws[i % QMM_WEIGHTS])

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        run(W)
        torch.cuda.synchronize()
        g = capture(lambda: run(K), stream)
        g.replay()
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            ms = timed_events(g.replay, stream, world)
    per_step_ms = ms / K
    hbm, _, peak_kind = peaks()
    algo = QMM_WEIGHT_BYTES + 2 * M * QMM_K * 2
    achieved = algo / (per_step_ms * 1e-3) / 1e9
    xh = x0.cpu().pin_memory()
    yh = torch.empty(M, QMM_N, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x0)
    cur = torch.cuda.current_stream(dev)

    def e2e(n):
        for i in range(n):
            xd.copy_(xh, non_blocking=True)
            yh.copy_(b2moe.quantized_matmul(xd, *ws[i % QMM_WEIGHTS]), non_blocking=True)

    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), cur, world)
    rec = {
        "value": round(world * M * 1e3 / per_step_ms, 2), "unit": "tok/s", "steps": K, "warmup": W,
        "ms_per_step": round(per_step_ms, 6), "higher_is_better": True, "scaling": "weak", "dtype": DTYPE,
        "data": "synthetic: N(0,0.02) weights quantized to nvfp4 on device, N(0,1) bf16 x, seeded",
        "config": {"workload": f"quantized_matmul nvfp4 (BASELINE configs[0]), M={M}", "M": M, "N": QMM_N,
                   "K": QMM_K, "weights_rotated": QMM_WEIGHTS,
                   "l2": f"inputs larger than L2 ({QMM_WEIGHTS} distinct weights, "
                         f"{QMM_WEIGHTS * QMM_WEIGHT_BYTES / 1e6:.0f} MB)", "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": QMM_M1_TRAFFIC_BYTES if M == 1 else None,
                     "kernel": "qmv_mma_kernel (tensor-core GEMV, bf16 x, M <= 32)",
                     "algorithmic_bytes_per_launch": algo, "peak_source": peak_kind + " copy bandwidth (of measured)"},
        "e2e": {"value": round(world * K * M / (ms_e2e * 1e-3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": M * QMM_K * 2, "d2h_bytes_per_step": M * QMM_N * 2},
        "gpu_launches": K,
        "clocks": clk.summary(),
    }
    if cpu:
        rec["cpu_baseline"] = cpu_qmm_baseline(M, os.cpu_count() or 1)
    del ws
    torch.cuda.empty_cache()
    return rec


# --------------------------------------------------------------------------- EP prefill
def zipf_logit_bias(dev):
    """log of a Zipf(1.1) expert popularity over a seeded rank -> expert
    permutation: added to the router logits, it skews the load."""
    import numpy as np
    import torch

    perm = np.random.default_rng(5).permutation(E)
    pop = np.empty(E, np.float32)
    pop[perm] = (1.0 / np.arange(1, E + 1) ** ZIPF_S).astype(np.float32)
    return torch.from_numpy(np.log(pop)).to(dev)


def bench_ep_prefill(args, world, rank, local, cpu):
    import numpy as np
    import torch
    import torch.distributed as dist

    import b2moe
    import ep

    dev = torch.device("cuda", local)
    El = E // world
    T_l = EP_TOKENS // world
    gen = torch.Generator(device=dev).manual_seed(778)  # the same router and tokens on every rank
    wr = torch.randn(E, H, generator=gen, device=dev, dtype=torch.float32) * 0.02
    x_all = torch.randn(EP_TOKENS, H, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    x = x_all[rank * T_l:(rank + 1) * T_l].contiguous()
    del x_all
    bias = zipf_logit_bias(dev)
    # expert placement: balanced from the expert counts of a separate
    # calibration batch (same popularity, other tokens), the same on every
    # rank; or contiguous ranges
    slot = None
    if args.ep_impl == "peer" and args.ep_placement == "balanced" and world > 1:
        gc = torch.Generator(device=dev).manual_seed(779)
        xc = torch.randn(EP_TOKENS, H, generator=gc, device=dev, dtype=torch.float32).to(torch.bfloat16)
        ic, _ = b2moe.router_topk(b2moe.router_logits(xc, wr) + bias, TOPK)
        loads = torch.bincount(ic.reshape(-1).long(), minlength=E).cpu().tolist()
        slot = ep.balanced_placement(loads, world)
        del xc
    mine = list(range(rank * El, (rank + 1) * El)) if slot is None else ep.local_experts(slot, world, rank)
    bank = make_bank(dev, seed=31, experts=mine)
    if args.ep_impl == "nccl":
        if not dist.is_initialized():
            import datetime
            import socket

            with socket.socket() as so:
                so.bind(("127.0.0.1", 0))
                port = so.getsockname()[1]
            dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                    timeout=datetime.timedelta(seconds=120), device_id=dev)
        local_blk = b2moe.MoEBlock(bank, wr[:El].contiguous(), top_k=1, prepare_prefill=True)
        blk = ep.EPMoEBlock(E, TOPK, ep.GpuOps(local_blk, wr, b2moe.ROUTER_SOFTMAX, None, True))
    else:
        blk = ep.EPPrefill(bank, wr, TOPK, T_l, local_bank=True, expert_slot=slot)
    out = torch.empty_like(x)
    logits = torch.empty(T_l, E, device=dev, dtype=torch.float32)

    def step(xin, o):
        lg = b2moe.router_logits(xin, wr)
        torch.add(lg, bias, out=logits)
        if args.ep_impl == "nccl":
            o.copy_(blk(xin, logits=logits))
        else:
            blk(xin, logits=logits, out=o)

    K, W = args.steps, args.warmup
    stream = torch.cuda.current_stream(dev)
    for _ in range(W):
        step(x, out)
    torch.cuda.synchronize()

    def run():
        for _ in range(K):
            step(x, out)

    with ClockSampler(local) as clk:
        ms_total = timed_events(run, stream, world)
    ms = ms_total / K

    # routing of this step (identical every step): rows per owning rank
    lg = b2moe.router_logits(x, wr) + bias
    inds, _ = b2moe.router_topk(lg, TOPK)
    slot_t = torch.tensor(slot if slot is not None else list(range(E)), device=dev)
    owner = (slot_t[inds.long()] // El).reshape(-1)
    sent = torch.bincount(owner, minlength=world).to(torch.float64)  # rows of my tokens per owner
    if world > 1:
        allsent = [torch.empty_like(sent) for _ in range(world)]
        dist.all_gather(allsent, sent)
        M = torch.stack(allsent).cpu().numpy()  # M[src, dst]
    else:
        M = sent.cpu().numpy()[None, :]
    recv = M.sum(axis=0)  # rows each rank computes
    remote_in = recv - np.diag(M)  # rows a rank fetches over NVLink and returns over NVLink
    flop_rank = recv * EXPERT_FLOP_PER_ROW
    nvl_bytes = remote_in * H * 2 * 2
    _, tflops_peak, peak_kind = peaks()
    lb_rank = np.maximum(flop_rank / (tflops_peak * 1e12), nvl_bytes / (NVLINK_GBS * 1e9)) * 1e3
    busiest = int(np.argmax(lb_rank))
    lb_ms = float(lb_rank[busiest])
    bound = "tensor" if flop_rank[busiest] / (tflops_peak * 1e12) >= nvl_bytes[busiest] / (NVLINK_GBS * 1e9) \
        else "nvlink"
    achieved_tf = flop_rank[busiest] / (ms * 1e-3) / 1e12

    # per-phase device times of one call (max over ranks)
    phases = None
    if args.ep_impl == "peer":
        blk.set_phase_timing(True)
        step(x, out)
        torch.cuda.synchronize()
        ph = blk.phase_times()
        blk.set_phase_timing(False)
        phases = {k2: round(max_over_ranks(v, world), 4) for k2, v in ph.items()}

    # end to end: this rank's token shard from pinned host memory, its
    # outputs back, every step
    xh = x.cpu().pin_memory()
    yh = torch.empty(T_l, H, dtype=torch.bfloat16).pin_memory()
    xds = [torch.empty_like(x) for _ in range(2)]
    outs = [out, torch.empty_like(out)]

    def e2e(n):
        pipelined_e2e(step, xh, yh, xds, outs, stream, n)

    e2e(W)
    ms_e2e = timed_events(lambda: e2e(K), stream, world) / K
    total_flop = EP_TOKENS * TOPK * EXPERT_FLOP_PER_ROW
    rec = {
        "metric": METRIC, "value": round(EP_TOKENS * 1e3 / ms, 1), "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "nvfp4 weights dequantized exactly to bf16 in TMEM (tcgen05 A operand), bf16 activations, "
                 "f32 accumulate",
        "data": DATA + f", Zipf({ZIPF_S}) expert popularity added to the router logits",
        "config": {"workload": "ep_moe_prefill (BASELINE configs[4])", "tokens": EP_TOKENS, "tokens_per_rank": T_l,
                   "hidden": H, "experts": E, "experts_per_rank": El, "top_k": TOPK, "ffn": F,
                   "router": f"softmax top-8 over logits + log Zipf({ZIPF_S}) popularity",
                   "parallelism": f"ep{world}",
                   "placement": "balanced: LPT over the expert counts of a separate 8192-token calibration batch"
                   if slot is not None else "contiguous expert ranges",
                   "exchange": "NVLink peer loads (dispatch) and stores (return), flag barriers (b2_moe_ep_prefill)"
                   if args.ep_impl == "peer" else "NCCL all_to_all_single (dispatch + return)",
                   "l2": "inputs larger than L2 (340 MB expert bank in total, 67 MB of gathered rows per step)"},
        "roofline": {"bound": bound, "achieved": round(achieved_tf, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                     "frac": round(achieved_tf / tflops_peak, 4), "traffic": None,
                     "kernel": "busiest rank's expert GEMM flops / step time",
                     "lower_bound_ms": round(lb_ms, 4), "frac_of_lower_bound": round(lb_ms / ms, 4),
                     "rows_per_rank": [int(v) for v in recv], "busiest_rank": busiest,
                     "nvlink_bytes_busiest": int(nvl_bytes[busiest]),
                     "expert_tflops_per_gpu": round(total_flop / (ms * 1e-3) / 1e12 / world, 1),
                     "peak_source": f"{peak_kind} bf16 cuBLAS burst {tflops_peak} TFLOP/s, NVLink {NVLINK_GBS} GB/s "
                                    "per direction (measured peer copy)"},
        "phases_ms": phases,
        "e2e": {"value": round(EP_TOKENS * 1e3 / ms_e2e, 1), "unit": "tok/s",
                "h2d_bytes_per_step": EP_TOKENS * H * 2, "d2h_bytes_per_step": EP_TOKENS * H * 2,
                "pipeline": E2E_PIPELINE},
        # per rank and step: router logits, top-k, 2 barriers, keys, peer
        # copies, sort (2), tiles, gather, gate/up GEMM, down GEMM, combine
        # (+ one torch add); one rank alone runs no barrier and no copies
        "gpu_launches": (13 if world > 1 else 10) * K * world if args.ep_impl == "peer" else None,
        "clocks": clk.summary(),
    }
    if cpu:
        rec["cpu_baseline"] = cpu_block_baseline(os.cpu_count() or 1)
    if args.ep_impl == "peer":
        blk.close()
    del blk, bank
    torch.cuda.empty_cache()
    return rec


# --------------------------------------------------------------------------- reference arm
def run_reference_arm(args, world, rank):
    """The reference's CPU path (MLX's own fp_qmm_t from oracle/_ref when it
    was built here, else the restatement) on all host cores, for the same
    metric, unit and config as this arm's line."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    if args.workload == "qmm":
        cb = cpu_qmm_baseline(args.qmm_m, threads)
        cfg = {"workload": f"quantized_matmul nvfp4 (BASELINE configs[0]), M={args.qmm_m}", "M": args.qmm_m,
               "N": QMM_N, "K": QMM_K}
        ms = 1e3 * args.qmm_m / cb["value"]
    elif args.workload == "decode_step":
        cb = cpu_step_baseline(threads)
        ms = 1e3 / cb["value"]
        cfg = {"workload": "decode_step 4-layer stack (BASELINE configs[3])", "layers": STEP_LAYERS, "hidden": H,
               "q_heads": STEP_NQ, "kv_heads": STEP_NKV, "head_dim": STEP_HD, "kv_cache_len": STEP_SEQ}
    else:
        cb = cpu_block_baseline(threads)
        ms = 1e3 / cb["value"]
        if args.workload == "decode":
            cfg = {"workload": "moe_decode_block (BASELINE configs[1])", "hidden": H, "experts": E, "top_k": TOPK,
                   "ffn": F}
        elif args.workload == "prefill":
            cfg = {"workload": "moe_prefill_block (BASELINE configs[2])", "tokens": PREFILL_T, "hidden": H,
                   "experts": E, "top_k": TOPK, "ffn": F}
        else:
            cfg = {"workload": "ep_moe_prefill (BASELINE configs[4])", "tokens": EP_TOKENS, "hidden": H,
                   "experts": E, "top_k": TOPK, "ffn": F,
                   "router": f"softmax top-8 over logits + log Zipf({ZIPF_S}) popularity",
                   "parallelism": "host threads (the CPU path does not shard over GPUs)"}
    return {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4 weights, bf16 activations (MLX CPU path)",
            "data": "synthetic seeded", "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b2", choices=["b2", "reference"])
    ap.add_argument("--workload", default="all",
                    choices=["all", "ep_prefill", "decode", "prefill", "qmm", "decode_step", "w4a4"])
    ap.add_argument("--ep-impl", default="peer", choices=["peer", "nccl"],
                    help="EP exchange: NVLink peer memory (the library path) or NCCL all_to_all (baseline)")
    ap.add_argument("--ep-placement", default="balanced", choices=["balanced", "contiguous"],
                    help="EP expert placement (peer path): balanced by calibration-batch load, or contiguous")
    ap.add_argument("--qmm-m", type=int, default=1, choices=[1, 32], help="rows of x for --workload qmm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--blocks", type=int, default=N_BLOCKS,
                    help="distinct decode blocks chained (default 16: weights exceed L2)")
    ap.add_argument("--stacks", type=int, default=2, help="decode_step: distinct stacks alternated (default 2)")
    ap.add_argument("--layers", type=int, default=STEP_LAYERS, help="decode_step: layers per stack (default 4)")
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
    cpu = world == 1 and rank == 0 and not args.no_cpu_baseline
    t0 = time.time()
    if args.workload in ("all", "ep_prefill"):
        res = bench_ep_prefill(args, world, rank, local, cpu)
        if args.workload == "all" and world == 1:
            res["configs"] = {
                "decode": bench_decode(args, world, rank, local, cpu),
                "prefill": bench_prefill(args, world, rank, local, cpu),
                "qmm_m1": bench_qmm(args, world, rank, local, cpu, 1),
                "qmm_m32": bench_qmm(args, world, rank, local, cpu, 32),
                "decode_step": bench_decode_step(args, world, rank, local, cpu),
                "w4a4": bench_w4a4(args, world, rank, local, cpu),
            }
    else:
        fn = {"decode": bench_decode, "prefill": bench_prefill, "decode_step": bench_decode_step,
              "w4a4": bench_w4a4}.get(args.workload)
        res = fn(args, world, rank, local, cpu) if fn else bench_qmm(args, world, rank, local, cpu, args.qmm_m)
        res = {"metric": METRIC, **res, "n_gpus": world, "vs_baseline": None}
    res["wall_s"] = round(time.time() - t0, 1)
    if rank == 0:
        print(json.dumps(res), flush=True)
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
