"""Benchmark: the AnimaXS DiT attention workload (configuration 4) on B200.

One "step" = one batch of 8 images per GPU (configuration 4's batch of 8
prompts) through the full 8-step DiT attention workload at 1024x1024: 8 Euler
steps x 28 blocks x (4096-token self-attention with q/k RMSNorm + 3-D RoPE
(1x64x64), then 4096x512 cross-attention with q/k RMSNorm), 16 heads x 128;
every attention call carries the whole batch.  Images are independent, so N
GPUs each process their own batch of 8 (weak scaling, no data-path
collective); N=1 is configuration 4 exactly.

Printed JSON line (rank 0):
  value       images/s for the whole job, inputs resident in HBM
  e2e         the same metric through the C-ABI executor with pinned HOST
              buffers, host<->device copies inside the timed region
  roofline    the dominant kernel (the 4096-token self-attention flash kernel),
              algorithmic FLOPs / its CUDA-event launch duration, vs the
              measured dense tensor peak
  cpu_baseline the CPU oracle on a bounded sample (rank 0, N=1)

``--impl reference`` times the reference's own algorithm on the host CPU (the
numpy restatement of its PyTorch oracles, all host threads) on the same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

S_SELF = 4096
S_CTX = 512
HEADS = 16
HD = 128
BLOCKS = 28
EULER_STEPS = 8
CALLS_PER_IMAGE = BLOCKS * EULER_STEPS            # 224 (self, cross) pairs
SELF_FLOPS = 4.0 * S_SELF * S_SELF * HD * HEADS   # 137.4 GFLOP per self-attention
CROSS_FLOPS = 4.0 * S_SELF * S_CTX * HD * HEADS   # 17.2 GFLOP per cross-attention
IMAGE_FLOPS = CALLS_PER_IMAGE * (SELF_FLOPS + CROSS_FLOPS)
BATCH = 8                                         # images per GPU per step (config 4)
POOL_BLOCKS = 3                                   # distinct resident input sets (> L2)
# DRAM bytes (read + write) of one batch-8 self-attention flash launch: the ncu
# capture in profiles/attn_fwd_sm100_selfattn4096_batch4.md measured 245.5 MB
# for batch 4; traffic scales with the batch.
TRAFFIC_PER_LAUNCH_MB = 490.8

METRIC = ("DiT attention throughput, 8-step 1024x1024 workload "
          "(28 blocks x 8 steps x [4096-tok self rms+rope3d + 4096x512 cross rms])")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d["bf16_tflops_sustained"], d["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- CPU legs --
# The CPU sample of the workload: steps {0, 7} x blocks {0, 27} x prompts {0, 7},
# eight (self 4096 + cross 4096x512) blocks of configuration 4.
CPU_SUBSET = [(p, s, b) for p in (0, 7) for s in (0, 7) for b in (0, 27)]
CPU_SAMPLE = ("blocks (self 4096 rms+rope3d + cross 4096x512 rms) of prompts {0,7} x steps {0,7} x "
              "blocks {0,27}, numpy fp32 oracle on all host threads; img/s = 1 / (mean block time x 224)")


def cpu_blocks(samples):
    """Time the CPU oracle (numpy fp32, all host threads) on workload blocks
    (prompt, step, block): the 4096-token self-attention + the 4096x512
    cross-attention of each.  Input generation is not timed.  Returns the
    seconds of each block."""
    from oracle import inputs  # the checker, used here only as the CPU baseline
    times = []
    for p, st, b in samples:
        sc, cc = inputs.workload_block(p, st, b)
        t0 = time.perf_counter()
        sc.oracle()
        cc.oracle()
        times.append(time.perf_counter() - t0)
    return times


def run_reference(args, rank):
    if rank != 0:
        return
    # Each step is one bounded sample: one block of the CPU subset (cycled).
    cpu_blocks([CPU_SUBSET[i % len(CPU_SUBSET)] for i in range(args.warmup)])
    t0 = time.perf_counter()
    times = cpu_blocks([CPU_SUBSET[i % len(CPU_SUBSET)] for i in range(args.steps)])
    wall = time.perf_counter() - t0
    t_block = statistics.mean(times)
    cores = os.cpu_count() or 1
    img_s = 1.0 / (t_block * CALLS_PER_IMAGE)
    line = {
        "impl": "reference", "metric": METRIC, "value": img_s, "unit": "img/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_block * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (CPU oracle)", "data": "synthetic",
        "config": {"workload": "config4: 8-step DiT attention @1024^2, 1 image",
                   "step": "one block (self 4096 + cross 4096x512) of the CPU subset; ms_per_step is the "
                           "measured time of one block",
                   "extrapolation": f"img/s = 1 / (mean block time x {CALLS_PER_IMAGE} blocks per image)",
                   "timed_s": wall},
        "tflops": (SELF_FLOPS + CROSS_FLOPS) / t_block / 1e12,
        "cpu_baseline": {"value": img_s, "unit": "img/s", "cores": cores, "kind": "port",
                         "sample": CPU_SAMPLE, "blocks_timed": len(times)},
        "e2e": {"value": img_s, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU legs --
def make_pool(torch, device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    pool = []
    for _ in range(POOL_BLOCKS):
        def r(*shape):
            return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).half()
        pool.append({
            "sq": r(BATCH, S_SELF, HEADS, HD), "sk": r(BATCH, S_SELF, HEADS, HD),
            "sv": r(BATCH, S_SELF, HEADS, HD), "cq": r(BATCH, S_SELF, HEADS, HD),
            "ck": r(BATCH, S_CTX, HEADS, HD), "cv": r(BATCH, S_CTX, HEADS, HD),
        })
    return pool


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    # Two contexts: the self-attention one times its flash-kernel launches with
    # CUDA events (the dominant kernel's roofline), the cross one does not.
    ex = ax.AttentionExecutor(local_rank)
    ex_cross = ax.AttentionExecutor(local_rank)
    stream = torch.cuda.current_stream(device)
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 64, 64).reshape(S_SELF, 64, 2, 2)).to(device)
    pool = make_pool(torch, device, 1234 + rank)
    o_self = torch.empty(BATCH, S_SELF, HEADS, HD, dtype=torch.float16, device=device)
    o_cross = torch.empty_like(o_self)

    def image():
        i = 0
        for _ in range(EULER_STEPS):
            for _ in range(BLOCKS):
                blk = pool[i % POOL_BLOCKS]
                ex.attention(blk["sq"], blk["sk"], blk["sv"], out=o_self, qk_norm="rms_rope",
                             rope_table=rope, stream=stream)
                ex_cross.attention(blk["cq"], blk["ck"], blk["cv"], out=o_cross, qk_norm="rms",
                                   stream=stream)
                i += 1

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        image()
    barrier()
    ex.synchronize(stream)
    ex_cross.synchronize(stream)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    ex.set_kernel_timing(True)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        image()
    t1.record(stream)
    barrier()
    clocks = sampler.stop()
    ex.set_kernel_timing(False)
    n_kern, kern_total_ms, kern_max_ms = ex.kernel_timing()
    ex.synchronize(stream)
    ex_cross.synchronize(stream)
    elapsed_ms = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    images = args.steps * world * BATCH
    value = images / (elapsed_ms / 1e3)
    launches = args.steps * CALLS_PER_IMAGE * 4   # per block: 2 x (q/k prologue + flash kernel)

    # ---------------- e2e: fused C-ABI calls with pinned host buffers ----------------
    e2e = None if args.no_e2e else run_e2e(torch, ex, device, stream, rope, args, world)
    # ---------------- config 5 head-sharded over the ranks (N > 1) ----------------
    cfg5 = cfg5_sharded(torch, dist, ex, rank, world, local_rank) if world > 1 and not args.no_cfg5 else None
    # ---------------- configurations 1, 2, 3, 5 on one GPU (N = 1) ----------------
    secondary = None
    if world == 1 and not args.no_secondary:
        secondary = secondary_configs(torch, ax, ex, device, args)

    if rank != 0:
        return
    peak_burst, peak_sust, hbm, peak_kind = peaks()
    avg_kern = kern_total_ms / n_kern if n_kern else float("nan")
    achieved = BATCH * SELF_FLOPS / (avg_kern / 1e3) / 1e12
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    per_clock = per_clock_peak(sms, clocks.get("sm_mhz"))
    line = {
        "metric": METRIC, "value": value, "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": "config4: 8-step DiT attention @1024^2, batch of 8 prompts per GPU "
                               "(224 self 4096 + 224 cross 4096x512 calls per step, each over the batch)",
                   "images_per_gpu_per_step": BATCH, "global_batch": BATCH * world, "seq_len": S_SELF,
                   "ctx_len": S_CTX, "heads": HEADS, "head_dim": HD, "parallelism": f"batch-shard x{world}",
                   "l2": f"inputs cycled over a {POOL_BLOCKS * 68 * BATCH} MiB resident pool (> 126 MB L2)"},
        "tflops_per_gpu": BATCH * IMAGE_FLOPS * args.steps / (elapsed_ms / 1e3) / 1e12,
        "frac_of_peak_per_gpu": BATCH * IMAGE_FLOPS * args.steps / (elapsed_ms / 1e3) / 1e12 / peak_sust,
        "roofline": {"kernel": "attn_fwd_sm100_kernel (4096-token self-attention, batch 8, 16 heads)",
                     "bound": "tensor", "achieved": achieved, "peak": peak_sust, "unit": "TFLOP/s",
                     "frac": achieved / peak_sust, "peak_kind": f"{peak_kind} bf16 dense, sustained",
                     "frac_of_burst_peak": achieved / peak_burst,
                     "flops_per_launch": BATCH * SELF_FLOPS, "avg_launch_ms": avg_kern,
                     "max_launch_ms": kern_max_ms, "launches_timed": n_kern,
                     "traffic": TRAFFIC_PER_LAUNCH_MB * 1e6, "traffic_unit": "bytes per launch",
                     "algorithmic_bytes": BATCH * 4 * S_SELF * HEADS * HD * 2,
                     # secondary figure: the ncu DRAM bytes per launch over the timed launch
                     "hbm_gbs": TRAFFIC_PER_LAUNCH_MB * 1e6 / (avg_kern / 1e3) / 1e9,
                     "hbm_frac": TRAFFIC_PER_LAUNCH_MB * 1e6 / (avg_kern / 1e3) / 1e9 / peaks()[2],
                     # The sustained peak was measured at a lower median clock than this
                     # run's; the per-clock peak and the burst fraction (the north-star check,
                     # target 0.60) are the clock-honest figures.
                     "sm_mhz_median": clocks.get("sm_mhz"),
                     "per_clock_peak": per_clock, "per_clock_peak_unit": "TFLOP/s",
                     "per_clock_peak_basis": f"{sms} SMs x 8192 FLOP/clk (one 128x128x16 MMA per 64 "
                                             "cycles, measured) x median SM clock of the timed region",
                     "frac_per_clock": achieved / per_clock if per_clock else None,
                     "north_star": {"check": "frac_of_burst_peak >= 0.60", "value": achieved / peak_burst,
                                    "met": achieved / peak_burst >= 0.60}},
        "clocks": clocks,
        "gpu_launches": launches,
        "e2e": e2e,
    }
    if secondary is not None:
        line["secondary"] = secondary
    if cfg5 is not None:
        line["cfg5_head_sharded"] = cfg5
    if world == 1 and not args.no_cpu_baseline:
        times = cpu_blocks(CPU_SUBSET)
        t_block = statistics.mean(times)
        line["cpu_baseline"] = {"value": 1.0 / (t_block * CALLS_PER_IMAGE), "unit": "img/s",
                                "cores": os.cpu_count() or 1, "kind": "port", "sample": CPU_SAMPLE,
                                "blocks_timed": len(times), "s_per_block": t_block}
    print(json.dumps(line), flush=True)


def per_clock_peak(sms, mhz):
    """Dense fp16 tensor peak at the measured clock: 8192 FLOP per clock per SM."""
    return sms * 8192 * mhz * 1e6 / 1e12 if mhz else None


E2E_INPUTS = (("sq", (1, S_SELF, HEADS, HD)), ("sk", (1, S_SELF, HEADS, HD)), ("sv", (1, S_SELF, HEADS, HD)),
              ("cq", (1, S_SELF, HEADS, HD)), ("ck", (1, S_CTX, HEADS, HD)), ("cv", (1, S_CTX, HEADS, HD)))


def _packed_views(buf):
    """q/k/v views of one block's packed inputs (E2E_INPUTS order)."""
    views, off = {}, 0
    for name, shape in E2E_INPUTS:
        n = 1
        for x in shape:
            n *= x
        views[name] = buf[off:off + n].view(*shape)
        off += n
    return views


def run_e2e(torch, ex, device, stream, rope, args, world):
    """Same metric through the fused C-ABI call with pinned host inputs/outputs.
    Per call: one H2D copy of the call's packed q,k,v (self) + q (cross), two
    fused attention calls, one D2H copy of both outputs; copies and compute
    overlap across three streams.  The cross-attention K/V of a block do not
    change across the 8 Euler steps (the adapter context is fixed per prompt),
    so, as the reference's DiT block executor does with its cross-K/V cache
    (DiTBlockExecutor.swift:19-43, reuse at :1110-1161), each image uploads a
    block's K/V once, at its first step, into a CrossKVCache (K normalised
    there) and the cross calls normalise only q.  Every byte an image needs
    crosses PCIe inside its own timed region."""
    from animaxs_b200 import CrossKVCache
    nblk = 4
    g = torch.Generator().manual_seed(99)
    n_in = sum(int(torch.Size(shape).numel()) for _, shape in E2E_INPUTS)
    n_ctx = sum(int(torch.Size(shape).numel()) for name, shape in E2E_INPUTS if name in ("ck", "cv"))
    n_pre = n_in - n_ctx  # sq, sk, sv, cq: every call
    host = [torch.randn(n_in, generator=g).half().pin_memory() for _ in range(nblk)]
    n_out = 2 * S_SELF * HEADS * HD
    outs_h = [torch.empty(n_out, dtype=torch.float16).pin_memory() for _ in range(2)]
    dev_buf = [torch.empty(n_in, dtype=torch.float16, device=device) for _ in range(2)]
    dev_in = [_packed_views(b) for b in dev_buf]
    dev_out_buf = [torch.empty(n_out, dtype=torch.float16, device=device) for _ in range(2)]
    dev_out = [[b[:n_out // 2].view(1, S_SELF, HEADS, HD), b[n_out // 2:].view(1, S_SELF, HEADS, HD)]
               for b in dev_out_buf]
    cache = CrossKVCache(ex, blocks=BLOCKS, batch=1, tokens=S_CTX, kv_heads=HEADS, head_dim=HD)
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    h2d = (n_pre * CALLS_PER_IMAGE + n_ctx * BLOCKS) * 2
    d2h = n_out * 2 * CALLS_PER_IMAGE

    def one_image():
        in_ready = [None, None]
        comp_done = [torch.cuda.Event(), torch.cuda.Event()]
        out_done = [torch.cuda.Event(), torch.cuda.Event()]
        first = [True, True]
        for i in range(CALLS_PER_IMAGE):
            slot = i & 1
            blk = i % BLOCKS
            ctx_upload = i < BLOCKS  # the block's first Euler step
            src = host[i % nblk]
            n = n_in if ctx_upload else n_pre
            with torch.cuda.stream(s_in):
                if not first[slot]:
                    s_in.wait_event(comp_done[slot])
                dev_buf[slot][:n].copy_(src[:n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_in)
                in_ready[slot] = ev
            stream.wait_event(in_ready[slot])
            if not first[slot]:
                stream.wait_event(out_done[slot])
            d = dev_in[slot]
            ex.attention(d["sq"], d["sk"], d["sv"], out=dev_out[slot][0], qk_norm="rms_rope",
                         rope_table=rope, stream=stream)
            if ctx_upload:
                cache.fill(blk, d["ck"], d["cv"], stream=stream)
            ex.attention(d["cq"], cache.k(blk), cache.v(blk), out=dev_out[slot][1], qk_norm="rms",
                         qk_norm_targets="q", stream=stream)
            comp_done[slot].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[slot])
                outs_h[slot].copy_(dev_out_buf[slot], non_blocking=True)
                out_done[slot].record(s_out)
            first[slot] = False

    steps = max(1, args.steps)
    one_image()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(steps):
        one_image()
    torch.cuda.synchronize(device)
    el = time.perf_counter() - t0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([el], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    cache.close()
    return {"value": steps * world / el, "unit": "img/s", "images_per_call": 1,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "path": "AttentionExecutor.attention -> animaxs_attn_forward (fused rms/rope); "
                                    "cross K/V uploaded once per block and image into a CrossKVCache"}


def _graph_us(torch, stream, calls, reps=3):
    """Device microseconds per call of `calls()` (a list of enqueues) replayed
    from one CUDA graph: the kernels back to back, host cost excluded."""
    with torch.cuda.stream(stream):
        n = calls()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            calls()
        graph.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(reps):
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            graph.replay()
            t1.record(stream)
            torch.cuda.synchronize()
            best = min(best, t0.elapsed_time(t1) * 1e3 / n)
        del graph
    return best


def _eager_us(torch, stream, calls, reps=3):
    """Host wall-clock microseconds per call of the eager Python loop (enqueue
    through AttentionExecutor.attention -> ctypes -> C ABI, then wait)."""
    best = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            n = calls()
        torch.cuda.synchronize()
        best = min(best, (time.perf_counter() - t0) * 1e6 / n)
    return best


def secondary_configs(torch, ax, ex, device, args):
    """Configurations 1, 2, 3 and 5 of BASELINE.json on one GPU, each with the
    oracle inputs (seeds as stated there), figures per call:
      graph_us    whole call (q/k prologue + attention) replayed from a CUDA graph
      kernel_us   the attention kernel alone (events around its launches)
      eager_us    host wall clock of the eager Python loop (Python + ctypes + C + GPU)
      tflops / frac_*  algorithmic FLOPs (valid query-key pairs) / graph_us,
                  against the measured dense peaks
      max_abs / mean_abs  parity against the fp32 CPU oracle (config 5: the
                  reference-generated golden rows)
      cpu_oracle_s  the oracle on the host cores (config 5: 512 of 16384 rows, x32)
    plus `c_abi`, the same calls timed from C (animaxs_b200/_build/call_bench),
    which separates the library's host cost from Python's."""
    import numpy as np

    from oracle import attn_oracle as ora  # the checker, used here for parity and the CPU baseline
    from oracle import inputs
    peak_burst, peak_sust, _, peak_kind = peaks()
    stream = torch.cuda.Stream(device)
    cases = {
        "config1_dit_self_1024": [inputs.dit_self(seed=0, grid=(1, 32, 32))],
        "config2_dit_cross_4096x512_masked": [inputs.dit_cross(seed=0, kv_valid=128)],
        "config3_qwen_prefill_28_layers": [inputs.qwen_prefill(layer=layer) for layer in range(28)],
        "config5_dit_self_16384": [inputs.dit_self(seed=0, grid=(1, 128, 128))],
    }
    out = {}
    for name, cs in cases.items():
        head = name.startswith("config3")

        def dev(x):
            t = torch.from_numpy(x).to(device)
            return t.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3) if head else t
        dv = [(dev(c.q), dev(c.k), dev(c.v), None if c.rope_table is None else torch.from_numpy(c.rope_table).to(device),
               None if c.kv_valid_len is None else c.kv_valid_len[0]) for c in cs]
        outs = [torch.empty_like(q) for q, _, _, _, _ in dv]
        c0 = cs[0]

        def calls(reps=1):
            for _ in range(reps):
                for (q, k, v, rope, valid), o in zip(dv, outs):
                    ex.attention(q, k, v, out=o, causal=c0.causal, qk_norm=c0.qk_norm, rope_table=rope,
                                 kv_valid_len=valid, stream=torch.cuda.current_stream(device))
            return reps * len(dv)
        reps = 2 if name.startswith("config5") else (4 if head else 40)
        graph_us = _graph_us(torch, stream, lambda: calls(reps))
        eager_us = _eager_us(torch, stream, lambda: calls(reps))
        ex.set_kernel_timing(True)
        with torch.cuda.stream(stream):
            calls(reps)
        torch.cuda.synchronize()
        ex.set_kernel_timing(False)
        n_k, tot_ms, _ = ex.kernel_timing()
        kernel_us = tot_ms * 1e3 / n_k
        flops = sum(c.flops() for c in cs) / len(cs)
        torch.cuda.synchronize()
        ex.synchronize()
        got = np.concatenate([o.float().cpu().numpy() for o in outs], axis=0)
        t0 = time.perf_counter()
        if name.startswith("config5"):
            g = np.load(os.path.join(ROOT, "tests", "golden", "attn_configs.npz"))
            mx, mn = ora.parity(got[:, g["cfg5_rows"]], g["cfg5_out"])
            rows = np.arange(0, 16384, 32)
            t0 = time.perf_counter()
            c0.oracle(rows=rows)
            cpu_s = (time.perf_counter() - t0) * 32
            cpu_note = "512 of 16384 query rows, x32"
        else:
            want = np.concatenate([c.oracle() for c in cs], axis=0)
            cpu_s = time.perf_counter() - t0
            mx, mn = ora.parity(got, want)
            cpu_note = "full"
        per = len(cs)  # calls per item (28 for the Qwen prefill)
        out[name] = {
            "graph_us": graph_us * per, "kernel_us": kernel_us * per, "eager_us": eager_us * per,
            "calls": per, "gflop": flops * per / 1e9,
            "tflops": flops / (graph_us * 1e-6) / 1e12, "tflops_kernel": flops / (kernel_us * 1e-6) / 1e12,
            "frac_sustained_kernel": flops / (kernel_us * 1e-6) / 1e12 / peak_sust,
            "frac_burst_kernel": flops / (kernel_us * 1e-6) / 1e12 / peak_burst,
            "max_abs": mx, "mean_abs": mn, "parity_ok": bool(mx <= 2e-3 and mn <= 2e-4),
            "cpu_oracle_s": cpu_s, "cpu_oracle": cpu_note, "cpu_cores": os.cpu_count() or 1,
        }
        del dv, outs
    out["rows_f"] = rows_f_figures(torch, ax, ex, device, stream, peak_sust, peak_burst)
    out["peak_kind"] = f"{peak_kind} bf16 dense"
    exe = os.path.join(ROOT, "animaxs_b200", "_build", "call_bench")
    try:
        res = subprocess.run([exe, "200"], capture_output=True, text=True, timeout=120)
        out["c_abi"] = json.loads(res.stdout) if res.returncode == 0 else {"error": res.stderr.strip()[-300:]}
    except Exception as e:  # noqa: BLE001 -- reported in the line, not fatal
        out["c_abi"] = {"error": str(e)}
    return out


def rows_f_figures(torch, ax, ex, device, stream, peak_sust, peak_burst):
    """The kernels around the DiT attention call, each timed on its own with
    a parity check against the oracle: the VAE's middle attention (1 head x 384
    over 4096 positions, inputs cycled over 16 images > L2), the LLM adapter's
    attention (512 tokens x 16 heads x 64, rms + RoPE), the fused q|k|v
    projection of a batch-8 block ([32768, 2048] -> [32768, 6144], q/k RMSNorm +
    3-D RoPE in the epilogue; parity on the first 256 rows) and the W4 weight
    decode ([6144, 2048], bit-exact).  kernel_us: CUDA events around each
    launch (animaxs_attn_kernel_timing); graph_us: whole calls replayed from a
    CUDA graph."""
    import numpy as np

    from oracle import attn_oracle as ora  # the checker
    from oracle import inputs
    res = {}

    def kernel_us(calls):
        ex.set_kernel_timing(True)
        with torch.cuda.stream(stream):
            calls()
        torch.cuda.synchronize()
        ex.set_kernel_timing(False)
        n_k, tot_ms, _ = ex.kernel_timing()
        return tot_ms * 1e3 / n_k

    def tflops(flops, us):
        t = flops / (us * 1e-6) / 1e12
        return {"tflops": t, "frac_sustained": t / peak_sust, "frac_burst": t / peak_burst}

    # VAE middle attention: the oracle on the first 512 query rows of image 0.
    case = inputs.vae_attention(seed=0)
    g = torch.Generator(device=device).manual_seed(4321)
    pool = [torch.from_numpy(np.concatenate([case.q, case.k, case.v], axis=0)).to(device)]
    pool += [torch.randn(3, VAE_POS, 1, VAE_CH, generator=g, device=device).half() for _ in range(VAE_POOL - 1)]
    vo = torch.empty(1, VAE_POS, 1, VAE_CH, dtype=torch.float16, device=device)

    def vae_calls():
        for x in pool:
            ex.attention(x[0:1], x[1:2], x[2:3], out=vo, stream=torch.cuda.current_stream(device))
        return len(pool)
    g_us = _graph_us(torch, stream, vae_calls)
    k_us = kernel_us(vae_calls)
    ex.attention(pool[0][0:1], pool[0][1:2], pool[0][2:3], out=vo, stream=stream)
    torch.cuda.synchronize()
    ex.synchronize(stream)
    rows = np.arange(512)
    mx, mn = ora.parity(vo.float().cpu().numpy()[:, :512], case.oracle(rows=rows))
    res["vae_hd384_4096"] = {"graph_us": g_us, "kernel_us": k_us, **tflops(VAE_FLOPS, k_us),
                             "max_abs": mx, "mean_abs": mn, "parity_ok": bool(mx <= 2e-3 and mn <= 2e-4),
                             "parity_rows": "512 of 4096 query rows"}

    # LLM adapter attention, head dim 64 (the oracle on every row).
    case = inputs.adapter_attention(seed=0)
    aq, ak, av = (torch.from_numpy(x).to(device) for x in (case.q, case.k, case.v))
    arope = torch.from_numpy(case.rope_table).to(device)
    ao = torch.empty_like(aq)

    def adapter_calls(reps=40):
        for _ in range(reps):
            ex.attention(aq, ak, av, out=ao, qk_norm="rms_rope", rope_table=arope,
                         stream=torch.cuda.current_stream(device))
        return reps
    g_us = _graph_us(torch, stream, adapter_calls)
    k_us = kernel_us(adapter_calls)
    torch.cuda.synchronize()
    ex.synchronize(stream)
    mx, mn = ora.parity(ao.float().cpu().numpy(), case.oracle())
    res["adapter_hd64_512x16"] = {"graph_us": g_us, "kernel_us": k_us, **tflops(case.flops(), k_us),
                                  "max_abs": mx, "mean_abs": mn, "parity_ok": bool(mx <= 2e-3 and mn <= 2e-4)}

    # Fused q|k|v projection of a batch-8 block.
    pj = ax.ProjectionExecutor(ex)
    gp = torch.Generator(device=device).manual_seed(2024)
    m = BATCH * S_SELF
    x = torch.randn(m, D_MODEL, generator=gp, device=device).half()
    w = (torch.randn(3 * D_MODEL, D_MODEL, generator=gp, device=device) / D_MODEL ** 0.5).half()
    qw = (1 + 0.1 * torch.randn(HD, generator=gp, device=device)).half()
    kw = (1 + 0.1 * torch.randn(HD, generator=gp, device=device)).half()
    tab = ora.dit_rope_table(1, 64, 64)
    rope = torch.from_numpy(tab).to(device)
    y = torch.empty(m, 3 * D_MODEL, dtype=torch.float16, device=device)

    def proj_calls(reps=4):
        for _ in range(reps):
            pj.qkv(x, w, y, q_cols=D_MODEL, k_cols=D_MODEL, qk_norm="rms_rope", q_norm_weight=qw,
                   k_norm_weight=kw, rope_table=rope, tokens=S_SELF, stream=torch.cuda.current_stream(device))
        return reps
    g_us = _graph_us(torch, stream, proj_calls)
    k_us = kernel_us(proj_calls)
    torch.cuda.synchronize()
    want = ora.qkv_norm_projection(x[:256].cpu().numpy(), w.cpu().numpy(), q_cols=D_MODEL, k_cols=D_MODEL,
                                   q_norm_weight=qw.cpu().numpy(), k_norm_weight=kw.cpu().numpy(),
                                   rope_table=tab[:256], tokens=256)  # rows 0-255 = tokens 0-255 of image 0
    want16 = ora.to_fp16_storage(want)
    err = np.abs(y[:256].float().cpu().numpy() - want16)
    bound_ok = bool((err <= 2e-3 + 2e-3 * np.abs(want16)).all()
                    and err.mean() <= 2.0 ** -13 * float(np.abs(want16).mean()) + 1e-6)
    res["proj_qkv_rms_rope3d_batch8"] = {"graph_us": g_us, "kernel_us": k_us,
                                         **tflops(2.0 * m * 3 * D_MODEL * D_MODEL, k_us),
                                         "max_abs": float(err.max()), "mean_abs": float(err.mean()),
                                         "parity_ok": bound_ok,
                                         "parity_rows": "first 256 rows; |d| <= 2e-3 + 2e-3 |oracle|, mean "
                                                        "<= 2^-13 mean |oracle|"}
    del x, y

    # W4 decode: roofline on 6 weights cycled (> L2), bit-exact on one.
    packed, scale, zero = inputs.quant_weight(4, 3 * D_MODEL, D_MODEL, 4)
    qw4 = ax.QuantizedWeight(*(torch.from_numpy(a).to(device) for a in (packed, scale, zero)), 4, D_MODEL)
    dec = pj.dequant(qw4, stream=stream)
    torch.cuda.synchronize()
    exact = bool(np.array_equal(dec.cpu().numpy().view(np.uint16),
                                ora.dequant_to_half(packed, scale, zero, bits=4, k=D_MODEL).view(np.uint16)))
    # (decode_roofline records its events on the stream its graph replays on)
    res["dequant_w4_6144x2048"] = {**decode_roofline(pj, 4, device, torch.cuda.current_stream(device)),
                                   "bit_exact": exact}
    return res


def cfg5_sharded(torch, dist, ex, rank, world, local_rank, steps=20, warmup=3):
    """Configuration 5 (16384-token self-attention, rms + 3-D RoPE 1x128x128,
    16 heads) with its heads sharded over the `world` ranks, every rank ending
    with the full [16384, 2048] output: the all-gather fused into the attention
    epilogue (NVLink stores) and one NCCL all-gather.  Per path: calls/s
    (max-over-ranks device time), TFLOP/s, and every rank's check of its
    gathered output -- bit-identical to its own single-GPU call at 64 sampled
    rows, and within the north-star tolerance of the reference-generated golden
    rows."""
    import numpy as np

    import animaxs_b200 as ax
    from animaxs_b200.sharded import HeadShardedAttention, PeerShardedAttention, share_unique_id
    from oracle import attn_oracle as ora  # the checker (golden rows)
    from oracle import inputs
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    case = inputs.dit_self(seed=0, grid=(1, 128, 128))
    q, k, v = (torch.from_numpy(x).to(device) for x in (case.q, case.k, case.v))
    rope = torch.from_numpy(case.rope_table).to(device)
    single = ex.attention(q, k, v, qk_norm="rms_rope", rope_table=rope, stream=stream)
    g = np.load(os.path.join(ROOT, "tests", "golden", "attn_configs.npz"))
    sample = torch.arange(0, 16384, 256, device=device)
    flops = 4.0 * 16384 * 16384 * HD * HEADS
    res = {}
    for gather in ("peer", "nccl"):
        if gather == "nccl":
            sh = HeadShardedAttention(ex, rank, world, share_unique_id())
            out = torch.empty_like(q)
            call = lambda: sh(q, k, v, out=out, qk_norm="rms_rope", rope_table=rope, stream=stream)  # noqa: E731
        else:
            sh = PeerShardedAttention(ex, rank, world, q.shape)
            call = lambda: sh(q, k, v, qk_norm="rms_rope", rope_table=rope, stream=stream)  # noqa: E731
        for _ in range(warmup):
            got = call()
        dist.barrier()
        torch.cuda.synchronize(device)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            got = call()
        t1.record(stream)
        dist.barrier()
        torch.cuda.synchronize(device)
        ex.synchronize(stream)
        el = torch.tensor([t0.elapsed_time(t1)], device=device)
        dist.all_reduce(el, op=dist.ReduceOp.MAX)
        exact = bool(torch.equal(got[:, sample], single[:, sample]))
        mx, mn = ora.parity(got[:, torch.from_numpy(g["cfg5_rows"]).to(device)].float().cpu().numpy(),
                            g["cfg5_out"])
        ok = torch.tensor([1 if exact else 0, 1 if (mx <= 2e-3 and mn <= 2e-4) else 0], device=device)
        oks = [torch.zeros_like(ok) for _ in range(world)]
        dist.all_gather(oks, ok)
        sh.close()
        dist.barrier()
        ms = float(el.item()) / steps
        res[gather] = {"calls_per_s": 1e3 / ms, "ms_per_call": ms, "tflops_total": flops / (ms * 1e-3) / 1e12,
                       "tflops_per_rank": flops / (ms * 1e-3) / 1e12 / world, "ranks": world,
                       "heads_per_rank": HEADS // world,
                       "bit_exact_vs_single_gpu_per_rank": [bool(o[0].item()) for o in oks],
                       "golden_rows_within_tolerance_per_rank": [bool(o[1].item()) for o in oks],
                       "how": "gather fused into the attention epilogue (NVLink stores)" if gather == "peer"
                       else "one NCCL all-gather + permute"}
    res["config"] = "S=16384, 16 heads x 128, rms + rope3d(1,128,128), heads sharded, full output on every rank"
    res["gpus_active"] = world
    return res


def run_cfg5(args, rank, world, local_rank):
    """Config 5: 16384-token DiT self-attention (rms + 3-D RoPE 1x128x128), 16
    heads sharded over the ranks; every rank ends with the full [16384, 2048]
    fp16 output.  The gather is fused into the attention kernel by default
    (`--gather peer`: every rank's epilogue stores its tiles into every rank's
    output over NVLink) or one NCCL all-gather (`--gather nccl`); one GPU
    needs no gather.  value = calls/s."""
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    from animaxs_b200.sharded import HeadShardedAttention, PeerShardedAttention, share_unique_id
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ex = ax.AttentionExecutor(local_rank)
    s_len = 16384
    g = torch.Generator(device=device).manual_seed(0)
    q, k, v = (torch.randn(1, s_len, HEADS, HD, generator=g, device=device).half() for _ in range(3))
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 128, 128).reshape(s_len, 64, 2, 2)).to(device)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(device)
    gather = args.gather if world > 1 else "none"
    if gather == "nccl":
        sh = HeadShardedAttention(ex, rank, world, share_unique_id())
    elif gather == "peer":
        sh = PeerShardedAttention(ex, rank, world, q.shape)
    else:
        class _Single:
            def __call__(self, q, k, v, out=None, **kw):
                return ex.attention(q, k, v, out=out, **kw)

            def close(self):
                pass
        sh = _Single()
    if gather == "peer":
        call = lambda: sh(q, k, v, qk_norm="rms_rope", rope_table=rope, stream=stream)  # noqa: E731
    else:
        call = lambda: sh(q, k, v, out=out, qk_norm="rms_rope", rope_table=rope, stream=stream)  # noqa: E731

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        call()
    barrier()
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        call()
    t1.record(stream)
    barrier()
    clocks = sampler.stop()
    ex.synchronize(stream)
    el = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([el], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    flops = 4.0 * s_len * s_len * HD * HEADS
    sh.close()
    if rank != 0:
        return
    peak_burst, peak_sust, _, peak_kind = peaks()
    tf = flops * args.steps / (el / 1e3) / 1e12
    how = {"peer": "gather fused into the attention epilogue (NVLink stores)",
           "nccl": "NCCL all-gather", "none": "one GPU, no gather"}[gather]
    print(json.dumps({
        "metric": "config-5 DiT self-attention, 16384 tokens, heads sharded, every rank ends with the "
                  "full output",
        "value": args.steps / (el / 1e3), "unit": "calls/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": "config5: S=16384, 16 heads x 128, rms + rope3d(1,128,128)",
                   "parallelism": f"heads/{world}", "gather": how},
        "tflops_total": tf, "tflops_per_gpu": tf / world,
        "frac_of_sustained_peak_per_gpu": tf / world / peak_sust, "peak_kind": peak_kind,
        "clocks": clocks}), flush=True)


VAE_POS = 64 * 64
VAE_CH = 384
VAE_FLOPS = 4.0 * VAE_POS * VAE_POS * VAE_CH       # 25.8 GFLOP per image
VAE_POOL = 16                                      # 16 x 9.4 MiB of split QKV (> 126 MB L2)


def run_vae(args, rank, world, local_rank):
    """The VAE decoder's middle attention (VAEDecoder.swift:351-410): one head
    of 384 channels over the 64x64 latent positions, one image per call, in the
    reference's call form (AttentionExecutor.encode on a split [3 x positions,
    384] QKV buffer with byte offsets, head-major).  Images are independent:
    each rank decodes its own (weak scaling).  value = images/s over all ranks;
    inputs rotate through a pool larger than L2."""
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ex = ax.AttentionExecutor(local_rank)
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(4321 + rank)
    pool = [torch.randn(3 * VAE_POS, VAE_CH, generator=g, device=device).half() for _ in range(VAE_POOL)]
    out = torch.empty(VAE_POS, VAE_CH, dtype=torch.float16, device=device)
    kw = dict(heads=1, query_count=VAE_POS, key_count=VAE_POS, head_dim=VAE_CH,
              key_offset=VAE_POS * VAE_CH * 2, value_offset=2 * VAE_POS * VAE_CH * 2)

    # The timed loop calls the same C-ABI forward through the cached strided
    # descriptor ([1, positions, 1, 384] views of the split buffer: the same
    # descriptor contents as the head-major encode call, without rebuilding it
    # on the host every call); the e2e leg below uses encode itself.
    views = [tuple(x[j * VAE_POS:(j + 1) * VAE_POS].view(1, VAE_POS, 1, VAE_CH) for j in range(3))
             for x in pool]
    out_v = out.view(1, VAE_POS, 1, VAE_CH)

    def call(i):
        q, k, v = views[i % VAE_POOL]
        ex.attention(q, k, v, out=out_v, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    calls_per_step = 4096  # ~0.16 s per step: long enough for the clock sampler
    for i in range(args.warmup * calls_per_step):
        call(i)
    barrier()
    ex.synchronize(stream)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    ex.set_kernel_timing(True)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps * calls_per_step):
        call(i)
    t1.record(stream)
    barrier()
    clocks = sampler.stop()
    ex.set_kernel_timing(False)
    n_kern, kern_total_ms, kern_max_ms = ex.kernel_timing()
    ex.synchronize(stream)
    el = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([el], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    images = args.steps * calls_per_step * world

    e2e = None
    if not args.no_e2e:
        # Pinned host split-QKV in, output back to the host, every image.
        hg = torch.Generator().manual_seed(77)
        host = [torch.randn(3 * VAE_POS, VAE_CH, generator=hg).half().pin_memory() for _ in range(4)]
        host_out = torch.empty(VAE_POS, VAE_CH, dtype=torch.float16).pin_memory()
        dev_in = torch.empty(3 * VAE_POS, VAE_CH, dtype=torch.float16, device=device)
        n_e2e = max(16, args.steps * 8)
        for i in range(4):
            dev_in.copy_(host[i], non_blocking=True)
            ex.encode(stream, dev_in, dev_in, dev_in, out, **kw)
            host_out.copy_(out, non_blocking=True)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n_e2e):
            dev_in.copy_(host[i % 4], non_blocking=True)
            ex.encode(stream, dev_in, dev_in, dev_in, out, **kw)
            host_out.copy_(out, non_blocking=True)
        e1.record(stream)
        barrier()
        ee = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ee], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ee = float(t.item())
        e2e = {"value": n_e2e * world / (ee / 1e3), "unit": "img/s",
               "h2d_bytes_per_step": 3 * VAE_POS * VAE_CH * 2, "d2h_bytes_per_step": VAE_POS * VAE_CH * 2,
               "steps": n_e2e, "path": "AttentionExecutor.encode -> animaxs_attn_forward (host QKV in, output out)"}
    if rank != 0:
        return
    peak_burst, peak_sust, _, peak_kind = peaks()
    avg_kern = kern_total_ms / n_kern if n_kern else float("nan")
    achieved = VAE_FLOPS / (avg_kern / 1e3) / 1e12
    line = {
        "metric": "VAE middle attention throughput (1 head x 384 over the 64x64 latent, one image per call)",
        "value": images / (el / 1e3), "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": f"vae: {calls_per_step} images per step, 4096 positions x 384, heads 1, "
                               "split QKV buffer with byte offsets (the reference's call)",
                   "parallelism": f"images x{world}",
                   "l2": f"inputs cycled over a {VAE_POOL * 9} MiB resident pool (> 126 MB L2)"},
        "roofline": {"kernel": "attn_wide_sm100_kernel<384> (4096 x 4096 x 384, keys split over a cluster)",
                     "bound": "tensor", "achieved": achieved, "peak": peak_sust, "unit": "TFLOP/s",
                     "frac": achieved / peak_sust, "peak_kind": f"{peak_kind} bf16 dense, sustained",
                     "frac_of_burst_peak": achieved / peak_burst, "flops_per_launch": VAE_FLOPS,
                     "avg_launch_ms": avg_kern, "max_launch_ms": kern_max_ms, "launches_timed": n_kern,
                     "traffic": None, "algorithmic_bytes": 4 * VAE_POS * VAE_CH * 2},
        "clocks": clocks,
        "gpu_launches": args.steps * calls_per_step,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        from oracle import attn_oracle as ora  # the checker, used here only as the CPU baseline
        import numpy as np
        qkv = pool[0].float().cpu().numpy().reshape(3, 1, VAE_POS, 1, VAE_CH)
        rows = np.arange(512)
        t_c = time.perf_counter()
        ora.attention(qkv[0], qkv[1], qkv[2], rows=rows)
        t_c = time.perf_counter() - t_c
        line["cpu_baseline"] = {"value": 1.0 / (t_c * VAE_POS / len(rows)), "unit": "img/s",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": "512 of 4096 query rows of one image, numpy fp32 oracle, x8"}
    print(json.dumps(line), flush=True)


D_MODEL = HEADS * HD                               # 2048
QKV_FLOPS = 2.0 * S_SELF * 3 * D_MODEL * D_MODEL    # fused q|k|v projection, per image
PROJ_FLOPS = 2.0 * S_SELF * D_MODEL * D_MODEL       # one 2048 x 2048 projection, per image
BLOCK_PROJ_FLOPS = QKV_FLOPS + 3 * PROJ_FLOPS       # self q|k|v, self out, cross q, cross out


def run_proj(args, rank, world, local_rank):
    """The projections on either side of DiT attention, fused
    (DiTBlockExecutor.swift:1097-1131, 1223-1236): per block, for a batch of 8
    images -- self q|k|v with q/k RMSNorm + 3-D RoPE in the epilogue, the self
    out-projection + gated residual (fp32 residual += fp16 branch x gate), the
    cross q projection + RMSNorm and the cross out-projection + gated residual
    (the cross K/V come from the reference's CrossKVCache and are not
    re-projected).  One step = 224 blocks (28 blocks x 8 Euler steps) of one
    batch, like config 4; value = images/s; random-init weights of the DiT's
    shapes (2048 -> 6144 / 2048)."""
    import torch
    import torch.distributed as dist

    import animaxs_b200 as ax
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ex = ax.AttentionExecutor(local_rank)
    pj = ax.ProjectionExecutor(ex)
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(2024 + rank)
    m = BATCH * S_SELF
    xs = [torch.randn(m, D_MODEL, generator=g, device=device).half() for _ in range(POOL_BLOCKS)]
    bits = {"fp16": 16, "w8": 8, "w4": 4}[args.weights]

    def make_w(rows):
        w = (torch.randn(rows, D_MODEL, generator=g, device=device) / D_MODEL ** 0.5).half()
        return w if bits == 16 else quantize_groups(w, bits)

    w_qkv = make_w(3 * D_MODEL)
    w_so, w_cq, w_co = (make_w(D_MODEL) for _ in range(3))
    qw = (1 + 0.1 * torch.randn(HD, generator=g, device=device)).half()
    kw = (1 + 0.1 * torch.randn(HD, generator=g, device=device)).half()
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 64, 64).reshape(S_SELF, 64, 2, 2)).to(device)
    residual = torch.zeros(m, D_MODEL, device=device)
    gates = 0.1 * torch.randn(2, BATCH, D_MODEL, generator=g, device=device)
    qkv = torch.empty(m, 3 * D_MODEL, dtype=torch.float16, device=device)
    q_cross = torch.empty(m, D_MODEL, dtype=torch.float16, device=device)

    def block(i):
        x = xs[i % POOL_BLOCKS]
        pj.qkv(x, w_qkv, qkv, q_cols=D_MODEL, k_cols=D_MODEL, qk_norm="rms_rope", q_norm_weight=qw,
               k_norm_weight=kw, rope_table=rope, tokens=S_SELF, stream=stream)
        pj.out_gate_add(x, w_so, residual, gates[0], tokens=S_SELF, stream=stream)
        pj.qkv(x, w_cq, q_cross, q_cols=D_MODEL, k_cols=0, qk_norm="rms", q_norm_weight=qw, stream=stream)
        pj.out_gate_add(x, w_co, residual, gates[1], tokens=S_SELF, stream=stream)

    def step():
        for i in range(CALLS_PER_IMAGE):
            block(i)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        step()
    barrier()
    ex.synchronize(stream)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    barrier()
    ex.set_kernel_timing(True)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    clocks = sampler.stop()
    ex.set_kernel_timing(False)
    n_kern, kern_total_ms, kern_max_ms = ex.kernel_timing()
    ex.synchronize(stream)
    el = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([el], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    decode = decode_roofline(pj, bits, device, stream) if bits != 16 else None
    if rank != 0:
        return
    peak_burst, peak_sust, _, peak_kind = peaks()
    images = args.steps * world * BATCH
    flops = args.steps * CALLS_PER_IMAGE * BATCH * BLOCK_PROJ_FLOPS
    avg_kern = kern_total_ms / n_kern if n_kern else float("nan")
    achieved = BATCH * BLOCK_PROJ_FLOPS / 4 / (avg_kern / 1e3) / 1e12   # mean over the 4 launches
    line = {
        "metric": "DiT attention projections throughput, 8-step 1024x1024 workload (fused q|k|v "
                  "rms+rope3d, out-proj + gated residual, cross q rms, cross out-proj + gated residual)",
        "value": images / (el / 1e3), "unit": "img/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic, random-init weights",
        "config": {"workload": "proj: 224 blocks x batch 8, x [32768, 2048] -> q|k|v [32768, 6144] and 3 x "
                               "[32768, 2048] projections", "parallelism": f"batch-shard x{world}",
                   "weights": args.weights if bits == 16 else
                   f"{args.weights}: group-64 codes decoded to fp16 on every call, then the GEMM",
                   "l2": f"x cycled over {POOL_BLOCKS} x 128 MiB (> 126 MB L2)"},
        "tflops_per_gpu": flops / (el / 1e3) / 1e12,
        "roofline": {"kernel": "proj_sm100_kernel (CTA-pair tcgen05 GEMM, fused epilogues; mean of the 4 "
                               "launches of a block)",
                     "bound": "tensor", "achieved": achieved, "peak": peak_sust, "unit": "TFLOP/s",
                     "frac": achieved / peak_sust, "peak_kind": f"{peak_kind} bf16 dense, sustained",
                     "frac_of_burst_peak": achieved / peak_burst, "avg_launch_ms": avg_kern,
                     "max_launch_ms": kern_max_ms, "launches_timed": n_kern, "traffic": None},
        "clocks": clocks,
        # 4 GEMMs + the RoPE-table re-layout (+ 4 weight decodes)
        "gpu_launches": args.steps * CALLS_PER_IMAGE * (5 if bits == 16 else 9),
        "e2e": None,
    }
    if decode is not None:
        line["decode_roofline"] = decode
    print(json.dumps(line), flush=True)


def quantize_groups(w, bits):
    """Group-64 affine codes of an fp16 [n, k] weight on the device (the
    reference packer's plain range, scripts/pack_anima.py:217-262): scale =
    (max - min) / qmax, zero = min, q = rint((w - zero) / scale)."""
    import torch

    import animaxs_b200 as ax
    n, k = w.shape
    qmax = 15.0 if bits == 4 else 255.0
    grp = w.float().view(n, k // 64, 64)
    lo = grp.amin(dim=2)
    span = grp.amax(dim=2) - lo
    scale = torch.where(span >= 1e-8, span / qmax, torch.ones_like(span)).half()
    zero = lo.half()
    q = torch.clamp(torch.round((grp - zero.float()[..., None]) / scale.float()[..., None]), 0, qmax)
    q = q.to(torch.uint8).view(n, k)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous() if bits == 4 else q.contiguous()
    return ax.QuantizedWeight(packed, scale.contiguous(), zero.contiguous(), bits, k)


def decode_roofline(pj, bits, device, stream, pool=6, reps=5):
    """The weight decode alone (dequant_aligned_kernel): the DiT q|k|v weight shape
    [6144, 2048], cycled over `pool` weights whose fp16 outputs total > L2.
    Algorithmic bytes per launch = codes + scale + zero read + fp16 written."""
    import torch
    n, k = 3 * D_MODEL, D_MODEL
    g = torch.Generator(device=device).manual_seed(77)
    ws = [quantize_groups(torch.randn(n, k, generator=g, device=device).half(), bits) for _ in range(pool)]
    outs = [torch.empty(n, k, dtype=torch.float16, device=device) for _ in range(pool)]
    for w, o in zip(ws, outs):
        pj.dequant(w, o, stream=stream)
    torch.cuda.synchronize(device)
    # The launches are replayed from a CUDA graph so that the events time the
    # kernels back to back, not the host's per-call overhead.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            for w, o in zip(ws, outs):
                pj.dequant(w, o)
    graph.replay()
    torch.cuda.synchronize(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(device)
    per_launch_ms = t0.elapsed_time(t1) / (reps * pool)
    del graph
    nbytes = n * k * bits // 8 + 2 * n * (k // 64) * 2 + n * k * 2
    hbm = peaks()[2]
    achieved = nbytes / (per_launch_ms / 1e3) / 1e9
    return {"kernel": f"dequant_aligned_kernel<{bits}> ([6144, 2048] weight, {pool} weights cycled, "
                      f"{pool * n * k * 2 / 2**20:.0f} MiB of fp16 outputs > L2, {reps * pool} launches "
                      "replayed from a CUDA graph)",
            "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
            "bytes_per_launch": nbytes, "avg_launch_ms": per_launch_ms}


def profile_kernel(args):
    import torch

    import animaxs_b200 as ax
    ex = ax.AttentionExecutor(0)
    if args.workload == "proj":
        # warmup + steps fused q|k|v (rms + rope3d) projections of a batch of 4 images
        pj = ax.ProjectionExecutor(ex)
        g = torch.Generator(device="cuda").manual_seed(5)
        m = 4 * S_SELF
        x = torch.randn(m, D_MODEL, generator=g, device="cuda").half()
        w = (torch.randn(3 * D_MODEL, D_MODEL, generator=g, device="cuda") / D_MODEL ** 0.5).half()
        if args.weights != "fp16":   # each call then decodes the weight (dequant_kernel) first
            w = quantize_groups(w, 4 if args.weights == "w4" else 8)
        out = torch.empty(m, 3 * D_MODEL, dtype=torch.float16, device="cuda")
        nw = torch.ones(HD, dtype=torch.float16, device="cuda")
        rope = torch.from_numpy(ax.DitRoPE.generate(1, 64, 64).reshape(S_SELF, 64, 2, 2)).cuda()
        for _ in range(args.warmup + args.steps):
            pj.qkv(x, w, out, q_cols=D_MODEL, k_cols=D_MODEL, q_norm_weight=nw, k_norm_weight=nw,
                   rope_table=rope, tokens=S_SELF)
        torch.cuda.synchronize()
        ex.synchronize()
        print("profile-kernel done", flush=True)
        return
    if args.workload == "vae":
        # warmup + steps VAE middle-attention calls on distinct images (> L2 in total)
        g = torch.Generator(device="cuda").manual_seed(5)
        pool = [torch.randn(3 * VAE_POS, VAE_CH, generator=g, device="cuda").half() for _ in range(VAE_POOL)]
        out = torch.empty(VAE_POS, VAE_CH, dtype=torch.float16, device="cuda")
        stream = torch.cuda.current_stream()
        for i in range(args.warmup + args.steps):
            qkv = pool[i % VAE_POOL]
            ex.encode(stream, qkv, qkv, qkv, out, heads=1, query_count=VAE_POS, key_count=VAE_POS,
                      head_dim=VAE_CH, key_offset=VAE_POS * VAE_CH * 2, value_offset=2 * VAE_POS * VAE_CH * 2)
        torch.cuda.synchronize()
        ex.synchronize()
        print("profile-kernel done", flush=True)
        return
    if args.workload == "cfg1":
        # warmup + steps configuration-1 calls (1024 tokens x 16 heads, batch 1: a
        # single-tile launch, attn_s3_sm100_kernel; the inputs stay in L2 as in
        # the configuration itself)
        g = torch.Generator(device="cuda").manual_seed(5)
        q, k, v = (torch.randn(1, 1024, HEADS, HD, generator=g, device="cuda").half() for _ in range(3))
        out = torch.empty_like(q)
        rope = torch.from_numpy(ax.DitRoPE.generate(1, 32, 32).reshape(1024, 64, 2, 2)).cuda()
        for _ in range(args.warmup + args.steps):
            ex.attention(q, k, v, out=out, qk_norm="rms_rope", rope_table=rope)
        torch.cuda.synchronize()
        ex.synchronize()
        print("profile-kernel done", flush=True)
        return
    g = torch.Generator(device="cuda").manual_seed(5)
    shape = (4, S_SELF, HEADS, HD)
    q, k, v = (torch.randn(*shape, generator=g, device="cuda").half() for _ in range(3))
    out = torch.empty_like(q)
    rope = torch.from_numpy(ax.DitRoPE.generate(1, 64, 64).reshape(S_SELF, 64, 2, 2)).cuda()
    for _ in range(args.warmup + args.steps):
        ex.attention(q, k, v, out=out, qk_norm="rms_rope", rope_table=rope)
    torch.cuda.synchronize()
    ex.synchronize()
    print("profile-kernel done", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="animaxs", choices=["animaxs", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the configuration 1/2/3/5 figures of the N=1 line")
    ap.add_argument("--no-cfg5", action="store_true",
                    help="skip the head-sharded configuration-5 leg of an N>1 line")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="config-5 gather across ranks: fused NVLink stores or NCCL all-gather")
    ap.add_argument("--weights", default="fp16", choices=["fp16", "w8", "w4"],
                    help="projection weight storage for --workload proj")
    ap.add_argument("--workload", default="cfg4", choices=["cfg4", "cfg5", "vae", "proj", "cfg1"],
                    help="cfg4 (default): the 8-step DiT workload, batch-sharded; cfg5: the "
                         "16384-token self-attention, heads sharded + one NCCL all-gather; vae: "
                         "the VAE decoder's middle attention (one head of 384), images per rank; "
                         "proj: the fused projections around DiT attention; cfg1 (with "
                         "--profile-kernel only): configuration 1's calls")
    ap.add_argument("--profile-kernel", action="store_true",
                    help="only run the fused rms+rope3d self-attention (prologue + flash kernel) "
                         "on a batch-4 4096-token case (192 MiB of inputs, > L2), or with "
                         "--workload vae warmup+steps VAE middle-attention calls: the small "
                         "cases for ncu captures")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.profile_kernel:
        profile_kernel(args)
        return
    if args.workload == "cfg1":
        ap.error("--workload cfg1 is a --profile-kernel case (configuration 1 is timed in the secondary block)")
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "cfg5":
            run_cfg5(args, rank, world, local_rank)
        elif args.workload == "vae":
            run_vae(args, rank, world, local_rank)
        elif args.workload == "proj":
            run_proj(args, rank, world, local_rank)
        else:
            run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
