"""Benchmark of the BC_mamba event hot path on B200: fwd+bwd events/s.

Default workload: BASELINE.json configs[4] (``--config c4``), the block stack
the metric is quoted on: 4 event blocks in the ResidualPreNorm pattern
(v <- 0.95*v + block(v); each block thresholds its own input membrane at the
target density, extracts events, gathers x_conv, runs the depthwise scan,
restores to dense and projects back with out_proj), global B = 128 sequences
of L = 4000, D = 256, N = 16, fp32, rho = 10 % i.i.d. spikes, sharded by batch
rows over the ranks (strong scaling: every world size processes the same
global rows, generated per row from the row's own seed).  One step = forward
and backward of the whole stack, then one all-reduce per block of that
block's parameter gradients, launched from autograd as soon as the block's
backward has produced them.

Single-block configs (``--config c1`` .. ``c3``, and c0) run one block of the
event path per GPU with a fixed upstream gradient (weak scaling).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
                    [--config c4] [--rho 0.1] [--spikes iid|markov] [--sweep]

Prints ONE JSON line on rank 0 (``--sweep``: one line per density and spike
kind of configs[4]).  `value` = events of all ranks / max-over-ranks device
time per step with inputs resident in HBM; `e2e` = the same with pinned-host
inputs copied in and parameter gradients copied out inside every timed step.
L2 is flushed (256 MiB memset) before every timed step, outside its window;
the step's inputs are larger than L2 as well.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fwd+bwd events/s and % HBM roofline"
UNIT = "events/s"
SWEEP = [(rho, kind) for kind in ("iid", "markov") for rho in (0.05, 0.10, 0.25, 0.50)]


# ---------------------------------------------------------------- helpers ----
def measured_peak_gbs():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        """Start sampling and wait for the first sample (nvidia-smi start-up
        must not overlap the timed region)."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:
                time.sleep(0.05)
            time.sleep(0.2)
            self.skip = len(self.lines)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "skip", 0):]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# the API stages of one block (interface.cuda_stage names) -> op keys
STAGE_OPS = {
    "routing_index_extraction": "extract", "sparse_scan_forward": "scan_fwd",
    "dense_restoration_forward": "restore_fwd", "restore_backward": "restore_bwd",
    "sparse_scan_backward": "scan_bwd", "gather_scatter_backward": "gather_bwd",
}
def kernels_per_block(cfg, rows: int, sm_count: int, stack: bool) -> int:
    """Kernels of ours one block launches per step (forward and backward),
    from the launch list of the bench workload: extraction 3 (threshold +
    count, count scan, fill of the expanded stream with the gather of
    x_conv), restore forward 2 (event bitmap, word sweep), restore backward 1,
    gather backward 1 (row writer), in the stack also the parameter
    transforms 1 + 1, and the scan: staged dispatch 3 forward (decay table,
    row order, scan) + 4 backward (the same and the partial-sum reduction),
    event-parallel dispatch 2 + 3 (no row order).  The event-parallel kernels
    run where the staged ones do not divide the rows of a feature into whole
    warps, or where the staged backward would have fewer than 5 warps per SM
    (the library's dispatch rule, dstate <= 64)."""
    NP = 8 if cfg.N <= 8 else 16 if cfg.N <= 16 else 32 if cfg.N <= 32 else 64
    cpw_bwd = 128 // NP if NP <= 16 else 256 // NP      # channels per warp, staged backward
    cpw_fwd = 64 // NP                                  # and forward
    staged_ok = rows % cpw_bwd == 0 and rows % cpw_fwd == 0
    mode = os.environ.get("BCM_SCAN_SEG", "1")   # the library's dispatch override (0 never, 2 always)
    if mode == "0":
        seg = False
    elif mode == "1":
        seg = not staged_ok or rows * cfg.D // cpw_bwd < 5 * sm_count
    else:
        seg = True
    return 7 + (2 if stack else 0) + (5 if seg else 7)

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per stage and
# block from one ncu capture, summed over the stage's kernels (summaries in
# profiles/, one per workload).  Writes that stay in the 126 MB L2 when a
# kernel ends are not counted.  Re-measured whenever a kernel changes.
NCU_TRAFFIC = {
    ("c1", None): {"extract": 109.04e6, "scan_fwd": 27.45e6, "restore_fwd": 38.20e6, "restore_bwd": 70.59e6,
                   "scan_bwd": 70.54e6, "gather_bwd": 37.33e6},
}
# The same for ONE block of the configs[4] stack (B = 128, rho = 0.1 i.i.d.,
# 13.1 M events; profiles/dram_traffic_c4_block.txt); the stack's blocks carry
# the same event count, so a step moves `blocks` times this.
NCU_TRAFFIC_C4_BLOCK = {"extract": 966.0e6, "scan_fwd": 222.6e6, "restore_fwd": 653.7e6, "restore_bwd": 669.6e6,
                        "scan_bwd": 327.6e6, "gather_bwd": 574.3e6}


def algorithmic_bytes(cfg, E, NC, n_chunks):
    """Bytes each API call of one block must move once (inputs read once,
    outputs written once), per op, for one fwd+bwd."""
    s = torch.tensor([], dtype=cfg.dtype).element_size()
    sv = 4
    NCb = NC // cfg.expand
    L, N = cfg.L, cfg.N
    return {
        "extract": NCb * L * sv + 12 * E + 4 * NC + 2 * s * E,
        "scan_fwd": (2 * s + 4) * E + 8 * N * NC * n_chunks,
        "restore_fwd": (4 + s) * E + NC * L * s,
        "restore_bwd": NC * L * s + 8 * E,
        "scan_bwd": (3 * s + 4) * E + 8 * N * NC * n_chunks,
        "gather_bwd": NC * L * s + (s + 8) * E,
    }


def _dist():
    return torch.distributed if torch.distributed.is_available() and torch.distributed.is_initialized() else None


def _max_over_ranks(x: float, dev) -> float:
    d = _dist()
    if d is None:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    d.all_reduce(t, op=d.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, dev) -> float:
    d = _dist()
    if d is None:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    d.all_reduce(t)
    return float(t.item())


def _barrier():
    d = _dist()
    if d is not None:
        d.barrier()


def time_steps(step, zero, flush, steps):
    """K steps bracketed by CUDA events, each after an L2 flush outside its
    window; returns the summed device time (ms)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    _barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        zero()
        flush.zero_()
        starts[i].record()
        step()
        ends[i].record()
    torch.cuda.synchronize()
    _barrier()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends))


def stage_times(step, zero, flush, steps):
    """The same K steps again with every API stage bracketed by CUDA events
    on its launching stream (a separate pass: recording the events costs host
    time the timed steps should not carry).  Returns ms per op and step."""
    from bc_mamba_b200 import interface as itf

    with itf.stage_timing() as log:
        for _ in range(steps):
            zero()
            flush.zero_()
            step()
    torch.cuda.synchronize()
    per_op = {k: 0.0 for k in STAGE_OPS.values()}
    other = {}
    for name, s_ev, e_ev in log:
        ms = s_ev.elapsed_time(e_ev) / steps
        if name in STAGE_OPS:
            per_op[STAGE_OPS[name]] += ms
        else:
            other[name] = other.get(name, 0.0) + ms
    stage_times.other = other
    return per_op


def time_e2e(dev, host_inputs, run_on, grads, steps):
    """Pinned host inputs copied in on a copy stream (step i+1's inputs into
    the other half of a double buffer while step i computes) and the
    parameter gradients copied back every step; the window runs from the
    first copy to the last read-back.  Returns (ms per step, h2d, d2h bytes)."""
    h_in = [t.cpu().pin_memory() for t in host_inputs]
    h_grads = [torch.empty(g.shape, dtype=g.dtype).pin_memory() for g in grads()]
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = sum(t.numel() * t.element_size() for t in h_grads)
    bufs = [[torch.empty_like(t, device=dev) for t in h_in] for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    comp = torch.cuda.current_stream(dev)

    def h2d_into(b, wait_free):
        with torch.cuda.stream(copy_stream):
            if wait_free:
                copy_stream.wait_event(free[b])
            for d_t, h_t in zip(bufs[b], h_in):
                d_t.copy_(h_t, non_blocking=True)
            ready[b].record(copy_stream)

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier()
    torch.cuda.synchronize()
    e0.record(comp)
    copy_stream.wait_stream(comp)
    h2d_into(0, False)
    for i in range(steps):
        b = i % 2
        if i + 1 < steps:
            h2d_into(1 - b, i >= 1)          # the other half was last used by step i-1
        comp.wait_event(ready[b])
        run_on(bufs[b])
        for hg, g in zip(h_grads, grads()):
            hg.copy_(g, non_blocking=True)
        free[b].record(comp)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), dev) / steps
    _barrier()
    return ms, h2d, d2h


def clock_sampler(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    idx = int(vis.split(",")[local]) if vis else torch.cuda.current_device()
    return ClockSampler(idx).start()


def roofline_fields(per_op, alg, traffic):
    peak, peak_kind = measured_peak_gbs()
    dominant = max(per_op, key=lambda k: per_op[k])
    dom_ms = per_op[dominant]
    achieved = alg[dominant] / (dom_ms * 1e-3) / 1e9
    total_alg = sum(alg.values())
    kernel_ms = sum(per_op.values())
    roof = {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic.get(dominant) if traffic else None,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6650 GB/s",
            "algorithmic_bytes": alg[dominant], "ms": dom_ms}
    pipe = {"algorithmic_bytes": total_alg, "kernel_ms_sum": kernel_ms,
            "achieved_gbs_kernels": total_alg / (kernel_ms * 1e-3) / 1e9,
            "frac_kernels": total_alg / (kernel_ms * 1e-3) / 1e9 / peak}
    per_frac = {k: alg[k] / (per_op[k] * 1e-3) / 1e9 / peak for k in per_op if per_op[k] > 0}
    return roof, pipe, per_frac, peak


# ------------------------------------------------------ GPU arm: stack ----
def run_stack(args, cfg, rank, world, local, dev):
    """the block stack, strong-scaled over the ranks."""
    from bc_mamba_b200 import dp
    from bc_mamba_b200 import stack as stk

    b0, b1 = dp.shard_range(cfg.B, rank, world)
    inp = stk.stack_inputs(cfg, range(b0, b1), dev)
    model = stk.EventStack(cfg, dev, seed=cfg.seed, proj_tf32=True)
    thr = stk.calibrate_thresholds(model, inp["v0"], inp["x_conv"])
    # one gradient bucket per block, all-reduced from autograd as soon as the
    # block's backward has produced every one of its parameter gradients
    buckets = [dp.GradBucket(p.tensors(), overlap=True) for p in model.params] if world > 1 else None
    x_leaves = [x.detach().clone().requires_grad_(True) for x in inp["x_conv"]]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    info = {}

    def zero():
        if buckets is not None:
            for b in buckets:
                b.zero_grad()
        else:
            for p in model.all_params():
                p.grad = None
        for x in x_leaves:
            x.grad = None

    def run(v0, xs, dout):
        v, ev = model.forward(v0, xs, thr)
        v.backward(dout)
        if buckets is not None:
            for b in buckets:
                b.finish()
        info["ev"] = ev

    def step():
        run(inp["v0"], x_leaves, inp["dout"])

    for _ in range(args.warmup):
        zero()
        step()
    torch.cuda.synchronize()
    ev = info["ev"]
    E_local = sum(e for e, _ in ev)

    clocks = clock_sampler(local)
    t_ms = time_steps(step, zero, flush, args.steps)
    clk = clocks.stop()
    ms_per_step = _max_over_ranks(t_ms, dev) / args.steps
    E_all = _sum_over_ranks(E_local, dev)
    value = E_all / (ms_per_step * 1e-3)
    per_op = stage_times(step, zero, flush, args.steps)
    hot_ms = sum(per_op.values())

    e2e = None
    if not args.no_e2e:
        names = ["v0"] + [f"x{l}" for l in range(cfg.blocks)] + ["dout"]
        host = [inp["v0"]] + list(inp["x_conv"]) + [inp["dout"]]

        def run_on(bufs):
            zero()
            run(bufs[0], [b.detach().requires_grad_(True) for b in bufs[1:-1]], bufs[-1])

        e_ms, h2d, d2h = time_e2e(dev, host, run_on, lambda: [p.grad for p in model.all_params()], args.steps)
        e2e = {"value": E_all / (e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms, "inputs": names,
               "copies": "pinned host -> device on a copy stream, step i+1's inputs overlapping step i; "
                         "every parameter gradient read back each step"}

    NC = (b1 - b0) * cfg.D
    alg = {k: 0.0 for k in STAGE_OPS.values()}
    for e, mx in ev:
        for k, v in algorithmic_bytes(cfg, e, NC, max(1, (mx + 2047) // 2048)).items():
            alg[k] += v
    traffic = None
    if cfg.name == "c4_stack" and world == 1 and (cfg.rho, cfg.spikes) == (0.1, "iid"):
        traffic = {k: v * cfg.blocks for k, v in NCU_TRAFFIC_C4_BLOCK.items()}
    roof, pipe, per_frac, peak = roofline_fields(per_op, alg, traffic)
    pipe["achieved_gbs_step"] = sum(alg.values()) / (ms_per_step * 1e-3) / 1e9
    pipe["frac_step"] = pipe["achieved_gbs_step"] / peak
    dens = [e / ((b1 - b0) * cfg.L * cfg.D) for e, _ in ev]
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": "synthetic (seeded per global batch row; BASELINE.json configs[4] shapes and distributions)",
        "config": {"workload": f"{cfg.name}: {cfg.blocks} blocks, global B={cfg.B} (B/{world}={b1 - b0} per GPU), "
                               f"D={cfg.D} N={cfg.N} L={cfg.L} rho={cfg.rho} {cfg.spikes} expand={cfg.expand}",
                   "global_batch": cfg.B, "seq_len": cfg.L, "blocks": cfg.blocks,
                   "events_per_step_all_ranks": E_all, "events_per_block_rank0": [e for e, _ in ev],
                   "max_seqlen_per_block_rank0": [mx for _, mx in ev],
                   "density_per_block_rank0": dens,
                   "thresholds": "per feature, calibrated per block to the (1 - rho) quantile of the "
                                 "block's input membrane (range per block: "
                                 + ", ".join(f"[{float(t.min()):.3g}, {float(t.max()):.3g}]" for t in thr) + ")",
                   "parallelism": f"dp{world} (batch rows sharded, one gradient all-reduce per block)",
                   "l2": "256 MiB memset flush before every timed step, outside its window; inputs > L2"},
        "e2e": e2e,
        "roofline": roof,
        "pipeline_roofline": pipe,
        "hot_path": {"ms_per_step": hot_ms, "events_per_s": E_all / (hot_ms * 1e-3),
                     "other_ms_per_step": ms_per_step - hot_ms,
                     "other_timed_ms": getattr(stage_times, "other", {}),
                     "other": "out_proj GEMMs (TF32 tensor cores, outside the event path), membrane "
                              "updates, gradient all-reduces, launch gaps"},
        "per_op_ms": per_op,
        "per_op_frac_hbm": per_frac,
        "clocks": clk,
        "gpu_launches": cfg.blocks * args.steps * kernels_per_block(
            cfg, b1 - b0, torch.cuda.get_device_properties(dev).multi_processor_count, stack=True),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if buckets is not None:
        del buckets
    return line


# ------------------------------------------------ GPU arm: single block ----
def run_block(args, cfg, rank, world, local, dev):
    """One block of the event path per GPU (configs[0..3]; weak scaling)."""
    from bc_mamba_b200 import dp
    from bc_mamba_b200 import interface as itf
    from bc_mamba_b200.workloads import make_inputs

    inp = make_inputs(cfg, device=dev, rank=rank)
    thr = inp["threshold"]
    hs = inp["v"].contiguous()   # membrane in the (B, d_model, L) layout extract_base_events takes
    names = ["dt_idle", "dt_active", "A", "W_B", "W_C", "D"]
    params = {n: inp[n].clone().requires_grad_(True) for n in names}
    bucket = dp.GradBucket([params[n] for n in names], overlap=False) if world > 1 else None
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    u_leaf = inp["u"].detach().clone().requires_grad_(True)
    info = {}

    def run(hs_, u_, dout_):
        u = u_.requires_grad_(True) if not u_.requires_grad else u_
        ch, ts, kf, cu, mx, u_flat = itf.extract_events_base(hs_, u, thr, cfg.expand)
        y, _x = itf.selective_scan_flat_ch_fn(u_flat, kf, cu, mx, params["dt_idle"], params["dt_active"],
                                              params["A"], params["W_B"], params["W_C"], params["D"], None,
                                              is_depthwise_bc=True)
        dense = itf.restore_dense_fn(y, ts, cu, cfg.D, cfg.L)
        dense.backward(dout_)
        if bucket is not None:
            bucket.finish()
        info["ev"] = (int(ch.numel()), int(cu.numel() - 1), mx)

    def zero():
        if bucket is not None:
            bucket.zero_grad()
        else:
            for p in params.values():
                p.grad = None
        u_leaf.grad = None

    def step():
        run(hs, u_leaf, inp["dout"])

    for _ in range(args.warmup):
        zero()
        step()
    torch.cuda.synchronize()
    E, NC, mx = info["ev"]
    clocks = clock_sampler(local)
    t_ms = time_steps(step, zero, flush, args.steps)
    clk = clocks.stop()
    ms_per_step = _max_over_ranks(t_ms, dev) / args.steps
    value = _sum_over_ranks(E, dev) / (ms_per_step * 1e-3)
    per_op = stage_times(step, zero, flush, args.steps)

    e2e = None
    if not args.no_e2e:
        def run_on(bufs):
            zero()
            run(bufs[0], bufs[1].detach(), bufs[2])

        e_ms, h2d, d2h = time_e2e(dev, [hs, inp["u"], inp["dout"]], run_on,
                                  lambda: [params[n].grad for n in names], args.steps)
        e2e = {"value": _sum_over_ranks(E, dev) / (e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_ms,
               "copies": "pinned host -> device on a copy stream, step i+1's inputs overlapping step i"}

    alg = algorithmic_bytes(cfg, E, NC, max(1, (mx + 2047) // 2048))
    traffic = NCU_TRAFFIC.get((args.config, args.rho))
    roof, pipe, per_frac, peak = roofline_fields(per_op, alg, traffic)
    pipe["achieved_gbs_step"] = sum(alg.values()) / (ms_per_step * 1e-3) / 1e9
    pipe["frac_step"] = pipe["achieved_gbs_step"] / peak
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": f"synthetic (seeded, BASELINE.json {cfg.name} shapes and distributions)",
        "config": {"workload": f"{cfg.name}: B={cfg.B} D={cfg.D} N={cfg.N} L={cfg.L} rho={cfg.rho} "
                               f"{cfg.spikes} expand={cfg.expand} per GPU",
                   "events_per_gpu": E, "channels_per_gpu": NC, "max_seqlen": mx,
                   "parallelism": f"dp{world} (batch-sharded, grad all-reduce)",
                   "l2": "256 MiB memset flush before every timed step, outside its timing window"},
        "e2e": e2e,
        "roofline": roof,
        "pipeline_roofline": pipe,
        "per_op_ms": per_op,
        "per_op_frac_hbm": per_frac,
        "clocks": clk,
        "gpu_launches": args.steps * kernels_per_block(
            cfg, cfg.B, torch.cuda.get_device_properties(dev).multi_processor_count, stack=False),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if bucket is not None:
        del bucket
    return line


def resolve_config(args):
    from bc_mamba_b200.workloads import CONFIGS

    cfg = CONFIGS[args.config]
    if args.rho is not None:
        cfg = cfg.with_(rho=args.rho)
    if args.spikes is not None:
        cfg = cfg.with_(spikes=args.spikes)
    if args.blocks is not None:
        cfg = cfg.with_(blocks=args.blocks)
    return cfg


def run_ours(args):
    from bc_mamba_b200 import dp
    from bc_mamba_b200 import load_ops

    rank, world, local = dp.init_from_env("nccl")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    load_ops()
    points = [(args.rho, args.spikes)] if not args.sweep else SWEEP
    for rho, kind in points:
        args.rho, args.spikes = rho, kind
        cfg = resolve_config(args)
        fn = run_stack if cfg.name == "c4_stack" else run_block
        line = fn(args, cfg, rank, world, local, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
        torch.cuda.empty_cache()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------- CPU arm ----
def cpu_step_sample(cfg, batch_sub: int, seed_rank: int = 0):
    """One fwd+bwd of the reference's CPU path for one block on `batch_sub`
    batch rows: numpy restatements of extract / expand / gather / restore and
    the reference's pure-PyTorch scan (selective_scan_ref) on event-compacted
    tensors with autograd backward.  Returns (events, seconds)."""
    from bc_mamba_b200.workloads import make_inputs
    from oracle import events as ev
    from oracle import restore as rs
    from oracle.scan_ref import compact, depthwise_event_scan

    sub = cfg.with_(B=batch_sub)
    inp = make_inputs(sub, rank=seed_rank)
    t0 = time.perf_counter()
    v = inp["v"].numpy()
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(v, inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, sub.B, sub.d_model, sub.expand)
    u = inp["u"].float().numpy()
    u_flat = ev.gather_events_fwd(u, ch, t)
    u_c, km1, mask, idx = compact(u_flat, k, cu, sub.B, sub.D)
    u_c.requires_grad_(True)
    pr = {n: inp[n].clone().requires_grad_(True) for n in ["dt_idle", "dt_active", "A", "W_B", "W_C", "D"]}
    y_c = depthwise_event_scan(u_c, km1, mask.float(), pr["dt_idle"], pr["dt_active"], pr["A"], pr["W_B"],
                               pr["W_C"], pr["D"])
    msk = mask.numpy().reshape(-1)
    y_flat = np.zeros(u_flat.size, np.float32)
    y_flat[idx.reshape(-1)[msk]] = y_c.detach().numpy().reshape(-1)[msk]
    rs.restore_dense_fwd(y_flat, t, cu, sub.D, sub.L)
    dy = rs.restore_dense_bwd(inp["dout"].float().numpy(), t, cu, sub.D, sub.L)
    dy_c = torch.as_tensor(dy[idx], dtype=torch.float32) * mask
    (y_c * dy_c).sum().backward()
    du_flat = np.zeros(u_flat.size, np.float32)
    du_flat[idx.reshape(-1)[msk]] = u_c.grad.numpy().reshape(-1)[msk]
    ev.gather_events_bwd(du_flat, ch, t, sub.B * sub.D, sub.L)
    return int(ch.size), time.perf_counter() - t0


def cpu_sample_rows(cfg) -> int:
    return 1 if cfg.L * cfg.D >= 1_000_000 else max(1, min(cfg.B, 2))


def cpu_baseline(cfg, budget_s: float = 15.0):
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    batch_sub = cpu_sample_rows(cfg)
    ev_tot, t_tot, n = 0, 0.0, 0
    while t_tot < budget_s and n < 50:
        e, dt = cpu_step_sample(cfg, batch_sub, seed_rank=n)
        ev_tot += e
        t_tot += dt
        n += 1
    return {"value": ev_tot / t_tot, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} x fwd+bwd of one block on {batch_sub}/{cfg.B} batch rows of {cfg.name} "
                      f"(L={cfg.L}, D={cfg.D}, N={cfg.N}, rho={cfg.rho} {cfg.spikes}; {ev_tot} events, "
                      f"{t_tot:.1f} s): numpy extract/expand/gather/restore + torch selective_scan_ref "
                      f"restatement on event-compacted tensors"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cfg = resolve_config(args)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    batch_sub = cpu_sample_rows(cfg)
    for _ in range(args.warmup):
        cpu_step_sample(cfg, batch_sub)
    ev_tot, t_tot = 0, 0.0
    for i in range(args.steps):
        e, dt = cpu_step_sample(cfg, batch_sub, seed_rank=i)
        ev_tot += e
        t_tot += dt
    value = ev_tot / t_tot
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_tot / args.steps, "higher_is_better": True,
        "scaling": "strong" if cfg.name == "c4_stack" else "weak", "vs_baseline": None,
        "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": f"synthetic (seeded, BASELINE.json {cfg.name} shapes and distributions)",
        "config": {"workload": f"{cfg.name}: B={cfg.B} D={cfg.D} N={cfg.N} L={cfg.L} rho={cfg.rho} {cfg.spikes}",
                   "parallelism": "host CPU"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"each step: fwd+bwd of one block on {batch_sub}/{cfg.B} batch rows "
                                   f"({ev_tot // max(1, args.steps)} events)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c4")
    ap.add_argument("--rho", type=float, default=None)
    ap.add_argument("--spikes", default=None, choices=[None, "iid", "markov"])
    ap.add_argument("--sweep", action="store_true", help="configs[4]: every density and spike kind")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--blocks", type=int, default=None,
                    help="configs[4]: blocks in the stack (default 4; 1 = one block, for profiling)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.steps is None:
        args.steps = 30 if args.config == "c4" else 200
    if args.impl == "reference":
        if args.steps > 10 and args.config == "c4":
            args.steps = 10
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
