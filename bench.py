"""Benchmark of the BC_mamba event hot path on B200: fwd+bwd events/s.

One step = extract (threshold -> expanded events, gather of x_conv) -> sparse
selective scan forward -> ZOH restore forward, then the backward of all of
them (restore bwd -> scan bwd -> gather bwd), through the reference-facing
autograd Functions (bc_mamba_b200.interface), followed by the all-reduce of
the path's parameter gradients when N > 1.  Workload: configs[1] of
BASELINE.json (B=32, D=256, N=16, L=2048, 20 % i.i.d. spikes, fp32) per GPU
(weak scaling: every rank runs its own seeded batch).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config c1]

Prints ONE JSON line on rank 0.  `value` = events of all ranks / max-over-
ranks device time per step with inputs resident in HBM; `e2e` = the same
with pinned-host inputs copied in and parameter gradients copied out inside
every timed step.  L2 is flushed (256 MiB memset) before every timed step,
outside its timing window.
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


# the API stages of one step (interface.cuda_stage names) -> op keys
STAGE_OPS = {
    "routing_index_extraction": "extract", "sparse_scan_forward": "scan_fwd",
    "dense_restoration_forward": "restore_fwd", "restore_backward": "restore_bwd",
    "sparse_scan_backward": "scan_bwd", "gather_scatter_backward": "gather_bwd",
}
# kernels each stage launches (all ours): extract 3 (threshold + count,
# count scan, fill of the expanded stream with the gather of x_conv), scan fwd
# 1, restore fwd 1, restore bwd 1, scan bwd 2, gather bwd 1 (row writer)
KERNELS_PER_STEP = 9

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per stage on the
# c1 workload, summed over the stage's kernels, from one ncu capture of
# `python bench.py --steps 3 --warmup 3 --no-cpu-baseline` (summary in
# profiles/dram_traffic_c1.txt).  Writes that stay in the 126 MB L2 when a
# kernel ends are not counted.  Re-measured whenever a kernel changes.
NCU_TRAFFIC_C1 = {
    "extract": 109.04e6, "scan_fwd": 27.45e6, "restore_fwd": 38.20e6, "restore_bwd": 70.59e6,
    "scan_bwd": 70.54e6, "gather_bwd": 37.33e6,
}


def algorithmic_bytes(cfg, E, NC, n_chunks):
    """Bytes each API call must move once (inputs read once, outputs written
    once), per op, for one fwd+bwd step."""
    s = torch.tensor([], dtype=cfg.dtype).element_size()
    sv = 4
    NCb = NC // cfg.expand
    L, N = cfg.L, cfg.N
    b = {
        "extract": NCb * L * sv + 12 * E + 4 * NC + 2 * s * E,
        "scan_fwd": (2 * s + 4) * E + 8 * N * NC * n_chunks,
        "restore_fwd": (4 + s) * E + NC * L * s,
        "restore_bwd": NC * L * s + 8 * E,
        "scan_bwd": (3 * s + 4) * E + 8 * N * NC * n_chunks,
        "gather_bwd": NC * L * s + (s + 8) * E,
    }
    return b


# ------------------------------------------------------------- GPU arm ----
def run_ours(args):
    from bc_mamba_b200 import dp
    from bc_mamba_b200 import interface as itf
    from bc_mamba_b200 import load_ops
    from bc_mamba_b200.workloads import CONFIGS, make_inputs

    rank, world, local = dp.init_from_env("nccl")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    if args.rho is not None:
        cfg = cfg.with_(rho=args.rho)
    ops = load_ops()
    inp = make_inputs(cfg, device=dev, rank=rank)
    thr = inp["threshold"]
    hs = inp["v"].contiguous()   # membrane in the (B, d_model, L) layout extract_base_events takes
    names = ["dt_idle", "dt_active", "A", "W_B", "W_C", "D"]
    params = {n: inp[n].clone().requires_grad_(True) for n in names}
    # parameter gradients live in one bucket (autograd accumulates into it);
    # one all-reduce after the backward.  Launching it from autograd beside
    # the gather backward (overlap=True) measured ~10 % slower per step on
    # 2 x B200: the ~50 KB reduction is latency, not bandwidth
    bucket = dp.GradBucket([params[n] for n in names], overlap=False) if world > 1 else None
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step(hs_, u_, dout_):
        u = u_.requires_grad_(True) if not u_.requires_grad else u_
        ch, ts, kf, cu, mx, u_flat = itf.extract_events_base(hs_, u, thr, cfg.expand)
        y, _x = itf.selective_scan_flat_ch_fn(u_flat, kf, cu, mx, params["dt_idle"], params["dt_active"],
                                              params["A"], params["W_B"], params["W_C"], params["D"], None,
                                              is_depthwise_bc=True)
        dense = itf.restore_dense_fn(y, ts, cu, cfg.D, cfg.L)
        dense.backward(dout_)
        if bucket is not None:
            bucket.finish()
        return int(ch.numel()), int(cu.numel() - 1), mx

    # one x_conv leaf reused every step; its gradient (the gather backward's
    # dense output) is dropped before each step like the parameters' grads, so
    # every step allocates from the warm caching allocator
    u_leaf = inp["u"].detach().clone().requires_grad_(True)

    def zero():
        if bucket is not None:
            bucket.zero_grad()      # gradients are views into the all-reduce bucket
        else:
            for p in params.values():
                p.grad = None
        u_leaf.grad = None

    E, NC, mx = step(hs, u_leaf, inp["dout"])
    for _ in range(max(0, args.warmup - 1)):
        zero()
        step(hs, u_leaf, inp["dout"])
    torch.cuda.synchronize()

    # ---- value: device-resident inputs, K timed steps, L2 flushed before each
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                          else int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])).start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        zero()
        flush.zero_()
        starts[i].record()
        step(hs, u_leaf, inp["dout"])
        ends[i].record()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    # per-op device time: the same K steps again with every API stage
    # bracketed by CUDA events on its launching stream (mean per step).  A
    # separate pass, because creating and recording the events costs host time
    # the timed steps above should not carry.
    with itf.stage_timing() as stage_log:
        for i in range(args.steps):
            zero()
            flush.zero_()
            step(hs, u_leaf, inp["dout"])
    torch.cuda.synchronize()
    per_op = {k: 0.0 for k in STAGE_OPS.values()}
    for name, s_ev, e_ev in stage_log:
        per_op[STAGE_OPS[name]] += s_ev.elapsed_time(e_ev) / args.steps
    t_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t_max = torch.tensor([t_ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t_max, op=torch.distributed.ReduceOp.MAX)
    ms_per_step = float(t_max.item()) / args.steps
    value = world * E / (ms_per_step * 1e-3)

    # ---- e2e: pinned host inputs in, parameter gradients out, every step.
    # Step i+1's inputs are copied on a second stream into the other half of a
    # double buffer while step i computes (the way a data loader feeds a
    # training loop); the window runs from the first copy to the last
    # gradient read-back and is divided by K.  Each step reads 167 MB of fresh
    # inputs (larger than L2), so no flush is needed between steps.
    h_v = hs.cpu().pin_memory()
    h_u = inp["u"].cpu().pin_memory()
    h_dout = inp["dout"].cpu().pin_memory()
    h_grads = [torch.empty(params[n].shape, dtype=torch.float32).pin_memory() for n in names]
    h2d = h_v.numel() * h_v.element_size() + h_u.numel() * h_u.element_size() + \
        h_dout.numel() * h_dout.element_size()
    d2h = sum(g.numel() * 4 for g in h_grads)
    bufs = [(torch.empty_like(hs), torch.empty_like(inp["u"]), torch.empty_like(inp["dout"])) for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    comp = torch.cuda.current_stream(dev)

    def h2d_into(b, wait_free):
        with torch.cuda.stream(copy_stream):
            if wait_free:
                copy_stream.wait_event(free[b])
            for d_t, h_t in zip(bufs[b], (h_v, h_u, h_dout)):
                d_t.copy_(h_t, non_blocking=True)
            ready[b].record(copy_stream)

    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e_start.record(comp)
    copy_stream.wait_stream(comp)
    h2d_into(0, False)
    for i in range(args.steps):
        b = i % 2
        if i + 1 < args.steps:
            h2d_into(1 - b, i >= 1)          # the other half was last used by step i-1
        comp.wait_event(ready[b])
        zero()
        d_v, d_u, d_dout = bufs[b]
        step(d_v, d_u.detach(), d_dout)      # a fresh x_conv leaf over the buffer
        for g, n in zip(h_grads, names):
            g.copy_(params[n].grad, non_blocking=True)
        free[b].record(comp)
    e_end.record(comp)
    torch.cuda.synchronize()
    te = torch.tensor([e_start.elapsed_time(e_end)], device=dev)
    if world > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.barrier()
    e2e_ms = float(te.item()) / args.steps

    n_chunks = max(1, (mx + 2047) // 2048)
    alg = algorithmic_bytes(cfg, E, NC, n_chunks)
    peak, peak_kind = measured_peak_gbs()
    dominant = max(per_op, key=lambda k: per_op[k])
    dom_ms = per_op[dominant]
    achieved = alg[dominant] / (dom_ms * 1e-3) / 1e9
    total_alg = sum(alg.values())
    kernel_ms = sum(per_op.values())
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": "synthetic (seeded, BASELINE.json configs[1] shapes and distributions)",
        "config": {"workload": f"{cfg.name}: B={cfg.B} D={cfg.D} N={cfg.N} L={cfg.L} rho={cfg.rho} "
                               f"{cfg.spikes} expand={cfg.expand} per GPU",
                   "events_per_gpu": E, "channels_per_gpu": NC, "max_seqlen": mx,
                   "parallelism": f"dp{world} (batch-sharded, grad all-reduce)",
                   "l2": "256 MiB memset flush before every timed step, outside its timing window"},
        "e2e": {"value": world * E / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "copies": "pinned host -> device on a copy stream, step i+1's inputs overlapping step i"},
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_C1.get(dominant) if args.config == "c1" and args.rho is None else None,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6650 GB/s",
                     "algorithmic_bytes": alg[dominant], "ms": dom_ms},
        "pipeline_roofline": {"algorithmic_bytes": total_alg, "kernel_ms_sum": kernel_ms,
                              "achieved_gbs_kernels": total_alg / (kernel_ms * 1e-3) / 1e9,
                              "frac_kernels": total_alg / (kernel_ms * 1e-3) / 1e9 / peak,
                              "achieved_gbs_step": total_alg / (ms_per_step * 1e-3) / 1e9,
                              "frac_step": total_alg / (ms_per_step * 1e-3) / 1e9 / peak},
        "per_op_ms": per_op,
        "per_op_frac_hbm": {k: alg[k] / (per_op[k] * 1e-3) / 1e9 / peak for k in per_op},
        "clocks": clk,
        "gpu_launches": KERNELS_PER_STEP * args.steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if bucket is not None:
        del bucket
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------- CPU arm ----
def cpu_step_sample(cfg, batch_sub: int, seed_rank: int = 0):
    """One fwd+bwd of the reference's CPU path on `batch_sub` batch rows:
    numpy restatements of extract / expand / gather / restore and the
    reference's pure-PyTorch scan (selective_scan_ref) on event-compacted
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


def cpu_baseline(cfg, budget_s: float = 15.0):
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    batch_sub = max(1, min(cfg.B, 2))
    ev_tot, t_tot, n = 0, 0.0, 0
    while t_tot < budget_s and n < 50:
        e, dt = cpu_step_sample(cfg, batch_sub, seed_rank=n)
        ev_tot += e
        t_tot += dt
        n += 1
    return {"value": ev_tot / t_tot, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} x fwd+bwd on {batch_sub}/{cfg.B} batch rows of {cfg.name} "
                      f"({ev_tot} events, {t_tot:.1f} s): numpy extract/expand/gather/restore + "
                      f"torch selective_scan_ref restatement on event-compacted tensors"}


def run_reference(args):
    from bc_mamba_b200.workloads import CONFIGS

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    if args.rho is not None:
        cfg = cfg.with_(rho=args.rho)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    batch_sub = 2
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
        "scaling": "weak", "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""),
        "data": "synthetic (seeded, BASELINE.json configs[1] shapes and distributions)",
        "config": {"workload": f"{cfg.name}: B={cfg.B} D={cfg.D} N={cfg.N} L={cfg.L} rho={cfg.rho}",
                   "parallelism": "host CPU"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"each step: fwd+bwd on {batch_sub}/{cfg.B} batch rows ({ev_tot // max(1, args.steps)} events)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1")
    ap.add_argument("--rho", type=float, default=None)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
