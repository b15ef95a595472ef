"""Data-parallel path on CPU ranks (gloo, world size 2): batch-sharded
gradients after the bucketed all-reduce equal the full-batch gradients, and
rank failures / mismatched buckets surface as host-side errors."""
import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_grads(cfg, inp, b0, b1):
    """Parameter gradients of the pipeline for batch rows [b0, b1) (oracle)."""
    from oracle import events as ev
    from oracle import restore as rs
    from oracle import scan as sc

    sub = cfg.with_(B=b1 - b0)
    v = inp["v"][b0:b1].numpy()
    bch, bt, bk, bcu, _, _ = ev.extract_base_events(v, inp["threshold"])
    ch, t, k, cu, mx = ev.expand_base_events(bch, bt, bk, bcu, sub.B, sub.d_model, sub.expand)
    uf = ev.gather_events_fwd(inp["u"][b0:b1].numpy(), ch, t)
    p = {n: inp[n].numpy() for n in ["dt_idle", "dt_active", "A", "W_B", "W_C", "D"]}
    dy = rs.restore_dense_bwd(inp["dout"][b0:b1].numpy(), t, cu, sub.D, sub.L)
    g = sc.scan_bwd(uf, k, cu, int(mx), p["dt_idle"], p["dt_active"], p["A"], p["W_B"], p["W_C"], dy,
                    D=p["D"], is_depthwise_bc=True)
    return {"A": g[1], "W_B": g[2], "W_C": g[3], "dt_idle": g[4], "dt_active": g[5], "D": g[6]}


def _worker(rank, world, port, outdir, mode):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist

    from bc_mamba_b200 import dp
    from bc_mamba_b200.workloads import CONFIGS, make_inputs

    status = "ok"
    try:
        dp.init_from_env("gloo", timeout_s=10.0)
        cfg = CONFIGS["c0"].with_(B=4, L=128)
        inp = make_inputs(cfg)
        names = ["A", "W_B", "W_C", "dt_idle", "dt_active", "D"]
        params = {n: torch.zeros(inp[n].shape, dtype=torch.float64) for n in names}
        if mode == "mismatch" and rank == 1:
            params["D"] = torch.zeros(inp["D"].numel() + 3, dtype=torch.float64)
        b0, b1 = dp.shard_range(cfg.B, rank, world)
        g = _oracle_grads(cfg, inp, b0, b1)
        for n in names:
            if params[n].shape == g[n].shape:
                params[n].grad = torch.as_tensor(g[n])
            else:
                params[n].grad = torch.zeros_like(params[n])
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected rank failure before the collective")
        if mode == "overlap":
            # launched from autograd hooks; two steps re-arm through zero_grad
            leaves = {n: params[n].detach().clone().requires_grad_(True) for n in names}
            bucket = dp.GradBucket([leaves[n] for n in names], average=False, overlap=True)
            for _ in range(2):
                bucket.zero_grad()
                sum((leaves[n] * torch.as_tensor(g[n])).sum() for n in names).backward()
                bucket.finish()
            params = leaves
        else:
            bucket = dp.GradBucket([params[n] for n in names], average=False)
            bucket.start().finish()
        if mode in ("ok", "overlap"):
            full = _oracle_grads(cfg, inp, 0, cfg.B)
            for n in names:
                np.testing.assert_allclose(params[n].grad.numpy(), full[n], rtol=1e-9, atol=1e-9)
    except Exception as e:  # report, never hang: the test inspects the files
        status = f"error: {type(e).__name__}: {e}"
    finally:
        Path(outdir, f"rank{rank}.txt").write_text(status)
        try:
            import torch.distributed as dist2
            if dist2.is_initialized():
                dist2.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_worker, args=(2, port, d, mode), nprocs=2, join=False,
                                 start_method="spawn")
        for p in ctx.processes:
            p.join(120)
            if p.is_alive():
                p.kill()
        return [Path(d, f"rank{r}.txt").read_text() if Path(d, f"rank{r}.txt").exists() else "missing"
                for r in range(2)]


def test_sharded_grads_allreduce_equal_full_batch():
    res = _run("ok")
    assert res == ["ok", "ok"], res


def test_allreduce_launched_from_autograd_hooks():
    res = _run("overlap")
    assert res == ["ok", "ok"], res


def test_rank_failure_surfaces_on_host():
    res = _run("fail")
    assert res[1].startswith("error") and "injected" in res[1]
    assert res[0].startswith("error"), res  # the surviving rank's collective fails, not hangs


def test_mismatched_buckets_raise():
    res = _run("mismatch")
    assert any(r.startswith("error") for r in res), res


def test_shard_range_partitions():
    from bc_mamba_b200.dp import shard_range

    for n in [1, 7, 128]:
        for w in [1, 2, 3, 8]:
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))


def test_bucket_gradients_are_views_that_autograd_accumulates_into():
    """Gradients live in the bucket: autograd adds into the views, zero_grad
    clears them with one fill, and a .grad reset to None is re-bound."""
    from bc_mamba_b200 import dp

    a = torch.zeros(3, 4, dtype=torch.float32, requires_grad=True)
    b = torch.zeros(5, dtype=torch.float32, requires_grad=True)
    bucket = dp.GradBucket([a, b])
    lo, hi = bucket.flat.data_ptr(), bucket.flat.data_ptr() + bucket.flat.numel() * 4
    for step in range(2):
        bucket.zero_grad()
        ((a * 2.0).sum() + (b * 3.0).sum()).backward()
        for p in (a, b):
            assert lo <= p.grad.data_ptr() < hi
        assert torch.all(a.grad == 2.0) and torch.all(b.grad == 3.0)
    a.grad = None
    bucket.zero_grad()
    assert a.grad is not None and lo <= a.grad.data_ptr() < hi and float(bucket.flat.abs().sum()) == 0.0
