#!/usr/bin/env python
"""Benchmark of the B200 token-selection path (qsamp).

Workload (N=1): the batched-server-decode parameter distribution
(per-row T~U[0.2,1.2], top-k in {0,20,40,100}, top-p~U[0.8,1.0],
frequency/presence penalties over a 256-id history) at B=256, V=151936, fp32
logits -- the B=256 / V=151936 point of the headline metric. A step is one
batched selection call over B rows. The timed steps rotate over four seeded
batches of that distribution (their mix of full-vocabulary rows differs), the
same four on every rank. Under torchrun every rank runs its own B rows (weak
scaling, no collective on the data path).

  value    -- rows/s over all ranks, inputs resident in HBM, device-timed with
              CUDA events (max over ranks); the four batches (622 MB) exceed
              L2, so every step reads its logits from HBM.
  e2e      -- the same through qsamp_sample_host: pinned host logits, history
              and params copied in, ids and results copied out, every step.
  roofline -- algorithmic bytes of the dominant kernel per launch over its
              mean launch time, against the measured HBM copy bandwidth;
              step_frac: the whole step's algorithmic bytes over the step time.
  config4_B256 -- C4 (bf16, V=262144, soft-cap 30, full-vocabulary top-p) at
              B=256 with its own roofline; b10 -- the B=10 latency point;
  vshard   -- C5 (B=512, V=262144 fp32, k=64, p=0.95) split V/N over the
              ranks: shard_topk, an NCCL all-gather of the candidates,
              merge_topk; checked bit for bit against the unsharded call.

`--impl reference` times the reference's own CPU sampler (src/sampling
compiled unmodified with its Release flags, oracle/_ref) on the host cores.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B_DEFAULT = 256
V = 151936
HIST = 256
BATCH_SEEDS = (1000, 2000, 6000, 7000)  # the config2-B256 batches every rank serves, in rotation
V5 = 262144


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(key):
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d.get(key)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every few ms
    while the timed region runs (reads only; no setting is changed)."""

    HW, HW_THERMAL, SW_THERMAL, SW_POWER = 0x8, 0x40, 0x20, 0x4

    def __init__(self, index, period=0.005):
        self.index = index
        self.period = period
        self.samples = []
        self.stop = threading.Event()
        self.ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.ok = False
        return self

    def _run(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self.stop.set()
        if self.ok:
            self.t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        names = {self.HW: "hw_slowdown", self.HW_THERMAL: "hw_thermal_slowdown",
                 self.SW_THERMAL: "sw_thermal_slowdown", self.SW_POWER: "sw_power_cap"}
        for _, rs in self.samples:
            for bit, n in names.items():
                if rs & bit:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_sm,
                "reasons": sorted(reasons), "samples": len(self.samples)}


def algorithmic_bytes_per_row(V_, hist_len, bytes_per_logit=4, mask=False):
    # logits + allow-mask words + history ids + params/u/result per row
    return V_ * bytes_per_logit + (((V_ + 31) // 32) * 4 if mask else 0) + 4 * hist_len + 64


def _events_ms(stream, fn, reps):
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(reps):
        fn(i)
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _kernel_times(ctx, step, n):
    """Per-kernel device times of n steps (the library's own CUDA events around
    each launch, on the launching stream) and the rows each kernel served."""
    ctx.set_kernel_timing(True)
    rec = []
    for i in range(n):
        step(i)
        c = ctx.counters()
        rec.append((c["last_stream_kernel_ms"], c["last_rows_kernel_ms"], c["last_stream_rows"],
                    c["last_cluster_rows"], c["last_cluster_size"], c["last_clusters"], c["last_hist_kernel_ms"],
                    c["last_hist_rows"], c["last_hist_handed_on"]))
    ctx.set_kernel_timing(False)
    return rec


# ------------------------------------------------------------------ GPU arm
def run_gpu(args):
    import torch
    import torch.distributed as dist

    from qwenium_b200 import qsamp
    from qwenium_b200 import workloads as W

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    B = args.batch
    # weak scaling: every rank serves the same four seeded batches of B rows
    # on its own GPU (fixed work per GPU); the rotation spreads the timed
    # steps over batches with different mixes of full-vocabulary rows
    cfgs = [W.config2(seed=s, B=B) for s in BATCH_SEEDS]
    nb = len(cfgs)
    ctx = qsamp.Context(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    bytes_one = B * V * 4
    xs = [torch.from_numpy(c["logits"]).to(dev) for c in cfgs]
    hs = [torch.from_numpy(c["hist"]).to(dev) for c in cfgs]
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    res = torch.empty((B, 32), dtype=torch.uint8, device=dev)

    def step(i):
        c = cfgs[i % nb]
        ctx.sample_batch(xs[i % nb], c["params"], hist=hs[i % nb], hist_len=c["hist_len"], u=c["u"],
                         out_ids=ids, out_results=res, stream=stream.cuda_stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    ctx.poll_status()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.counters()["kernel_launches"]
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    gpu_launches = int(ctx.counters()["kernel_launches"] - launches0)
    ctx.poll_status()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # per-kernel device time: the same steps with the library's own events
    # around each kernel launch (on the launching stream)
    krec = _kernel_times(ctx, step, max(nb, min(args.steps, 4 * nb)))
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())

    # e2e through the host entry point with pinned buffers
    e2e_rows_s = None
    h2d = d2h = 0
    if not args.no_e2e:
        hxs = [torch.from_numpy(c["logits"]).pin_memory() for c in cfgs]
        hhs = [torch.from_numpy(c["hist"]).pin_memory() for c in cfgs]
        e2e_steps = max(nb, min(args.steps, 5 * nb))

        def hstep(i):
            c = cfgs[i % nb]
            ctx.sample_host(hxs[i % nb].numpy(), c["params"], hist=hhs[i % nb].numpy(), hist_len=c["hist_len"],
                            u=c["u"])

        for i in range(2):
            hstep(i)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            hstep(i)
        el = time.perf_counter() - t0
        el_t = torch.tensor([el], device=dev)
        if world > 1:
            dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
        e2e_rows_s = world * B * e2e_steps / float(el_t.item())
        h2d = B * V * 4 + B * HIST * 4 + B * (48 + 8 + 4)
        d2h = B * (4 + 32)
        hxs.clear()
        hhs.clear()

    peak, peak_kind = measured_peaks()
    # B=10 latency point (device-timed, same parameter distribution)
    b10 = None
    if rank == 0 and not args.no_b10:
        c10 = W.config2(seed=77, B=10)
        x10 = [torch.from_numpy(c10["logits"]).to(dev) for _ in range(8)]
        h10 = torch.from_numpy(c10["hist"]).to(dev)
        i10 = torch.empty(10, dtype=torch.int32, device=dev)
        f10 = lambda i: ctx.sample_batch(x10[i % 8], c10["params"], hist=h10, hist_len=c10["hist_len"], u=c10["u"],
                                         out_ids=i10, stream=stream.cuda_stream)
        for i in range(5):
            f10(i)
        torch.cuda.synchronize()
        t10 = _events_ms(stream, f10, 50)
        alg10 = 10 * algorithmic_bytes_per_row(V, HIST)
        b10 = {"ms_per_step": round(t10, 4), "rows_per_s": round(10 / (t10 * 1e-3), 1),
               "roofline": {"bound": "hbm", "bytes_per_step": alg10,
                            "achieved": round(alg10 / (t10 * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                            "frac": round(alg10 / (t10 * 1e-3) / 1e9 / peak, 4),
                            "note": "latency-bound: 10 rows cannot fill 148 SMs"}}
        x10.clear()

    c4 = run_config4(ctx, dev, stream, peak) if (rank == 0 and not args.no_c4) else None
    vsh = run_vshard(ctx, dev, stream, world, rank, args, peak) if not args.no_vshard else None
    extras = run_extras(ctx, dev, stream) if (rank == 0 and args.extras) else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfgs, seconds=args.cpu_seconds)

    vsh_bad = vsh is not None and vsh.get("bit_exact") is False
    if world > 1:
        flag = torch.tensor([1 if vsh_bad else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        vsh_bad = bool(flag.item())
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        if vsh_bad:
            sys.exit(3)
        return
    # the dominant kernel: the larger mean device time per step
    k_stream = statistics.mean(r[0] for r in krec)
    k_rows = statistics.mean(r[1] for r in krec)
    n_stream = statistics.mean(r[2] for r in krec)
    n_cluster = statistics.mean(r[3] for r in krec)
    per_row = algorithmic_bytes_per_row(V, HIST)
    if k_rows >= k_stream:
        kname, units, launch_ms = "qs_rows_kernel", n_cluster, k_rows
    else:
        kname, units, launch_ms = "qs_stream_kernel", n_stream, k_stream
    alg = per_row * units
    achieved = alg / (launch_ms * 1e-3) / 1e9
    traffic = ncu_traffic(f"{kname}/config2-B256")
    ms_step = ms / args.steps
    step_bytes = per_row * B
    out = {
        "metric": "sampled rows/s (batched token selection, B=256, V=151936)",
        "value": round(world * B * args.steps / (ms * 1e-3), 1),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded config-2 distribution)",
        "config": {"workload": "config2-B256: batched server decode parameters at B=256, V=151936 fp32",
                   "B_per_gpu": B, "V": V, "history": HIST, "parallelism": f"rows x{world}",
                   "batch_seeds": list(BATCH_SEEDS),
                   "rows_per_batch": {"stream": [int(r[2]) for r in krec[:nb]],
                                      "cluster": [int(r[3]) for r in krec[:nb]]},
                   "l2": f"{nb} rotating seeded batches ({nb * bytes_one / 1e6:.0f} MB) > L2"},
        "e2e": {"value": round(e2e_rows_s, 1) if e2e_rows_s else None, "unit": "rows/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": gpu_launches,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                     "kernel": kname, "rows_per_launch": round(units, 2), "bytes_per_launch": round(alg),
                     "launch_ms": round(launch_ms, 4),
                     "kernels_ms": {"qs_stream_kernel": round(k_stream, 4), "qs_rows_kernel": round(k_rows, 4)},
                     "cluster_plan": {"ctas_per_cluster": krec[0][4], "clusters": krec[0][5]},
                     "step_bytes": step_bytes,
                     "step_frac": round(step_bytes / (ms_step * 1e-3) / 1e9 / peak, 4),
                     "target_frac": 0.70},
        "clocks": clk.summary(),
    }
    if b10:
        out["b10"] = b10
    if c4:
        out["config4_B256"] = c4
    if vsh:
        out["vshard"] = vsh
    if extras:
        out["extras"] = extras
    if cpu:
        out["cpu_baseline"] = cpu
    print(json.dumps(out))
    if vsh_bad:
        sys.exit(3)


def run_config4(ctx, dev, stream, peak):
    """C4 at B=256: bf16 V=262144, soft-cap 30, full-vocabulary top-p 0.9,
    repetition penalty over 512 ids; two seeded batches rotated (268 MB > L2)."""
    import torch

    from qwenium_b200 import workloads as W

    cfgs = [W.config4(4, B=256), W.config4(44, B=256)]
    xs = [torch.from_numpy(np.ascontiguousarray(c["logits"]).view(np.int16)).to(dev) for c in cfgs]
    hs = [torch.from_numpy(c["hist"]).to(dev) for c in cfgs]
    f = lambda i: ctx.sample_batch(xs[i % 2], cfgs[i % 2]["params"], hist=hs[i % 2], hist_len=cfgs[i % 2]["hist_len"],
                                   u=cfgs[i % 2]["u"], stream=stream.cuda_stream)
    for i in range(3):
        f(i)
    ms = _events_ms(stream, f, 6)
    ctx.poll_status()
    krec = _kernel_times(ctx, f, 4)
    # the histogram kernel serves these rows (bf16, full vocabulary); rows it
    # cannot prove exact go on to the cluster kernel in the same call
    hms = statistics.mean(r[6] for r in krec)
    cms = statistics.mean(r[1] for r in krec)
    per_row = algorithmic_bytes_per_row(V5, 512, bytes_per_logit=2)
    hrows = krec[0][7]
    alg = hrows * per_row
    xs.clear()
    hs.clear()
    return {"workload": "config4-B256: bf16 V=262144, soft-cap 30, T 1.0, top-p 0.9, top-k 0, repetition 1.05/512",
            "softcap_parity": "unpinned: the reference applies the soft-cap as ggml ops (layers/attention.cpp:30-36) "
                              "and ggml is not in the reference tree; this build uses a correctly rounded tanh",
            "ms_per_step": round(ms, 4), "rows_per_s": round(256 / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "kernel": "qs_hist_kernel", "rows_per_launch": hrows,
                         "bytes_per_launch": alg, "launch_ms": round(hms, 4),
                         "achieved": round(alg / (hms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / (hms * 1e-3) / 1e9 / peak, 4),
                         "traffic": ncu_traffic("qs_hist_kernel/config4-B256"),
                         "step_frac": round(256 * per_row / (ms * 1e-3) / 1e9 / peak, 4),
                         "handed_on_rows": [r[8] for r in krec], "cluster_kernel_ms": round(cms, 4),
                         "cluster_plan": {"ctas_per_cluster": krec[0][4], "clusters": krec[0][5]}}}


def run_vshard(ctx, dev, stream, world, rank, args, peak):
    """C5: B=512, V=262144 fp32 logits split contiguously V/N over the ranks
    (rank r holds shard_range(V, N, r)); per step shard_topk (k=64), an NCCL
    all-gather of the [B][k] value and id blocks, merge_topk. Strong scaling
    (the total work is fixed). Rank 0 checks the merged rows against the
    unsharded call on the full logits, bit for bit."""
    import torch
    import torch.distributed as dist

    from qwenium_b200 import qsamp
    from qwenium_b200 import shard
    from qwenium_b200 import workloads as W

    cfg = W.config5(5, B=512)
    p, u = cfg["params"], cfg["u"]
    k = 64
    lo, n = shard.shard_range(V5, world, rank)
    one = 512 * n * 4
    ncp = max(2, int(np.ceil(3 * 126e6 / one)) + 1)
    xl = [torch.from_numpy(np.ascontiguousarray(cfg["logits"][:, lo:lo + n])).to(dev) for _ in range(ncp)]
    cv = torch.empty((512, k), dtype=torch.float32, device=dev)
    ci = torch.empty((512, k), dtype=torch.int32, device=dev)
    av = torch.empty((world, 512, k), dtype=torch.float32, device=dev)
    ai = torch.empty((world, 512, k), dtype=torch.int32, device=dev)
    oid = torch.empty(512, dtype=torch.int32, device=dev)
    ores = torch.empty((512, 32), dtype=torch.uint8, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step(i, timed=False):
        if timed:
            ev[0].record(stream)
        ctx.shard_topk(xl[i % ncp], p, lo, V5, k, cand_vals=cv, cand_ids=ci, stream=stream.cuda_stream)
        if timed:
            ev[1].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(av, cv)
            dist.all_gather_into_tensor(ai, ci)
        else:
            av[0].copy_(cv)
            ai[0].copy_(ci)
        if timed:
            ev[2].record(stream)
        ctx.merge_topk(av, ai, p, u=u, out_ids=oid, out_results=ores, stream=stream.cuda_stream)
        if timed:
            ev[3].record(stream)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    ctx.poll_status()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    steps = max(5, min(args.steps, 20))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(steps):
        step(i)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    parts = []
    for i in range(5):
        step(i, timed=True)
        torch.cuda.synchronize()
        parts.append((ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3]),
                      ev[0].elapsed_time(ev[3])))
    t = torch.tensor([ms] + [statistics.mean(x[j] for x in parts) for j in range(4)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, t_shard, t_gather, t_merge, t_all = (float(v) for v in t.tolist())
    bit_exact = None
    if rank == 0:
        got = ores.cpu().numpy().copy()
        xl.clear()
        xf = torch.from_numpy(cfg["logits"]).to(dev)
        want = ctx.sample_batch(xf, p, u=u)
        torch.cuda.synchronize()
        ctx.poll_status()
        bit_exact = bool(np.array_equal(want.cpu().numpy(), got))
        del xf
    alg = 512 * n * 4
    return {"workload": "config5-B512: fp32 V=262144 split V/N per rank, local top-64, NCCL all-gather, merge",
            "n_ranks": world, "scaling": "strong", "ms_per_step": round(ms, 4),
            "rows_per_s": round(512 / (ms * 1e-3), 1),
            "step_parts_ms": {"shard_topk": round(t_shard, 4), "all_gather": round(t_gather, 4),
                              "merge_topk": round(t_merge, 4)},
            "all_gather_share": round(t_gather / t_all, 4) if t_all > 0 else None,
            "gather_bytes_per_rank": 512 * k * 8,
            "shard_roofline": {"bound": "hbm", "bytes_per_launch": alg, "launch_ms": round(t_shard, 4),
                               "frac": round(alg / (t_shard * 1e-3) / 1e9 / peak, 4)},
            "bit_exact": bit_exact}


def run_extras(ctx, dev, stream):
    """Secondary measurements (device-timed, inputs resident, rotating buffers):
    C4 at B=1024, batched greedy draft verification and grammar char-class
    masks; with the reference's own CPU time per unit where it compiled
    (oracle/_ref)."""
    import ctypes

    import torch

    from qwenium_b200 import qsamp
    from qwenium_b200 import workloads as W

    out = {}
    peak, _ = measured_peaks()
    # C4 at B=1024 (its own seeded batch; two copies on the device, 1.07 GB)
    c4 = W.config4(4, B=1024)
    xs = [torch.from_numpy(np.ascontiguousarray(c4["logits"]).view(np.int16)).to(dev) for _ in range(2)]
    h4 = torch.from_numpy(c4["hist"]).to(dev)
    f4 = lambda i: ctx.sample_batch(xs[i % 2], c4["params"], hist=h4, hist_len=c4["hist_len"], u=c4["u"],
                                    stream=stream.cuda_stream)
    for i in range(2):
        f4(i)
    ms = _events_ms(stream, f4, 3)
    out["config4_B1024"] = {"ms_per_call": round(ms, 4), "rows_per_s": round(1024 / (ms * 1e-3), 1)}
    del xs, h4
    # greedy verification: 128 slots x 5 drafts, V=151936 fp32
    rng = np.random.default_rng(0)
    n, K = 640, 5
    vx = [torch.from_numpy((rng.standard_normal((n, V)) * 3).astype(np.float32)).to(dev) for _ in range(3)]
    off = torch.from_numpy(np.arange(0, n + 1, K, dtype=np.int32)).to(dev)
    dr = torch.from_numpy(rng.integers(0, V, n).astype(np.int32)).to(dev)
    fv = lambda i: ctx.verify_greedy(vx[i % 3], off, dr, -1, stream=stream.cuda_stream)
    for i in range(3):
        fv(i)
    ms = _events_ms(stream, fv, 20)
    gbs = n * V * 4 / (ms * 1e-3) / 1e9
    out["verify_greedy"] = {"rows": n, "V": V, "us_per_call": round(ms * 1e3, 1), "gbs": round(gbs, 1),
                            "frac_of_measured_hbm": round(gbs / peak, 3)}
    # char-class masks: 256 states, negated class [^"\\] over the C3 vocabulary
    vocab = W.config3_vocab()
    table = qsamp.first_byte_table(vocab)
    cls = np.stack([qsamp.char_class_bits(['"', "\\"], True) for _ in range(256)])
    dt = torch.from_numpy(table.view(np.int16)).to(dev)
    dc = torch.from_numpy(cls.view(np.int32)).to(dev)
    dm = torch.zeros((256, (len(vocab) + 31) // 32), dtype=torch.int32, device=dev)
    fc = lambda i: ctx.char_class_masks(dt, dc, dm, stream=stream.cuda_stream)
    for i in range(3):
        fc(i)
    ms = _events_ms(stream, fc, 50)
    out["char_class_masks"] = {"states": 256, "V": len(vocab), "us_per_call": round(ms * 1e3, 2)}
    # the reference's per-unit CPU times (one host thread), where it compiled
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if O.ref_available("strict"):
        lib = O.ref_lib("strict")
        x5 = (rng.standard_normal((K, V)) * 3).astype(np.float32)
        d5 = np.arange(K, dtype=np.int32)
        a_, b_, h_ = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        t0 = time.perf_counter()
        for _ in range(20):
            lib.qwref_spec_verify(O._ptr(x5), K, V, O._ptr(d5), -1, ctypes.byref(a_), ctypes.byref(b_), ctypes.byref(h_))
        out["verify_greedy"]["reference_us_per_slot"] = round((time.perf_counter() - t0) / 20 * 1e6, 1)
        rv = O.RefVocab(vocab)
        arr = np.frombuffer(b'"\\', np.uint8).copy()
        mk = np.zeros(len(vocab), np.uint8)
        t0 = time.perf_counter()
        for _ in range(20):
            lib.qwref_trie_mark_char_class(rv.trie, O._ptr(arr), 2, 1, len(vocab), O._ptr(mk))
        out["char_class_masks"]["reference_us_per_state"] = round((time.perf_counter() - t0) / 20 * 1e6, 1)
    return out


# ------------------------------------------------------------------ CPU legs
def _ref_batch(lib, cfg, rows, threads):
    import ctypes

    P = ctypes.c_void_p
    x = np.ascontiguousarray(cfg["logits"][rows])
    p = cfg["params"][rows]
    T = np.ascontiguousarray(p["temperature"], np.float32)
    k = np.ascontiguousarray(p["top_k"], np.int32)
    tp = np.ascontiguousarray(p["top_p"], np.float32)
    rep = np.ascontiguousarray(p["repetition_penalty"], np.float32)
    lb = np.ascontiguousarray(p["repetition_lookback"], np.int32)
    h = np.ascontiguousarray(cfg["hist"][rows])
    hl = np.ascontiguousarray(cfg["hist_len"][rows])
    seeds = np.ascontiguousarray(cfg["seeds"][rows], np.uint32)
    out = np.empty(len(rows), np.int32)
    f = lambda a: a.ctypes.data_as(P)
    lib.qwref_temperature_sample_batch(f(x), len(rows), x.shape[1], x.shape[1], f(T), f(k), f(tp), f(rep), f(lb), f(h),
                                       h.shape[1], f(hl), f(seeds), f(out), threads)
    return out


def c1_latency():
    """Per-call latency of one row (C1 shape) through the drop-in C++ samplers
    (CudaTemperatureSampler / CudaGreedySampler: host logits, qsamp_sample_host)
    and through the reference's own samplers, from oracle/_ref/adapter_check,
    which links both."""
    exe = os.path.join(ROOT, "oracle", "_ref", "adapter_check")
    if not os.path.exists(exe):
        return None
    try:
        r = subprocess.run([exe, "--time", "100"], capture_output=True, text=True, timeout=300)
        return json.loads(r.stdout.strip().splitlines()[-1]) if r.returncode == 0 else None
    except Exception:
        return None


def cpu_baseline(cfgs, seconds=10.0):
    """The reference's own CPU sampler (Release build) on the host cores, over
    the same rotating batches."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    threads = os.cpu_count() or 1
    B = len(cfgs[0]["params"])
    done, t0, i = 0, time.perf_counter(), 0
    if O.ref_available("release"):
        lib = O.ref_lib("release")
        kind = "reference"
        while time.perf_counter() - t0 < seconds:
            _ref_batch(lib, cfgs[i % len(cfgs)], np.arange(B), threads)
            done += B
            i += 1
        el = time.perf_counter() - t0
        sample = (f"{done} rows of the config2-B256 batches (seeds {', '.join(map(str, BATCH_SEEDS))}) through "
                  "TemperatureSampler::sample (frequency/presence have no reference code and are off), one sampler "
                  f"per row, {threads} std::threads")
    else:
        kind = "port"
        while time.perf_counter() - t0 < seconds:
            c = cfgs[i % len(cfgs)]
            O.oracle_sample(c["logits"], c["params"], c["hist"], c["hist_len"], None, c["u"], n_threads=threads)
            done += B
            i += 1
        el = time.perf_counter() - t0
        sample = f"{done} rows of config2-B256 through the C restatement, {threads} threads"
    out = {"value": round(done / el, 2), "unit": "rows/s", "cores": threads, "cpu_model": cpu_model(), "kind": kind,
           "sample": sample}
    lat = c1_latency()
    if lat:
        out["c1_latency_ms"] = lat
    return out


def run_reference(args):
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    from qwenium_b200 import workloads as W

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    if not O.ref_available("release"):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqwref_release.so was not built"}))
        return
    cfgs = [W.config2(seed=s, B=args.batch) for s in BATCH_SEEDS]
    lib = O.ref_lib("release")
    threads = os.cpu_count() or 1
    # each step: a bounded sample of one B-row batch (whole rows, all cores),
    # the steps rotating over the four batches; the reference's cost per row
    # is its full std::sort of V pairs whatever the row's top-k, so a sample
    # of rows gives the batch's rows/s
    rows_per_step = max(threads, min(args.batch, 4 * threads))
    rows = np.arange(rows_per_step) % args.batch
    for i in range(args.warmup):
        _ref_batch(lib, cfgs[i % len(cfgs)], rows, threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        _ref_batch(lib, cfgs[i % len(cfgs)], rows, threads)
    el = time.perf_counter() - t0
    v = rows_per_step * args.steps / el
    out = {
        "impl": "reference",
        "metric": "sampled rows/s (batched token selection, B=256, V=151936)",
        "value": round(v, 2),
        "unit": "rows/s",
        "n_gpus": env_int("WORLD_SIZE", 1),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded config-2 distribution)",
        "config": {"workload": "config2-B256: batched server decode parameters at B=256, V=151936 fp32",
                   "rows_per_step": rows_per_step, "V": V, "batch_seeds": list(BATCH_SEEDS),
                   "note": "each step samples rows_per_step of a B=256 batch: the reference's per-row cost is its "
                           "full std::sort of V pairs whatever the row's top-k, so the sample gives the batch's "
                           "rows/s"},
        "cpu_baseline": {"value": round(v, 2), "unit": "rows/s", "cores": threads, "cpu_model": cpu_model(),
                         "kind": "reference",
                         "sample": f"{rows_per_step} rows per step through TemperatureSampler::sample (Release "
                                   "flags, frequency/presence off: no reference code)"},
        "e2e": {"value": round(v, 2), "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="qsamp", choices=["qsamp", "reference"])
    ap.add_argument("--batch", type=int, default=B_DEFAULT)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-b10", action="store_true")
    ap.add_argument("--no-c4", action="store_true")
    ap.add_argument("--no-vshard", action="store_true")
    ap.add_argument("--extras", action="store_true",
                    help="also time C4 at B=1024, draft verification and char-class masks (rank 0)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
