#!/usr/bin/env python
"""Benchmark of the B200 token-selection path (qsamp).

Workload (N=1): the batched-server-decode parameter distribution
(per-row T~U[0.2,1.2], top-k in {0,20,40,100}, top-p~U[0.8,1.0],
frequency/presence penalties over a 256-id history) at B=256, V=151936, fp32
logits -- the B=256 / V=151936 point of the headline metric. A step is one
batched selection call over B rows. Under torchrun every rank runs its own B
rows (weak scaling, no collective on the data path).

  value  -- rows/s over all ranks, inputs resident in HBM, device-timed with
            CUDA events (max over ranks); inputs rotate over copies whose
            total exceeds L2, so every step reads logits from HBM.
  e2e    -- the same through qsamp_sample_host: pinned host logits, history
            and params copied in, ids and results copied out, every step.
  roofline -- algorithmic bytes of the selection kernel per launch over its
            mean launch time, against the measured HBM copy bandwidth.

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
BATCH_SEED = 1000  # the config2-B256 batch every rank serves


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


def stream_rows(params, V_, window=HIST):
    """Rows the library routes to the stream kernel (qsamp_api.cu's rule):
    greedy rows and 0 < top_k <= 1024, top_k < V, with a penalty window of at
    most 1024 ids; the rest go to the cluster kernel."""
    T, k = params["temperature"], params["top_k"]
    return (T <= 0) | ((k > 0) & (k <= 1024) & (k < V_) & (window <= 1024))


def algorithmic_bytes_per_row(V_, hist_len, bytes_per_logit=4, mask=False):
    # logits + allow-mask words + history ids + params/u/result per row
    return V_ * bytes_per_logit + (((V_ + 31) // 32) * 4 if mask else 0) + 4 * hist_len + 64


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
    # weak scaling: every rank serves the same seeded batch of B rows on its
    # own GPU (fixed work per GPU; batches of other seeds differ in their mix
    # of full-vocabulary rows, and the max over ranks would then time the
    # heaviest batch rather than the scaling)
    cfg = W.config2(seed=BATCH_SEED, B=B)
    ctx = qsamp.Context(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    # rotating copies: > 2x L2 between reuses of a buffer
    bytes_one = B * V * 4
    ncopies = max(2, int(np.ceil(3 * 126e6 / bytes_one)) + 1)
    xs = [torch.from_numpy(cfg["logits"]).to(dev) for _ in range(ncopies)]
    hist = torch.from_numpy(cfg["hist"]).to(dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    res = torch.empty((B, 32), dtype=torch.uint8, device=dev)

    def step(i):
        ctx.sample_batch(xs[i % ncopies], cfg["params"], hist=hist, hist_len=cfg["hist_len"], u=cfg["u"],
                         out_ids=ids, out_results=res, stream=stream.cuda_stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ctx.counters()["kernel_launches"]
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
    gpu_launches = int(ctx.counters()["kernel_launches"] - launches0)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    # per-kernel device time: the same steps with the library's own events
    # around each kernel launch (on the launching stream)
    ctx.set_kernel_timing(True)
    per_stream, per_rows = [], []
    for i in range(min(args.steps, 20)):
        step(i)
        c = ctx.counters()
        per_stream.append(c["last_stream_kernel_ms"])
        per_rows.append(c["last_rows_kernel_ms"])
    ctx.set_kernel_timing(False)
    k_stream, k_rows = statistics.mean(per_stream), statistics.mean(per_rows)
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())

    # e2e through the host entry point with pinned buffers
    e2e_rows_s = None
    h2d = d2h = 0
    if not args.no_e2e:
        hx = torch.from_numpy(cfg["logits"]).pin_memory()
        hh = torch.from_numpy(cfg["hist"]).pin_memory()
        hl = cfg["hist_len"]
        e2e_steps = max(3, min(args.steps, 20))
        for _ in range(2):
            ctx.sample_host(hx.numpy(), cfg["params"], hist=hh.numpy(), hist_len=hl, u=cfg["u"])
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ctx.sample_host(hx.numpy(), cfg["params"], hist=hh.numpy(), hist_len=hl, u=cfg["u"])
        el = time.perf_counter() - t0
        el_t = torch.tensor([el], device=dev)
        if world > 1:
            dist.all_reduce(el_t, op=dist.ReduceOp.MAX)
        e2e_rows_s = world * B * e2e_steps / float(el_t.item())
        h2d = B * V * 4 + B * HIST * 4 + B * (48 + 8 + 4)
        d2h = B * (4 + 32)

    # B=10 latency point (device-timed, same parameter distribution)
    b10 = None
    if rank == 0 and not args.no_b10:
        c10 = W.config2(seed=77, B=10)
        x10 = [torch.from_numpy(c10["logits"]).to(dev) for _ in range(8)]
        h10 = torch.from_numpy(c10["hist"]).to(dev)
        i10 = torch.empty(10, dtype=torch.int32, device=dev)
        for i in range(5):
            ctx.sample_batch(x10[i % 8], c10["params"], hist=h10, hist_len=c10["hist_len"], u=c10["u"], out_ids=i10)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n10 = 50
        a.record(stream)
        for i in range(n10):
            ctx.sample_batch(x10[i % 8], c10["params"], hist=h10, hist_len=c10["hist_len"], u=c10["u"], out_ids=i10,
                             stream=stream.cuda_stream)
        b.record(stream)
        torch.cuda.synchronize()
        t10 = a.elapsed_time(b) / n10
        b10 = {"ms_per_step": round(t10, 4), "rows_per_s": round(10 / (t10 * 1e-3), 1)}

    extras = run_extras(ctx, dev, stream) if (rank == 0 and args.extras) else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, seconds=args.cpu_seconds)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = measured_peaks()
    n_stream = int(stream_rows(cfg["params"], V).sum())
    if k_rows >= k_stream:
        kname, units, launch_ms = "qs_rows_kernel", B - n_stream, k_rows
    else:
        kname, units, launch_ms = "qs_stream_kernel", n_stream, k_stream
    alg = algorithmic_bytes_per_row(V, HIST) * units
    achieved = alg / (launch_ms * 1e-3) / 1e9
    traffic = ncu_traffic(f"{kname}/config2-B256")
    ms_step = ms / args.steps
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
                   "batch_seed": BATCH_SEED,
                   "l2": f"rotating {ncopies} input copies ({ncopies * bytes_one / 1e6:.0f} MB) > L2"},
        "e2e": {"value": round(e2e_rows_s, 1) if e2e_rows_s else None, "unit": "rows/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": gpu_launches,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                     "kernel": kname, "rows_per_launch": units, "bytes_per_launch": alg,
                     "launch_ms": round(launch_ms, 4),
                     "kernels_ms": {"qs_stream_kernel": round(k_stream, 4), "qs_rows_kernel": round(k_rows, 4)}},
        "clocks": clk.summary(),
    }
    if b10:
        out["b10"] = b10
    if extras:
        out["extras"] = extras
    if cpu:
        out["cpu_baseline"] = cpu
    print(json.dumps(out))


def _events_ms(stream, fn, reps):
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(reps):
        fn(i)
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_extras(ctx, dev, stream):
    """Secondary measurements (device-timed, inputs resident, rotating buffers):
    C4 (bf16 V=262144, soft-cap, full-vocabulary top-p), batched greedy draft
    verification and grammar char-class masks; with the reference's own CPU
    time per unit where it compiled (oracle/_ref)."""
    import ctypes

    import torch

    from qwenium_b200 import qsamp
    from qwenium_b200 import workloads as W

    out = {}
    peak, _ = measured_peaks()
    # C4 at B=256: every row takes the cluster kernel
    c4 = W.config4(4, B=256)
    xs = [torch.from_numpy(np.ascontiguousarray(c4["logits"]).view(np.int16)).to(dev) for _ in range(2)]
    h4 = torch.from_numpy(c4["hist"]).to(dev)
    f4 = lambda i: ctx.sample_batch(xs[i % 2], c4["params"], hist=h4, hist_len=c4["hist_len"], u=c4["u"],
                                    stream=stream.cuda_stream)
    for i in range(3):
        f4(i)
    ms = _events_ms(stream, f4, 5)
    out["config4_B256"] = {"ms_per_call": round(ms, 4), "rows_per_s": round(256 / (ms * 1e-3), 1)}
    # C4 at B=1024 (its own seeded batch; two copies on the device, 1.07 GB)
    del xs
    c4 = W.config4(4, B=1024)
    xs = [torch.from_numpy(np.ascontiguousarray(c4["logits"]).view(np.int16)).to(dev) for _ in range(2)]
    h4 = torch.from_numpy(c4["hist"]).to(dev)
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


def cpu_baseline(cfg, seconds=10.0):
    """The reference's own CPU sampler (Release build) on the host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    threads = os.cpu_count() or 1
    if O.ref_available("release"):
        lib = O.ref_lib("release")
        kind = "reference"
        B = len(cfg["params"])
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rows = np.arange(B)
            _ref_batch(lib, cfg, rows, threads)
            done += B
        el = time.perf_counter() - t0
        sample = (f"{done} rows of the config2-B256 workload through TemperatureSampler::sample "
                  "(frequency/presence have no reference code and are off), one sampler per row, "
                  f"{threads} std::threads")
    else:
        kind = "port"
        B = len(cfg["params"])
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            O.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None, cfg["u"],
                            n_threads=threads)
            done += B
        el = time.perf_counter() - t0
        sample = f"{done} rows of config2-B256 through the C restatement, {threads} threads"
    return {"value": round(done / el, 2), "unit": "rows/s", "cores": threads, "kind": kind, "sample": sample}


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
    cfg = W.config2(seed=1000, B=args.batch)
    lib = O.ref_lib("release")
    threads = os.cpu_count() or 1
    # each step: a bounded sample of the B-row workload (whole rows, all cores)
    rows_per_step = max(threads, min(args.batch, 4 * threads))
    rows = np.arange(rows_per_step) % args.batch
    for _ in range(args.warmup):
        _ref_batch(lib, cfg, rows, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _ref_batch(lib, cfg, rows, threads)
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
                   "rows_per_step": rows_per_step, "V": V},
        "cpu_baseline": {"value": round(v, 2), "unit": "rows/s", "cores": threads, "kind": "reference",
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
    ap.add_argument("--extras", action="store_true",
                    help="also time C4 (bf16, V=262144), draft verification and char-class masks (rank 0)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
