"""Per-row phase timing of qs_rows_kernel (profiling build).

Builds ``libqsamp_phase.so`` (the library compiled with ``-DQS_PHASE_TIMING``:
thread 0 of each cluster's leading CTA stamps %globaltimer at the phase
boundaries of every row it serves and sums clock64 cycles of the leader's
sub-phases), runs the config2-B256 batch on one GPU and prints the mean time
of each phase per row, the gathered-list lengths per pass, and the rows'
total work against the kernel's span.

    python -m qwenium_b200.phase_timing --build     # here or on the GPU box
    python -m qwenium_b200.phase_timing             # on a GPU box

The shipped library (``libqsamp.so``) has none of these stamps. Slot numbers
follow the QS_TMARK / QS_SUB / QS_NOTE calls in csrc/qsamp_kernels.cu.
"""
from __future__ import annotations

import ctypes
import os
import statistics
import subprocess
import sys

import numpy as np

from . import build as B

OUT = os.path.join(B.HERE, "libqsamp_phase.so")
SLOTS = 48
SUB = ["ksum prefix", "sort block", "S walk", "S re-prediction", "top-p predictions", "cumulative walk",
       "top-p re-prediction", "draw", "finish", "gather set"]
SORT_SUB = {16: "zero fill", 17: "bitonic sort", 18: "expf of the list"}


def build_phase_lib() -> str:
    cmd = [B.nvcc(), "-shared", *B.ARCH, *B.FLAGS, "-DQS_PHASE_TIMING", "-o", OUT, *B.SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    return OUT


def run(seed: int = 1000, B_rows: int = 256, sm_mhz: float = 1965.0) -> None:
    import torch

    from . import qsamp, workloads as W

    lib = qsamp.load(OUT)
    cfg = W.config2(seed=seed, B=B_rows)
    ctx = qsamp.Context(0)
    dev = torch.device("cuda", 0)
    xs = [torch.from_numpy(cfg["logits"]).to(dev) for _ in range(4)]
    hist = torch.from_numpy(cfg["hist"]).to(dev)
    ids = torch.empty(B_rows, dtype=torch.int32, device=dev)
    res = torch.empty((B_rows, 32), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    def step(i):
        ctx.sample_batch(xs[i % 4], cfg["params"], hist=hist, hist_len=cfg["hist_len"], u=cfg["u"], out_ids=ids,
                         out_results=res, stream=st.cuda_stream)

    for i in range(5):
        step(i)
    torch.cuda.synchronize()
    lib.qs_phase_clear.restype = ctypes.c_int
    lib.qs_phase_read.restype = ctypes.c_int
    if lib.qs_phase_clear() != 0:
        raise RuntimeError("qs_phase_clear failed")
    step(5)
    torch.cuda.synchronize()
    ph = np.zeros((8192, SLOTS), np.uint64)
    if lib.qs_phase_read(ph.ctypes.data_as(ctypes.c_void_p)) != 0:
        raise RuntimeError("qs_phase_read failed")
    ph = ph[:B_rows].astype(np.int64)
    crow = [r for r in range(B_rows) if ph[r, 5] != 0]  # rows that took the full-vocabulary path
    if not crow:
        print("no full-vocabulary rows")
        return
    t0 = min(ph[r, 0] for r in crow)
    us = lambda a: a / 1000.0  # noqa: E731  (globaltimer ns)
    rows = []
    for r in crow:
        t = ph[r]
        nit = int(t[23])
        d = dict(row=r, start=us(t[0] - t0), total=us(t[4] - t[0]), pen=us(t[1] - t[0]),
                 xf=us(t[2] - t[1]), mx=us(t[3] - t[2]), cnt=us(t[5] - t[3]), red=us(t[6] - t[5]),
                 pred=us(t[7] - t[6]), nit=nit)
        prev, pas, rd = t[7], [], []
        for i in range(min(nit + 1, 5)):
            a, b_, c = t[8 + 3 * i], t[9 + 3 * i], t[10 + 3 * i]
            if a == 0:
                break
            pas.append(us(a - prev))
            rd.append(us(b_ - a) if b_ else 0.0)
            prev = c if c else (b_ if b_ else a)
        d["pass"], d["red2"] = pas, rd
        d["spec"] = [int(t[35 + i]) for i in range(min(nit + 1, 5))]
        rows.append(d)
    mean = lambda f: statistics.mean(f(d) for d in rows)  # noqa: E731
    print(f"rows on the cluster kernel: {len(rows)}")
    for k, name in [("pen", "penalty table"), ("xf", "transform"), ("mx", "cluster max"), ("cnt", "bin counts"),
                    ("red", "cluster reduction"), ("pred", "first predictions")]:
        print(f"  {name:28s} {mean(lambda d: d[k]):7.1f} us")
    print(f"  {'first element pass':28s} {mean(lambda d: d['pass'][0]):7.1f} us")
    print(f"  {'later passes':28s} {mean(lambda d: sum(d['pass'][1:])):7.1f} us")
    print(f"  {'reductions after passes':28s} {mean(lambda d: sum(d['red2'])):7.1f} us")
    for j, name in list(enumerate(SUB)) + list(SORT_SUB.items()):
        v = statistics.mean(ph[d["row"], 24 + j] for d in rows) / sm_mhz
        print(f"  CTA 0: {name:21s} {v:7.1f} us")
    print(f"  {'whole row (mean / median)':28s} {mean(lambda d: d['total']):7.1f} / "
          f"{statistics.median(d['total'] for d in rows):.1f} us")
    flat = sorted(x for d in rows for x in d["spec"])
    print("gathered list per pass, quantiles 0/.5/.9/1:",
          [flat[int(q * (len(flat) - 1))] for q in (0, .5, .9, 1)])
    end = max(d["start"] + d["total"] for d in rows)
    print(f"work {sum(d['total'] for d in rows):.0f} us over the rows, span {end:.1f} us")

    # stream kernel rows (one CTA per row): marks 0-4 only
    srow = [r for r in range(B_rows) if ph[r, 0] != 0 and ph[r, 5] == 0 and ph[r, 4] != 0]
    if srow:
        p = cfg["params"]
        st_rows = [dict(k=int(p["top_k"][r]), win=us(ph[r, 1] - ph[r, 0]), stream=us(ph[r, 2] - ph[r, 1]),
                        select=us(ph[r, 3] - ph[r, 2]), finish=us(ph[r, 4] - ph[r, 3]), total=us(ph[r, 4] - ph[r, 0]),
                        start=us(ph[r, 0] - t0)) for r in srow]
        print(f"rows on the stream kernel: {len(st_rows)}")
        # thread 0's clock64 sums over the chunk loop: loads + raw filter, exact path, super-chunk barriers
        for j, name in enumerate(["loads + raw filter", "exact path", "barriers + compactions"]):
            v = statistics.mean(ph[r, 24 + j] for r in srow) / sm_mhz
            print(f"  stream loop: {name:21s} {v:7.1f} us")
        for k, name in [("win", "penalty window table"), ("stream", "stream of the row"),
                        ("select", "last compaction + sort"), ("finish", "top-p, softmax, draw"),
                        ("total", "whole row")]:
            print(f"  {name:28s} {statistics.mean(d[k] for d in st_rows):7.1f} us")
        for kk in sorted({d["k"] for d in st_rows}):
            sel = [d for d in st_rows if d["k"] == kk]
            print(f"  top_k {kk:4d}: {len(sel):3d} rows, stream {statistics.mean(d['stream'] for d in sel):6.1f} us, "
                  f"whole row {statistics.mean(d['total'] for d in sel):6.1f} us")
        print(f"  span {max(d['start'] + d['total'] for d in st_rows):.1f} us")


if __name__ == "__main__":
    if "--build" in sys.argv:
        print(build_phase_lib())
    else:
        run()
