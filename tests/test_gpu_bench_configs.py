"""GPU parity on the benchmarked shapes themselves.

The configurations whose throughput is reported run here in full, through
the C ABI, against the C restatement (bit for bit, every field):

* C4 at B=256 and B=1024 (bf16, V=262144, soft-cap 30, full-vocabulary
  top-p): these batch sizes take the launch plan the C4 numbers come from,
  and the test asserts that plan (CTAs per cluster), so a planner change
  cannot leave the measured shape untested;
* C5 at B=512 (V=262144, k=64, p=0.95) through the vocab-sharded path at
  N=2/4/8 emulated ranks, against the unsharded path and the oracle.

The tests sit in a file that sorts before the long parity files, so that a
run stopping at the first failure reaches them early.
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIELDS = ("token", "position", "n_keep", "drew", "sum_exp", "sum_keep", "max_logit", "prob")

# CTAs per cluster the planner picks for bf16 rows of V=262144 at B >= 256 on
# a B200 (148 SMs, 227 KB of shared memory per CTA): two clusters of 9 per GPC
C4_CLUSTER = 9


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    return qsamp.Context(0)


def diff_rows(got, want):
    bad = []
    for b in range(len(want)):
        for f in FIELDS:
            g, w = got[b][f], want[b][f]
            if f in FIELDS[:4]:
                ok = int(g) == int(w)
            else:
                ok = np.float32(g).view(np.uint32) == np.float32(w).view(np.uint32) or (np.isnan(g) and np.isnan(w))
            if not ok:
                bad.append((b, f, g, w))
    return bad


def run_device(ctx, cfg):
    import torch

    from qwenium_b200 import qsamp

    x = cfg["logits"]
    dx = torch.from_numpy(np.ascontiguousarray(x).view(np.int16) if cfg["bf16"] else x).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda() if cfg.get("hist") is not None else None
    res = ctx.sample_batch(dx, cfg["params"], hist=hist, hist_len=cfg.get("hist_len"), u=cfg["u"])
    torch.cuda.synchronize()
    ctx.poll_status()
    return res.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1)


@pytest.mark.parametrize("B", [256, 1024])
def test_config4_full_batch(ctx, oracle_mod, B):
    """Both paths a C4 row can take: the histogram kernel (the default for
    bf16 full-vocabulary rows) and, with it switched off, the cluster kernel
    with its 9-CTA plan (which also serves any row the histogram kernel hands
    on)."""
    cfg = W.config4(4, B=B)
    want, _, _, _ = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None,
                                             cfg["u"], bf16=True)
    try:
        ctx.set_limits(hist_path=0)
        got = run_device(ctx, cfg)
        c = ctx.counters()
        assert c["last_cluster_rows"] == B and c["last_stream_rows"] == 0 and c["last_hist_rows"] == 0
        assert c["last_cluster_size"] == C4_CLUSTER, c
        assert c["last_clusters"] < B  # rows come from the queue
        bad = diff_rows(got, want)
        assert not bad, f"C4 B={B}, cluster kernel: {len(bad)} mismatches, first {bad[:6]}"
    finally:
        ctx.set_limits(hist_path=1)
    got = run_device(ctx, cfg)
    c = ctx.counters()
    assert c["last_hist_rows"] == B and c["last_cluster_rows"] == 0, c
    bad = diff_rows(got, want)
    assert not bad, f"C4 B={B}, histogram kernel: {len(bad)} mismatches, first {bad[:6]}"


@pytest.fixture(scope="module")
def c5(ctx, oracle_mod):
    cfg = W.config5(5, B=512)
    cfg["hist"] = np.zeros((512, 1), np.int32)
    cfg["hist_len"] = np.zeros(512, np.int32)
    want, _, _, _ = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], None, None, None, cfg["u"])
    base = run_device(ctx, cfg)
    bad = diff_rows(base, want)
    assert not bad, f"C5 unsharded: {len(bad)} mismatches, first {bad[:6]}"
    return cfg, want


@pytest.mark.parametrize("n_ranks", [2, 4, 8])
def test_config5_sharded(ctx, c5, n_ranks):
    from test_gpu_vshard import run_sharded

    cfg, want = c5
    got = run_sharded(ctx, cfg, n_ranks)
    bad = diff_rows(got, want)
    assert not bad, f"C5 N={n_ranks}: {len(bad)} mismatches, first {bad[:6]}"
