"""GPU parity of the live-list path (fp32 rows with a full-vocabulary top-p).

With live_path 1 such rows are shared between the cluster kernel and the
live-list kernel:
the cluster kernel claims them from the front of a list ordered by falling
temperature, the live-list kernel from the back. The live-list kernel serves
a row whose elements within 17.5 of the maximum number at most 4096 (sorted
in shared memory; the histogram path's group walks add the sums) and returns
any other row to the cluster kernel. Every field of every row must equal the
C restatement's and the cluster kernel's alone (live path off), bit for bit,
whichever kernel served it: on the config2 batches, on random fp32 rows
(peaked and flat, duplicate-heavy, soft-capped, masked, penalised windows
holding the maximum), on rows built to be returned, and with every row
returned (live_path 2: the second cluster launch serves them all).
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIELDS = ("token", "position", "n_keep", "drew", "sum_exp", "sum_keep", "max_logit", "prob")


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    c = qsamp.Context(0)
    yield c
    c.set_limits(live_path=0)


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


def run(ctx, cfg, live_path=1, philox=False):
    import torch

    from qwenium_b200 import qsamp

    ctx.set_limits(live_path=live_path)
    dx = torch.from_numpy(np.ascontiguousarray(cfg["logits"], np.float32)).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda() if cfg.get("hist") is not None else None
    masks = torch.from_numpy(cfg["masks"].view(np.int32)).cuda() if cfg.get("masks") is not None else None
    res = ctx.sample_batch(dx, cfg["params"], hist=hist, hist_len=cfg.get("hist_len"), masks=masks,
                           u=None if philox else cfg["u"], rng_offset=7)
    torch.cuda.synchronize()
    ctx.poll_status()
    return res.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1), ctx.counters()


def oracle(O, cfg):
    out, _, _, _ = O.oracle_sample(cfg["logits"], cfg["params"], cfg.get("hist"), cfg.get("hist_len"),
                                   cfg.get("masks"), cfg["u"])
    return out


def full_rows(cfg):
    p = cfg["params"]
    V = cfg["logits"].shape[1]
    k = p["top_k"]
    return int(np.sum((p["temperature"] > 0) & ((k <= 0) | (k >= V)) & (p["top_p"] > 0) & (p["top_p"] < 1)))


@pytest.mark.parametrize("seed", [1000, 2000, 3000])
def test_config2_batch(ctx, oracle_mod, seed):
    cfg = W.config2(seed, B=256)
    got, c = run(ctx, cfg)
    print(f"\nconfig2 seed {seed}: {c['last_live_candidates']} shared rows, the live-list kernel served "
          f"{c['last_live_rows']} and returned {c['last_live_returned']}")
    assert c["last_live_candidates"] == full_rows(cfg), c
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"
    assert c["last_live_rows"] > 0, c
    alone, c0 = run(ctx, cfg, live_path=0)
    assert c0["last_live_candidates"] == 0, c0
    bad = diff_rows(got, alone)
    assert not bad, f"live path vs cluster kernel alone: {len(bad)} mismatches, first {bad[:6]}"


def test_config2_all_returned(ctx, oracle_mod):
    """live_path 2: the live-list kernel returns every row it takes after its
    passes; the first cluster launch serves none of them, the second all."""
    cfg = W.config2(1000, B=256)
    got, c = run(ctx, cfg, live_path=2)
    assert c["last_live_rows"] == 0 and c["last_live_returned"] > 0, c
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"


def test_philox_mode(ctx):
    """u == NULL (the in-kernel Philox uniforms): both paths draw alike."""
    cfg = W.config2(2000, B=128)
    got, _ = run(ctx, cfg, philox=True)
    alone, _ = run(ctx, cfg, live_path=0, philox=True)
    bad = diff_rows(got, alone)
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"


def _random_fp32(seed, B, V):
    rng = np.random.default_rng(seed)
    x = np.empty((B, V), np.float32)
    for b in range(B):
        kind = b % 6
        if kind == 0:  # peaked: a few boosted ids over noise
            x[b] = rng.standard_normal(V) * 1.5
            x[b, rng.choice(V, 40, replace=False)] += rng.uniform(8, 20)
        elif kind == 1:  # a Zipf head over noise
            x[b] = rng.standard_normal(V) * 2
            x[b, rng.permutation(V)] += 1.1 * (np.log(V) - np.log(np.arange(1, V + 1)))
        elif kind == 2:  # few distinct values (heavy duplicates, ties at the maximum)
            x[b] = rng.integers(-8, 9, V) * 0.5
            x[b, rng.choice(V, 300, replace=False)] = 9.0
        elif kind == 3:  # a wide spread
            x[b] = rng.standard_normal(V) * 12
        elif kind == 4:  # flat: nearly every element within reach of the maximum
            x[b] = rng.standard_normal(V) * 0.5
        else:  # bf16-valued logits (runs of equal values) with a peak
            x[b] = W.bf16_bits_to_f32(W.f32_to_bf16_bits(rng.standard_normal(V).astype(np.float32) * 3))
            x[b, rng.integers(0, V)] = 25.0
    p = W.default_params(B)
    p["temperature"] = rng.choice([0.2, 0.5, 0.8, 1.0, 1.5], B)
    p["top_k"] = rng.choice([0, 0, V, V + 7], B)
    p["top_p"] = rng.choice([0.5, 0.8, 0.9, 0.95, 0.99], B)
    p["repetition_penalty"] = rng.choice([1.0, 1.05, 1.3], B)
    p["repetition_lookback"] = rng.choice([16, 64, 512], B)
    p["frequency_penalty"] = rng.choice([0.0, 0.2], B)
    p["presence_penalty"] = rng.choice([0.0, 0.3], B)
    p["softcap"] = rng.choice([0.0, 0.0, 30.0], B)
    H = 600
    hist = rng.integers(0, V, size=(B, H), dtype=np.int64).astype(np.int32)
    hist[:, -3:] = np.argsort(-x, axis=1)[:, :3].astype(np.int32)  # windows holding the maximum
    hl = rng.integers(0, H + 1, size=B).astype(np.int32)
    hl[::3] = H
    masks = None
    if seed % 2:
        keep = rng.random((B, V)) < 0.7
        keep[:, 0] = True
        words = (V + 31) // 32
        pad = np.zeros((B, words * 32), np.uint8)
        pad[:, :V] = keep
        masks = np.packbits(pad, axis=1, bitorder="little").view(np.uint32).reshape(B, words)
    seeds = rng.integers(0, 2**32, size=B, dtype=np.uint64).astype(np.uint32)
    return dict(name=f"fp32-random-{seed}", logits=x, bf16=False, params=p, hist=hist, hist_len=hl,
                masks=masks, seeds=seeds, u=W.uniforms_for(seeds))


@pytest.mark.parametrize("seed,V", [(1, 1000), (2, 4099), (3, 65536), (4, 151936), (5, 262144)])
def test_random_fp32_rows(ctx, oracle_mod, seed, V):
    cfg = _random_fp32(seed, 36, V)
    got, c = run(ctx, cfg)
    assert c["last_live_candidates"] == full_rows(cfg), c
    print(f"\nV={V}: {c['last_live_candidates']} shared rows, live-list kernel served {c['last_live_rows']}, "
          f"returned {c['last_live_returned']}")
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"live path vs oracle: {len(bad)} mismatches, first {bad[:6]}"
    alone, _ = run(ctx, cfg, live_path=0)
    bad = diff_rows(got, alone)
    assert not bad, f"live path vs cluster kernel alone: {len(bad)} mismatches, first {bad[:6]}"
    every, c2 = run(ctx, cfg, live_path=2)
    assert c2["last_live_rows"] == 0, c2
    bad = diff_rows(every, alone)
    assert not bad, f"every row returned vs cluster kernel alone: {len(bad)} mismatches, first {bad[:6]}"


def test_rows_returned(ctx, oracle_mod):
    """Rows the live-list kernel returns, beside rows it keeps: one value
    everywhere (V live elements), exactly 4096 and 4097 elements tied at the
    maximum, -inf logits, a top-p of 0.999 over a flat row, every element
    masked but one."""
    V = 20000
    B = 12
    rng = np.random.default_rng(77)
    x = (rng.standard_normal((B, V)) * 0.3 - 40.0).astype(np.float32)
    x[0] = 1.0                                   # one value everywhere
    x[1, :4096] = 5.0                            # exactly 4096 live (ties at the maximum)
    x[2, :4097] = 5.0                            # 4097 live
    x[3, ::2] = -np.inf                          # -inf logits beside finite ones
    x[3, 123] = 3.0
    x[4] = rng.standard_normal(V).astype(np.float32)  # flat, top-p 0.999
    x[5, 7] = 3.0                                # a single live element
    x[6, 100:140] = 2.0                          # a few ties
    for b in range(7, B):                        # peaked rows kept by the live-list kernel
        x[b, rng.choice(V, 500, replace=False)] += rng.uniform(30, 45)
    p = W.default_params(B)
    p["temperature"] = 0.7
    p["top_k"] = 0
    p["top_p"] = 0.9
    p["top_p"][4] = 0.999
    keep = np.ones((B, V), bool)
    keep[8] = False
    keep[8, 4321] = True                         # every element masked but one
    words = (V + 31) // 32
    pad = np.zeros((B, words * 32), np.uint8)
    pad[:, :V] = keep
    masks = np.packbits(pad, axis=1, bitorder="little").view(np.uint32).reshape(B, words)
    seeds = np.arange(B, dtype=np.uint32) + np.uint32(99)
    cfg = dict(name="returned", logits=x, bf16=False, params=p, hist=None, hist_len=None, masks=masks,
               seeds=seeds, u=W.uniforms_for(seeds))
    got, c = run(ctx, cfg)
    print(f"\nreturned rows: {c['last_live_returned']} of {c['last_live_candidates']} "
          f"(served {c['last_live_rows']})")
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"
    alone, _ = run(ctx, cfg, live_path=0)
    bad = diff_rows(got, alone)
    assert not bad, f"live path vs cluster kernel alone: {len(bad)} mismatches, first {bad[:6]}"


def test_limits_validation(ctx):
    from qwenium_b200 import qsamp

    with pytest.raises(qsamp.QsampError):
        ctx.set_limits(live_path=3)
    ctx.set_limits(live_path=1)
    assert ctx.limits()["live_path"] == 1
    ctx.set_limits(live_path=0)
