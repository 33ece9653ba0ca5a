"""GPU parity of the histogram path (bf16 rows with a full-vocabulary top-p).

The histogram kernel answers such rows from counts of their bf16 values
(runs of equal terms added in closed form) and hands any row it cannot prove
exact to the cluster kernel. Every field of every row must equal the C
restatement's and the cluster kernel's (the same call with the histogram path
off), bit for bit, on the C4 batches, on random bf16 rows (duplicate-heavy,
soft-capped or not, masked, penalised windows holding the maximum) and on
rows built to be handed on.
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
    c.set_limits(hist_path=1)


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


def run(ctx, cfg, hist_path=1):
    import torch

    from qwenium_b200 import qsamp

    ctx.set_limits(hist_path=hist_path)
    bits = np.ascontiguousarray(cfg["logits"])
    dx = torch.from_numpy(bits.view(np.int16)).cuda()
    hist = torch.from_numpy(cfg["hist"]).cuda() if cfg.get("hist") is not None else None
    masks = torch.from_numpy(cfg["masks"].view(np.int32)).cuda() if cfg.get("masks") is not None else None
    res = ctx.sample_batch(dx, cfg["params"], hist=hist, hist_len=cfg.get("hist_len"), masks=masks, u=cfg["u"])
    torch.cuda.synchronize()
    ctx.poll_status()
    return res.cpu().numpy().view(qsamp.ROW_RESULT).reshape(-1), ctx.counters()


def oracle(O, cfg):
    out, _, _, _ = O.oracle_sample(cfg["logits"], cfg["params"], cfg.get("hist"), cfg.get("hist_len"),
                                   cfg.get("masks"), cfg["u"], bf16=True)
    return out


@pytest.mark.parametrize("seed", [4, 44])
def test_config4_batch(ctx, oracle_mod, seed):
    cfg = W.config4(seed, B=256)
    got, c = run(ctx, cfg)
    assert c["last_hist_rows"] == 256, c
    print(f"\nC4 seed {seed}: {c['last_hist_handed_on']} of 256 rows handed on to the cluster kernel")
    assert c["last_hist_handed_on"] <= 8, c
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"


def _random_bf16(seed, B, V):
    rng = np.random.default_rng(seed)
    x = np.empty((B, V), np.float32)
    for b in range(B):
        kind = b % 4
        if kind == 0:
            x[b] = rng.standard_normal(V) * rng.uniform(0.5, 6)
        elif kind == 1:  # a Zipf head over noise
            x[b] = rng.standard_normal(V) * 2
            x[b, rng.permutation(V)] += 1.1 * (np.log(V) - np.log(np.arange(1, V + 1)))
        elif kind == 2:  # few distinct values (heavy duplicates)
            x[b] = rng.integers(-8, 9, V) * 0.5
        else:  # a wide spread
            x[b] = rng.standard_normal(V) * 12
    p = W.default_params(B)
    p["temperature"] = rng.choice([0.3, 0.7, 1.0, 1.5], B)
    p["top_k"] = rng.choice([0, 0, V, V + 7], B)
    p["top_p"] = rng.choice([0.5, 0.8, 0.9, 0.95, 0.99], B)
    p["repetition_penalty"] = rng.choice([1.0, 1.05, 1.3], B)
    p["repetition_lookback"] = rng.choice([16, 64, 512], B)
    p["frequency_penalty"] = rng.choice([0.0, 0.2], B)
    p["presence_penalty"] = rng.choice([0.0, 0.3], B)
    p["softcap"] = rng.choice([0.0, 30.0, 10.0], B)
    H = 600
    hist = rng.integers(0, V, size=(B, H), dtype=np.int64).astype(np.int32)
    # windows that hold the row's maximum (its value leaves the histogram)
    hist[:, -3:] = np.argsort(-x, axis=1)[:, :3].astype(np.int32)
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
    return dict(name=f"bf16-random-{seed}", logits=W.f32_to_bf16_bits(x), bf16=True, params=p, hist=hist,
                hist_len=hl, masks=masks, seeds=seeds, u=W.uniforms_for(seeds))


@pytest.mark.parametrize("seed,V", [(1, 1000), (2, 4099), (3, 65536), (4, 151936), (5, 262144)])
def test_random_bf16_rows(ctx, oracle_mod, seed, V):
    cfg = _random_bf16(seed, 24, V)
    got, c = run(ctx, cfg)
    cl, _ = run(ctx, cfg, hist_path=0)
    assert c["last_hist_rows"] == 24, c
    bad = diff_rows(got, cl)
    assert not bad, f"histogram vs cluster path: {len(bad)} mismatches, first {bad[:6]}"
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"histogram path vs oracle: {len(bad)} mismatches, first {bad[:6]}"


def test_rows_handed_on(ctx, oracle_mod):
    """Rows the histogram path hands to the cluster kernel: one value 70000
    times (a 16-bit count overflows), magnitudes spread over 70 binades at a
    high temperature (more groups within reach of the maximum than the path
    walks), a top-p just below 1; and rows it keeps beside them."""
    V = 70000
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((6, V)) * 3).astype(np.float32)
    x[0] = 2.5
    x[1] = (np.sign(rng.standard_normal(V)) * np.exp2(rng.uniform(-60, 14, V))).astype(np.float32)
    p = W.default_params(6)
    p["temperature"] = [1.0, 1000.0, 1.0, 1.0, 0.5, 2.0]
    p["top_p"] = [0.9, 0.9, np.float32(0.99999994), 0.5, 0.9, 0.95]
    p["softcap"] = [0.0, 0.0, 0.0, 5.0, 6.0, 7.0]
    seeds = np.arange(6, dtype=np.uint32) + 77
    cfg = dict(name="handed-on", logits=W.f32_to_bf16_bits(x), bf16=True, params=p, hist=None, hist_len=None,
               masks=None, seeds=seeds, u=W.uniforms_for(seeds))
    got, c = run(ctx, cfg)
    print(f"\n{c['last_hist_handed_on']} of 6 rows handed on")
    assert c["last_hist_rows"] == 6 and c["last_hist_handed_on"] >= 2, c
    bad = diff_rows(got, oracle(oracle_mod, cfg))
    assert not bad, f"{len(bad)} mismatches, first {bad[:6]}"
