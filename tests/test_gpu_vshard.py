"""GPU parity of the vocab-sharded path (qsamp_shard_topk + qsamp_merge_topk).

N ranks are emulated on one GPU: each vocabulary slice goes through
shard_topk, the [B][k] blocks are stacked rank-major (the all-gather's
layout) and merged. The merged rows must equal the unsharded path's rows and
the oracle's, field for field, for every N: with top_k > 0 the merge is
exact (src/sampling/sampling.cpp:158-190 only ever see the top-k set).
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu

FIELDS = ("token", "position", "n_keep", "drew", "sum_exp", "sum_keep", "max_logit", "prob")
RES = np.dtype([(f, "<i4" if f in FIELDS[:4] else "<f4") for f in FIELDS])


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwenium_b200 import qsamp

    return qsamp.Context(0)


def slice_mask(mask, lo, n):
    """Bits [lo, lo + n) of packed allow-masks [B][words] as local masks."""
    B = mask.shape[0]
    bits = np.unpackbits(mask.view(np.uint8).reshape(B, -1), axis=1, bitorder="little")[:, lo:lo + n]
    words = (n + 31) // 32
    pad = np.zeros((B, words * 32), np.uint8)
    pad[:, :n] = bits
    return np.packbits(pad, axis=1, bitorder="little").view(np.uint32).reshape(B, words)


def case(seed, B, V, bf16=False, masks=False):
    cfg = W.config5(seed, B=B, V=V)
    rng = np.random.default_rng(seed + 1000)
    p = cfg["params"]
    p["temperature"] = rng.uniform(0.3, 1.3, B).astype(np.float32)
    p["temperature"][::7] = 0.0                      # greedy rows
    p["top_k"] = rng.choice(np.array([1, 8, 40, 64], np.int32), B)
    p["top_p"] = rng.uniform(0.5, 1.0, B).astype(np.float32)
    p["repetition_penalty"] = 1.1
    p["repetition_lookback"] = 64
    p["frequency_penalty"] = rng.uniform(0, 0.5, B).astype(np.float32)
    p["presence_penalty"] = rng.uniform(0, 0.5, B).astype(np.float32)
    if B > 3:
        p["force_token"][3] = V - 5                   # held by the last shard only
    hist = rng.integers(0, V, (B, 96), dtype=np.int64).astype(np.int32)
    hist[:, :8] = np.argsort(-cfg["logits"], axis=1)[:, :8].astype(np.int32)  # penalise the leaders
    cfg["hist"], cfg["hist_len"] = hist, rng.integers(0, 97, B).astype(np.int32)
    if bf16:
        cfg["logits"] = W.bf16_bits_to_f32(W.f32_to_bf16_bits(cfg["logits"]))
        cfg["bf16"] = True
        p["softcap"] = np.where(np.arange(B) % 2 == 0, 30.0, 0.0).astype(np.float32)
    if masks:
        allow = rng.random((B, V)) < 0.9
        words = (V + 31) // 32
        pad = np.zeros((B, words * 32), np.uint8)
        pad[:, :V] = allow
        cfg["masks"] = np.packbits(pad, axis=1, bitorder="little").view(np.uint32).reshape(B, words)
    return cfg


def to_dev(x, bf16):
    import torch

    if bf16:
        return torch.from_numpy(np.ascontiguousarray(W.f32_to_bf16_bits(x)).view(np.int16)).cuda()
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_unsharded(ctx, cfg):
    import torch

    B = cfg["logits"].shape[0]
    masks = torch.from_numpy(cfg["masks"].view(np.int32)).cuda() if cfg.get("masks") is not None else None
    res = ctx.sample_batch(to_dev(cfg["logits"], cfg["bf16"]), cfg["params"], hist=torch.from_numpy(cfg["hist"]).cuda(),
                           hist_len=cfg["hist_len"], masks=masks, u=cfg["u"])
    torch.cuda.synchronize()
    return res.cpu().numpy().view(RES).reshape(B)


def run_sharded(ctx, cfg, n_ranks, k=64):
    import torch

    from qwenium_b200 import shard

    x = cfg["logits"]
    B, V = x.shape
    hist = torch.from_numpy(cfg["hist"]).cuda()
    vals, ids = [], []
    for r in range(n_ranks):
        lo, n = shard.shard_range(V, n_ranks, r)
        m = None
        if cfg.get("masks") is not None:
            m = torch.from_numpy(slice_mask(cfg["masks"], lo, n).view(np.int32)).cuda()
        v, i = ctx.shard_topk(to_dev(np.ascontiguousarray(x[:, lo:lo + n]), cfg["bf16"]), cfg["params"], lo, V, k,
                              hist=hist, hist_len=cfg["hist_len"], masks=m)
        vals.append(v)
        ids.append(i)
    res = ctx.merge_topk(torch.stack(vals), torch.stack(ids), cfg["params"], u=cfg["u"])
    torch.cuda.synchronize()
    return res.cpu().numpy().view(RES).reshape(B)


def assert_same(a, b, what):
    """Bit-identical rows (NaN probabilities of all-masked rows match NaN)."""
    for f in FIELDS:
        x, y = np.asarray(a[f]), np.asarray(b[f])
        if f in FIELDS[:4]:
            ok = x.astype(np.int64) == y.astype(np.int64)
        else:
            x, y = x.astype(np.float32), y.astype(np.float32)
            ok = (x.view(np.uint32) == y.view(np.uint32)) | (np.isnan(x) & np.isnan(y))
        assert np.all(ok), f"{what}: field {f} differs at rows {np.nonzero(~ok)[0][:10]}"


@pytest.mark.parametrize("n_ranks", [1, 2, 3, 8])
def test_vshard_matches_unsharded(ctx, n_ranks):
    cfg = case(51, 48, 65536)
    base = run_unsharded(ctx, cfg)
    got = run_sharded(ctx, cfg, n_ranks)
    assert_same(got, base, f"N={n_ranks}")


def test_vshard_bf16_softcap_masks(ctx):
    cfg = case(52, 40, 50000, bf16=True, masks=True)
    base = run_unsharded(ctx, cfg)
    for n in (2, 4):
        assert_same(run_sharded(ctx, cfg, n), base, f"bf16 N={n}")


def test_vshard_against_oracle(ctx, oracle_mod):
    cfg = case(53, 32, 30011)
    out, _, _, _ = oracle_mod.oracle_sample(cfg["logits"], cfg["params"], cfg["hist"], cfg["hist_len"], None,
                                            cfg["u"], bf16=False)
    assert_same(run_sharded(ctx, cfg, 4), out, "oracle N=4")


def test_vshard_config5_shape(ctx):
    """C5: B=512, V=262144, k=64, p=0.95 over 8 shards."""
    cfg = W.config5(5, B=64, V=W.V_GEMMA)
    cfg["hist"] = np.zeros((64, 1), np.int32)
    cfg["hist_len"] = np.zeros(64, np.int32)
    base = run_unsharded(ctx, cfg)
    assert_same(run_sharded(ctx, cfg, 8), base, "C5 N=8")


def test_vshard_rejects_full_vocab_rows(ctx):
    import torch

    from qwenium_b200 import qsamp

    cfg = case(54, 4, 4096)
    cfg["params"]["temperature"] = 1.0
    cfg["params"]["top_k"] = 0
    with pytest.raises(qsamp.QsampError) as e:
        ctx.shard_topk(torch.from_numpy(cfg["logits"][:, :2048].copy()).cuda(), cfg["params"], 0, 4096, 64)
    assert "UNSUPPORTED" in str(e.value) or e.value.status == 3
    with pytest.raises(qsamp.QsampError):
        v = torch.zeros((2, 4, 1024), device="cuda")
        i = torch.zeros((2, 4, 1024), dtype=torch.int32, device="cuda")
        p = W.default_params(4)
        p["top_k"] = 1
        ctx.merge_topk(torch.cat([v] * 3), torch.cat([i] * 3), p)  # 6 x 1024 > 5120 candidates


def test_cluster_rows_after_a_sharded_call(oracle_mod):
    """A context whose first call is qsamp_shard_topk must still serve
    full-vocabulary rows afterwards (the cluster kernel's launch attributes
    are set by its own first use, whoever computed the context's limits)."""
    import torch

    from qwenium_b200 import qsamp

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = qsamp.Context(0)
    cfg = case(71, 8, 50000)
    c.shard_topk(to_dev(np.ascontiguousarray(cfg["logits"][:, :25000]), False), cfg["params"], 0, 50000, 64,
                 hist=torch.from_numpy(cfg["hist"]).cuda(), hist_len=cfg["hist_len"])
    full = case(72, 8, 131072, bf16=True)
    full["params"]["top_k"] = 0
    full["params"]["temperature"] = 0.8
    full["params"]["force_token"] = -1
    got = run_unsharded(c, full)
    want, _, _, _ = oracle_mod.oracle_sample(W.f32_to_bf16_bits(full["logits"]), full["params"], full["hist"],
                                             full["hist_len"], None, full["u"], bf16=True)
    assert_same(got, want, "full-vocabulary rows after a sharded call")
    c.close()
