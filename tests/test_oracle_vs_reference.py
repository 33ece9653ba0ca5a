"""Pin the C restatement (oracle/qsamp_oracle.c) to the reference itself.

The reference's src/sampling sources are compiled unmodified at -O2
(oracle/_ref/libqwref_strict.so: IEEE float in source order). For every case
the oracle must reproduce, bit for bit, the logits the reference leaves behind
after sample() (pruning, grammar mask, repetition penalty, temperature) and
the token it returns -- up to the order of equal logits, which std::sort
leaves unspecified (the oracle orders ties by ascending id).
"""
import numpy as np
import pytest

from qwenium_b200 import workloads as W


def _params(B, **kw):
    p = W.default_params(B)
    for k, v in kw.items():
        p[k] = v
    return p


def _same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _check_row(O, logits, hist, T, rep, lb, k, p, seed, greedy_cls=False):
    V = logits.size
    params = _params(1, temperature=T, top_k=k, top_p=p, repetition_penalty=rep, repetition_lookback=lb)
    u = np.array([W.mt19937_first_uniform(seed)])
    hl = np.array([hist.size], np.int32)
    hh = hist.reshape(1, -1) if hist.size else np.zeros((1, 1), np.int32)
    out, _, _, lo = O.oracle_sample(logits.reshape(1, V), params, hh, hl, None, u, want_logits=True, n_threads=1)
    if greedy_cls:
        tok, rl = O.ref_greedy_sample(logits, hist, rep, lb, want_logits=True)
    else:
        tok, ru, drew, rl = O.ref_temperature_sample(logits, hist, T, rep, lb, k, p, seed, want_logits=True)
        assert ru == u[0]
        assert drew == out[0]["drew"], (drew, out[0])
    assert _same_bits(rl, lo[0]), "transformed logits differ"
    o = int(out[0]["token"])
    if tok != o:
        # only legal when both ids sit in the same tie group
        assert lo[0][tok] == lo[0][o], (tok, o, lo[0][tok], lo[0][o])
    return out[0]


CASES = []
_rng = np.random.default_rng(12345)
for V in (1, 2, 3, 31, 32, 33, 257, 4097):
    for _ in range(6):
        CASES.append((V, float(_rng.choice([0.0, 0.3, 0.8, 1.0, 1.7])), int(_rng.choice([0, 1, 5, 40, V - 1, V, V + 3])),
                      float(_rng.choice([0.0, 0.5, 0.9, 0.95, 0.999, 1.0])), float(_rng.choice([1.0, 1.1, 1.3])),
                      int(_rng.choice([0, 32, 64, -1])), int(_rng.integers(0, 2**32))))


@pytest.mark.parametrize("V,T,k,p,rep,lb,seed", CASES)
def test_small_vocab_cases(ref_mod, V, T, k, p, rep, lb, seed):
    rng = np.random.default_rng(seed % 100000)
    x = (rng.standard_normal(V) * 3).astype(np.float32)
    hist = rng.integers(-2, V + 2, size=int(rng.integers(0, 80)), dtype=np.int64).astype(np.int32)
    _check_row(ref_mod, x, hist, T, rep, lb, k, p, seed)


@pytest.mark.parametrize("kind", ["normal", "ties", "masked", "spiky"])
def test_full_vocab_rows(ref_mod, kind):
    V = W.V_QWEN
    rng = np.random.default_rng({"normal": 1, "ties": 2, "masked": 3, "spiky": 4}[kind])
    for r in range(6):
        x = rng.standard_normal(V).astype(np.float32) * np.float32(rng.uniform(1, 5))
        if kind == "ties":  # bf16-rounded: large tie groups
            x = W.bf16_bits_to_f32(W.f32_to_bf16_bits(x))
        if kind == "masked":
            x[rng.random(V) < 0.7] = -np.inf
        if kind == "spiky":
            x[rng.choice(V, 20, replace=False)] += 8
        hist = rng.integers(0, V, 64, dtype=np.int64).astype(np.int32)
        T = float(rng.choice([0.5, 0.8, 1.0, 1.2]))
        k = int(rng.choice([0, 40, 100]))
        p = float(rng.choice([0.8, 0.9, 0.95, 1.0]))
        _check_row(ref_mod, x, hist, T, 1.1, 64, k, p, int(rng.integers(0, 2**32)))


def test_greedy_sampler_class(ref_mod):
    rng = np.random.default_rng(7)
    for V in (1, 5, 1000, W.V_QWEN):
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        hist = rng.integers(0, V, 32, dtype=np.int64).astype(np.int32)
        _check_row(ref_mod, x, hist, 0.0, 1.2, 32, 0, 0.0, 0, greedy_cls=True)


def test_all_masked_row_greedy(ref_mod):
    x = np.full(100, -np.inf, np.float32)
    _check_row(ref_mod, x, np.zeros(0, np.int32), 0.0, 1.2, 32, 0, 0.0, 0, greedy_cls=True)


def test_config1_and_greedy(ref_mod):
    for cfg in (W.config1(1), W.config1(1, greedy=True), W.config1(11)):
        p = cfg["params"][0]
        _check_row(ref_mod, cfg["logits"][0], cfg["hist"][0], float(p["temperature"]), float(p["repetition_penalty"]),
                   int(p["repetition_lookback"]), int(p["top_k"]), float(p["top_p"]), int(cfg["seeds"][0]))


def test_config4_rows_without_extensions(ref_mod):
    """bf16 logits, k=0, p=0.9: the reference gets the soft-capped values
    (soft-cap is a model-graph op in the reference), the oracle applies it."""
    O = ref_mod
    cfg = W.config4(4, B=3)
    x = W.bf16_bits_to_f32(cfg["logits"])
    lib = O.oracle_lib()
    for b in range(3):
        sc = np.array([lib.qso_softcap(float(v), 30.0) for v in x[b]], np.float32)
        params = cfg["params"][b : b + 1].copy()
        out, _, _, lo = O.oracle_sample(cfg["logits"][b : b + 1], params, cfg["hist"][b : b + 1],
                                        cfg["hist_len"][b : b + 1], None, cfg["u"][b : b + 1], want_logits=True,
                                        n_threads=1, bf16=True)
        tok, ru, drew, rl = O.ref_temperature_sample(sc, cfg["hist"][b], 1.0, 1.05, 512, 0, 0.9, int(cfg["seeds"][b]),
                                                     want_logits=True)
        assert ru == cfg["u"][b]
        assert _same_bits(rl, lo[0])
        o = int(out[0]["token"])
        assert tok == o or lo[0][tok] == lo[0][o]


def test_uniform_stream_matches_engine(ref_mod):
    for s in [0, 1, 2, 5489, 7919, 123456789, 2**31, 2**32 - 1]:
        assert W.mt19937_first_uniform(s) == ref_mod.ref_first_uniform(s)


def test_oracle_expf_is_glibc(oracle_mod):
    lib = oracle_mod.oracle_lib()
    xs = np.linspace(-104, 0, 10001, dtype=np.float32)
    got = np.array([lib.qso_expf(float(v)) for v in xs], np.float32)
    assert np.all(np.abs(got.astype(np.float64) - np.exp(xs.astype(np.float64))) <= 1e-6 * np.exp(xs) + 1e-45)
