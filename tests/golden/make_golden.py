"""Generates the golden fixtures in this directory from the reference itself.

Needs the reference harness oracle/_ref/libqwref_strict.so, compiled by
oracle/Makefile from the reference's unmodified src/sampling sources (so it
runs only where the reference tree is present). Inputs are not stored: every
case is regenerated from its seed by qwenium_b200.workloads, so a fixture
holds only what the reference returned.

  golden_tokens.npz  per case: the reference's token, whether it drew, and
                     the uniform its engine yielded (TemperatureSampler::sample,
                     src/sampling/sampling.cpp:137-194)
  config3.npz        the C3 grammar states: allow-masks [10][4748] taken from
                     the logits the reference leaves after sample() (finite =
                     allowed), the stuck-grammar forced ids, the accepting
                     flags, the random walks that reached the states, and the
                     reference's tokens through the full Sampler::sample path
                     with the grammar attached (sampling.cpp:25-81)

Usage:  python tests/golden/make_golden.py      (about six minutes: the
reference builds its token trie once per sampler)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402

from qwenium_b200 import qsamp  # noqa: E402
from qwenium_b200 import workloads as W  # noqa: E402


def ref_rows(cfg):
    """The reference's TemperatureSampler on every row of a config."""
    x, p = cfg["logits"], cfg["params"]
    B = x.shape[0]
    tok = np.zeros(B, np.int32)
    drew = np.zeros(B, np.int32)
    u = np.zeros(B, np.float64)
    for b in range(B):
        assert p["frequency_penalty"][b] == 0 and p["presence_penalty"][b] == 0 and p["softcap"][b] == 0
        h = cfg["hist"][b, : cfg["hist_len"][b]] if cfg.get("hist") is not None else np.zeros(0, np.int32)
        t, uu, d, _ = O.ref_temperature_sample(x[b], h, float(p["temperature"][b]), float(p["repetition_penalty"][b]),
                                               int(p["repetition_lookback"][b]), int(p["top_k"][b]),
                                               float(p["top_p"][b]), int(cfg["seeds"][b]))
        tok[b], drew[b], u[b] = t, d, uu
    return tok, drew, u


def no_ext(cfg):
    cfg["params"]["frequency_penalty"] = 0.0
    cfg["params"]["presence_penalty"] = 0.0
    return cfg


def token_cases():
    cases = {
        "config1_s1": W.config1(1),
        "config1_s3": W.config1(3),
        "config1_greedy": W.config1(1, greedy=True),
        "config2_b10": no_ext(W.config2(2, B=10)),
        "config2_s7_b16": no_ext(W.config2(7, B=16)),
        "config5_b16": W.config5(5, B=16),
    }
    out = {}
    for name, cfg in cases.items():
        t, d, u = ref_rows(cfg)
        assert np.array_equal(u, cfg["u"]), name
        out[name + "_token"], out[name + "_drew"], out[name + "_u"] = t, d, u
        print(f"{name}: tokens {t[:8]}")
    return out


# The mix of states C3 covers: (kind, how many). "string": inside a JSON
# string (most of the vocabulary is valid); "struct": between tokens of the
# structure (a few ids); "accept": the object is closed (the EOS rules of
# sampling.cpp:66-75 apply); "stuck": no valid id (EOS forced, sampling.cpp:40-60).
STATE_MIX = (("start", 1), ("struct", 3), ("string", 3), ("accept", 2), ("stuck", 1))


def _kind(n_valid, acc, walk_len):
    if n_valid == 0:
        return "stuck"
    if acc:
        return "accept"
    if walk_len == 0:
        return "start"
    return "string" if n_valid > 100000 else "struct"


def grammar_states(seed=33, max_walks=400):
    """Random walks from the start state. A step takes a single-byte token
    with probability 0.85 (those never cut a literal), otherwise any valid
    id; multi-byte ids the reference lists as valid can still lead to a dead
    state, which is how the stuck state arises."""
    vocab = W.config3_vocab()
    V = len(vocab)
    rv = O.RefVocab(vocab)
    g = O.RefGrammar(W.JSON_GBNF, rv)
    rng = np.random.default_rng(seed)
    eos_string = qsamp.find_eos_string(vocab)
    assert eos_string == W.EOT_ID
    want = dict(STATE_MIX)
    found = {k: [] for k in want}
    for _ in range(max_walks):
        if all(len(found[k]) >= n for k, n in want.items()):
            break
        g.reset()
        walk = []
        for _ in range(int(rng.integers(0, 40))):
            valid = g.valid_tokens()
            if valid.size == 0:
                break
            singles = valid[valid < 256]
            pool = singles if (singles.size and rng.random() < 0.85) else valid
            tok = int(rng.choice(pool))
            g.accept(tok)
            walk.append(tok)
        valid = g.valid_tokens()
        acc = g.accepting()
        kind = _kind(valid.size, acc, len(walk))
        if len(found[kind]) < want[kind]:
            m, f = qsamp.grammar_mask(valid, acc, eos_string, W.IM_END_ID, V)
            found[kind].append((walk, acc, valid.size, m, f))
            print(f"{kind}: walk {len(walk)} tokens, {valid.size} valid, accepting={acc}, force={f}")
    missing = {k: n - len(found[k]) for k, n in want.items() if len(found[k]) < n}
    assert not missing, f"walks did not reach {missing}"
    states = [st for k, _ in STATE_MIX for st in found[k]]
    walks = [st[0] for st in states]
    return (vocab, rv, g, walks, np.array([st[1] for st in states]), np.array([st[2] for st in states]),
            np.stack([st[3] for st in states]), np.array([st[4] for st in states], np.int32))


def grammar_reference_tokens(vocab, rv, g, walks, masks, force):
    """The reference's Sampler::sample with the grammar attached, per state
    (TemperatureSampler with C3's per-row parameters, extensions off). The
    mask each row was sampled under is read back from the logits it leaves."""
    cfg = W.config3(masks, force, extensions=False)
    x, p = cfg["logits"], cfg["params"]
    B, V = x.shape
    lib = O.ref_lib("strict")
    tok = np.zeros(B, np.int32)
    seen = np.zeros_like(masks)
    for b in range(B):
        g.reset()
        for t in walks[b]:
            g.accept(t)
        h = np.ascontiguousarray(cfg["hist"][b, : cfg["hist_len"][b]], np.int32)
        lo = np.empty(V, np.float32)
        u = O.ctypes.c_double()
        xb = np.ascontiguousarray(x[b], np.float32)
        tok[b] = lib.qwref_sampler_sample_full(
            1, float(p["temperature"][b]), float(p["repetition_penalty"][b]), int(p["repetition_lookback"][b]),
            int(p["top_k"][b]), float(p["top_p"][b]), g.handle, rv.handle, W.IM_END_ID, None, -1,
            O._ptr(xb), V, O._ptr(h), h.size, int(cfg["seeds"][b]), O.ctypes.byref(u), O._ptr(lo))
        # the sampler built its own trie and attached it to the grammar; it is
        # gone with the sampler, so the grammar gets the persistent one back
        lib.qwref_grammar_set_trie(g.handle, rv.trie)
        assert u.value == cfg["u"][b]
        allowed = np.isfinite(lo)
        pad = np.zeros(masks.shape[1] * 32, np.uint8)
        pad[:V] = allowed
        seen[b] = np.packbits(pad, bitorder="little").view(np.uint32)
        print(f"row {b}: reference token {tok[b]}, {int(allowed.sum())} allowed")
    return tok, seen


def main():
    O.build()
    if not O.ref_available("strict"):
        sys.exit("oracle/_ref/libqwref_strict.so is missing: build it with make -C oracle ref")
    np.savez_compressed(os.path.join(HERE, "golden_tokens.npz"), **token_cases())
    vocab, rv, g, walks, acc, n_valid, masks, force = grammar_states()
    tok, seen = grammar_reference_tokens(vocab, rv, g, walks, masks, force)
    # the masks are the reference's own: stuck rows keep only the EOS string
    for b in range(len(masks)):
        if force[b] >= 0:
            exp = np.zeros_like(masks[b])
            exp[force[b] // 32] = np.uint32(1) << np.uint32(force[b] % 32)
            assert np.array_equal(seen[b], exp), b
        else:
            assert np.array_equal(seen[b], masks[b]), b
    wl = np.array([len(w) for w in walks], np.int32)
    wf = np.full((len(walks), max(1, wl.max())), -1, np.int32)
    for i, w in enumerate(walks):
        wf[i, : len(w)] = w
    np.savez_compressed(os.path.join(HERE, "config3.npz"), masks=masks, force=force, accepting=acc,
                        n_valid=n_valid, walk_len=wl, walks=wf, token=tok)
    print("wrote golden_tokens.npz and config3.npz")


if __name__ == "__main__":
    main()
