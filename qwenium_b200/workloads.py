"""Seeded synthetic inputs for the five token-selection configurations.

The reference (rye-001/Qwenium) publishes no benchmark data for this path; the
configurations are the synthetic ones defined for this build. Every array is a
pure function of its seed (numpy PCG64), so tests on the GPU box regenerate
exactly the inputs the golden fixtures were made from.

The per-row uniform ``u`` is what the reference's own engine would draw:
``std::generate_canonical<double,53>(std::mt19937(seed))`` as libstdc++ 13
computes it (two 32-bit outputs, ``(double)g1 + (double)g2 * 2**32`` rounded
once, then divided by 2**64). ``TemperatureSampler`` consumes exactly that
value in ``std::discrete_distribution`` (src/sampling/sampling.cpp:192-193).
"""
from __future__ import annotations

import numpy as np

from .qsamp import ROW_PARAMS

V_QWEN = 151936
V_GEMMA = 262144


def mt19937_first_uniform(seed: int) -> float:
    """generate_canonical<double,53> of a fresh std::mt19937(seed)."""
    bg = np.random.MT19937(0)
    bg._legacy_seeding(int(seed) & 0xFFFFFFFF)
    g = bg.random_raw(2)
    s = float(int(g[0])) + float(int(g[1])) * 4294967296.0
    u = s / 18446744073709551616.0
    if u >= 1.0:
        u = np.nextafter(1.0, 0.0)
    return u


def uniforms_for(seeds) -> np.ndarray:
    return np.array([mt19937_first_uniform(int(s)) for s in seeds], np.float64)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (finite inputs)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = (b + np.uint32(0x7FFF) + ((b >> 16) & np.uint32(1))) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def default_params(B: int) -> np.ndarray:
    p = np.zeros(B, ROW_PARAMS)
    p["temperature"] = 1.0
    p["repetition_penalty"] = 1.0
    p["repetition_lookback"] = 64
    p["force_token"] = -1
    return p


def _hist(rng, B, H, V):
    hist = rng.integers(0, V, size=(B, H), dtype=np.int64).astype(np.int32)
    return hist, np.full(B, H, np.int32)


def config1(seed: int = 1, greedy: bool = False, V: int = V_QWEN) -> dict:
    """B=1: N(0,3^2) logits plus 20 ids boosted by +8; 64-id history;
    repetition penalty 1.1 over 64; T 0.8, top-k 40, top-p 0.95 (or T=0)."""
    rng = np.random.default_rng(seed)
    B = 1
    x = rng.standard_normal((B, V)) * 3.0
    for b in range(B):
        x[b, rng.choice(V, 20, replace=False)] += 8.0
    hist, hl = _hist(rng, B, 64, V)
    p = default_params(B)
    p["temperature"] = 0.0 if greedy else 0.8
    p["top_k"] = 40
    p["top_p"] = 0.95
    p["repetition_penalty"] = 1.1
    p["repetition_lookback"] = 64
    seeds = np.arange(B, dtype=np.uint32) + np.uint32(seed * 7919)
    return dict(name="config1" + ("-greedy" if greedy else ""), logits=x.astype(np.float32),
                bf16=False, params=p, hist=hist, hist_len=hl, masks=None, seeds=seeds,
                u=uniforms_for(seeds))


def config2(seed: int = 2, B: int = 10, V: int = V_QWEN) -> dict:
    """Batched server decode: N(0,2^2) logits plus a Zipf(s=1.1) log-probability
    head over a seed-permuted vocab order (+1.1*ln(V/(r+1)) for rank r);
    per-row T~U[0.2,1.2], top-k in {0,20,40,100}, top-p~U[0.8,1.0],
    frequency/presence ~U[0,0.5] over a 256-id history."""
    rng = np.random.default_rng(seed)
    x = np.empty((B, V), np.float32)
    head = 1.1 * (np.log(V) - np.log(np.arange(1, V + 1, dtype=np.float64)))
    for b in range(B):
        perm = rng.permutation(V)
        row = rng.standard_normal(V) * 2.0
        row[perm] += head
        x[b] = row.astype(np.float32)
    hist, hl = _hist(rng, B, 256, V)
    p = default_params(B)
    p["temperature"] = rng.uniform(0.2, 1.2, B).astype(np.float32)
    p["top_k"] = rng.choice(np.array([0, 20, 40, 100], np.int32), B)
    p["top_p"] = rng.uniform(0.8, 1.0, B).astype(np.float32)
    p["frequency_penalty"] = rng.uniform(0.0, 0.5, B).astype(np.float32)
    p["presence_penalty"] = rng.uniform(0.0, 0.5, B).astype(np.float32)
    p["repetition_lookback"] = 256
    seeds = np.arange(B, dtype=np.uint32) + np.uint32(seed * 7919)
    return dict(name=f"config2-B{B}", logits=x, bf16=False, params=p, hist=hist, hist_len=hl,
                masks=None, seeds=seeds, u=uniforms_for(seeds))


# ---- C3: a grammar-constrained batch -----------------------------------
# Ids of the two end-of-text strings in the synthetic vocabulary (the
# positions they hold in Qwen2's vocabulary).
EOT_ID = 151643   # "<|endoftext|>"
IM_END_ID = 151645  # "<|im_end|>"

# A JSON-object grammar written for this build in the reference's GBNF
# dialect (src/sampling/grammar_vocab.cpp parse_impl). The dialect has no
# bounded repetition, so nesting depth <= 3 comes from per-depth rules.
JSON_GBNF = r"""
root   ::= obj1 ws
obj1   ::= "{" ws ( pair1 ( ws "," ws pair1 )* )? ws "}"
pair1  ::= string ws ":" ws val1
val1   ::= obj2 | arr2 | scalar
obj2   ::= "{" ws ( pair2 ( ws "," ws pair2 )* )? ws "}"
arr2   ::= "[" ws ( val2 ( ws "," ws val2 )* )? ws "]"
pair2  ::= string ws ":" ws val2
val2   ::= obj3 | arr3 | scalar
obj3   ::= "{" ws ( pair3 ( ws "," ws pair3 )* )? ws "}"
arr3   ::= "[" ws ( scalar ( ws "," ws scalar )* )? ws "]"
pair3  ::= string ws ":" ws scalar
scalar ::= string | number | "true" | "false" | "null"
string ::= "\"" [^"\\]* "\""
number ::= "-"? [0-9]+ ( "." [0-9]+ )?
ws     ::= [ \t\n]*
"""


def config3_vocab(seed: int = 3, V: int = V_QWEN) -> list:
    """256 single bytes, then V-256 random printable strings of 2-16 bytes,
    with the two end-of-text strings at EOT_ID / IM_END_ID."""
    rng = np.random.default_rng(seed)
    strs = [bytes([i]) for i in range(256)]
    n = V - 256
    lens = rng.integers(2, 17, n)
    chars = rng.integers(0x20, 0x7F, int(lens.sum())).astype(np.uint8).tobytes()
    offs = np.concatenate([[0], np.cumsum(lens)])
    strs += [chars[offs[i]:offs[i + 1]] for i in range(n)]
    if V > IM_END_ID:
        strs[EOT_ID] = b"<|endoftext|>"
        strs[IM_END_ID] = b"<|im_end|>"
    return strs


def config3(masks: np.ndarray, force: np.ndarray, seed: int = 3, extensions: bool = True) -> dict:
    """C2's logits and parameters for len(masks) rows, each row constrained by
    one grammar state: masks [B][ceil(V/32)] allow-bits (the reference's
    valid ids plus its EOS rules, sampling.cpp:62-75) and force [B] (the EOS
    string id for a stuck grammar, sampling.cpp:40-60, else -1). Without
    extensions the frequency / presence penalties are off (the reference has
    neither)."""
    B = int(masks.shape[0])
    cfg = config2(seed, B=B)
    cfg["name"] = f"config3-B{B}"
    cfg["masks"] = np.ascontiguousarray(masks, np.uint32)
    cfg["params"]["force_token"] = np.asarray(force, np.int32)
    if not extensions:
        cfg["params"]["frequency_penalty"] = 0.0
        cfg["params"]["presence_penalty"] = 0.0
    return cfg


def config4(seed: int = 4, B: int = 256, V: int = V_GEMMA) -> dict:
    """Large vocab: bf16 logits ~N(0,4^2), soft-cap 30, T 1.0, top-p 0.9,
    top-k 0, repetition penalty 1.05 over 512-id histories."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(4.0))
    bits = f32_to_bf16_bits(x)
    hist, hl = _hist(rng, B, 512, V)
    p = default_params(B)
    p["temperature"] = 1.0
    p["top_k"] = 0
    p["top_p"] = 0.9
    p["softcap"] = 30.0
    p["repetition_penalty"] = 1.05
    p["repetition_lookback"] = 512
    seeds = np.arange(B, dtype=np.uint32) + np.uint32(seed * 7919)
    return dict(name=f"config4-B{B}", logits=bits, bf16=True, params=p, hist=hist, hist_len=hl,
                masks=None, seeds=seeds, u=uniforms_for(seeds))


def config5(seed: int = 5, B: int = 512, V: int = V_GEMMA) -> dict:
    """Vocab-sharded: fp32 N(0,3^2) plus 50 spikes of +6 per row; T 1.0,
    top-k 64, top-p 0.95; no penalties."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, V), dtype=np.float32) * np.float32(3.0)
    for b in range(B):
        x[b, rng.choice(V, 50, replace=False)] += np.float32(6.0)
    p = default_params(B)
    p["temperature"] = 1.0
    p["top_k"] = 64
    p["top_p"] = 0.95
    seeds = np.arange(B, dtype=np.uint32) + np.uint32(seed * 7919)
    return dict(name=f"config5-B{B}", logits=x, bf16=False, params=p, hist=None, hist_len=None,
                masks=None, seeds=seeds, u=uniforms_for(seeds))
