"""Greedy verification of prompt-lookup drafts: a numpy restatement of
SpeculativeDecoder::try_speculative_step's acceptance (speculative.h:190-225)
and argmax (speculative.h:248-258), and the seeded cases the tests use."""
import numpy as np


def ref_argmax(row):
    """best = 0; for i >= 1: if row[i] > row[best]: best = i (NaN never larger)."""
    if row[0] != row[0]:
        return 0
    finite = ~np.isnan(row)
    m = row[finite].max()
    return int(np.nonzero(finite & (row == m))[0][0])  # -0 == +0: the first of them


def verify_one(rows, draft, eos):
    K = len(draft)
    if K == 0:
        return 0, -1, 0
    if K == 1:
        b = ref_argmax(rows[0])
        return 1, b, int(b != eos)
    for i in range(K - 1):
        p = ref_argmax(rows[i])
        if p != draft[i + 1]:
            return i + 1, p, int(p != eos)
        if draft[i + 1] == eos:
            return i + 1, eos, 0
    b = ref_argmax(rows[K - 1])
    return K, b, int(b != eos)


def make_cases(seed, B, V, bf16=False):
    """B slots, K in 0..8 each; drafts follow the argmax for a random prefix
    so that acceptance lengths vary; ties, -0/+0, NaN and EOS sprinkled in."""
    rng = np.random.default_rng(seed)
    Ks = rng.integers(0, 9, B)
    Ks[0] = 1
    n = int(Ks.sum())
    x = (rng.standard_normal((max(n, 1), V)) * 3).astype(np.float32)
    if bf16:
        from qwenium_b200 import workloads as W
        x = W.bf16_bits_to_f32(W.f32_to_bf16_bits(x))
    eos = int(rng.integers(0, V))
    drafts = np.zeros(max(n, 1), np.int32)
    off = np.zeros(B + 1, np.int32)
    off[1:] = np.cumsum(Ks)
    for b in range(B):
        r0, K = off[b], Ks[b]
        if K == 0:
            continue
        good = int(rng.integers(0, K + 1))
        drafts[r0] = int(rng.integers(0, V))
        kind = rng.integers(0, 6)
        for i in range(K):
            row = x[r0 + i]
            if kind == 0 and V > 2:      # a tie for the maximum
                j = int(np.argmax(row)); k2 = int(rng.integers(0, V)); row[k2] = row[j]
            elif kind == 1 and V > 1:    # NaN inside the row
                row[int(rng.integers(1, V))] = np.nan
            elif kind == 2 and i == 0:   # NaN at index 0: argmax is 0
                row[0] = np.nan
            elif kind == 3:              # -0 / +0 maxima
                row[:] = -np.abs(row) - 1.0
                row[int(rng.integers(0, V))] = -0.0
                row[int(rng.integers(0, V))] = 0.0
        for i in range(K - 1):
            p = ref_argmax(x[r0 + i])
            drafts[r0 + i + 1] = p if i < good else (p + 1) % V
            if kind == 4 and i == good - 1:
                drafts[r0 + i + 1] = p
                eos = p if rng.random() < 0.5 else eos
    return x[:n] if n else x[:0], drafts[:n], off, eos
