"""The compact token trie (qsamp_trie_*, qwenium_b200/trie) against the
reference's TokenTrie (src/sampling/token-trie.cpp, compiled unmodified in
oracle/_ref): every query returns the same ids in the same order.

The reference's own trie tests compare the trie with brute force
(tests/unit/test_token_trie.cpp:306-325, first-char buckets) and the grammar's
valid sets with and without a trie (:443-464); here the compact trie is
compared with the reference trie itself, query by query, on a byte-level
vocabulary with duplicates, prefixes of other tokens, empty tokens and bytes
above 127, then timed on the full config-3 vocabulary."""
import time

import numpy as np
import pytest

import oracle as O
from qwenium_b200 import qsamp
from qwenium_b200 import workloads as W


def _vocab(n_random=20000, seed=7):
    rng = np.random.default_rng(seed)
    v = [bytes([i]) for i in range(256)]
    alpha = np.frombuffer(b'{}[]":, \t\n0123456789abcdefghijklmnopqrstuvwxyz\\-.tfn', np.uint8)
    for _ in range(n_random):
        n = int(rng.integers(1, 9))
        if rng.random() < 0.7:
            s = bytes(rng.choice(alpha, n))
        else:
            s = bytes(rng.integers(0, 256, n, dtype=np.uint8))
        v.append(s)
    # duplicates, empty tokens, tokens that prefix others, the EOS strings
    v += [b"true", b"true", b"", b"tr", b"t", b"", b'{"', b'{"a', b'{"ab', b"<|endoftext|>", b"<|im_end|>"]
    return v


@pytest.fixture(scope="module")
def tries(ref_mod):
    vocab = _vocab()
    ref = O.RefVocab(vocab)
    ours = qsamp.TokenTrie(vocab)
    return vocab, ref, ours


def _ref_ids(fn, *args):
    n = fn(*args, None, 0)
    out = np.empty(max(n, 1), np.int32)
    fn(*args, O._ptr(out), n)
    return out[:n]


def test_counts(tries):
    vocab, ref, ours = tries
    assert ours.token_count() == ref.lib.qwref_trie_token_count(ref.trie) == sum(1 for s in vocab if s)


def test_collect_by_first_char(tries):
    _, ref, ours = tries
    for c in range(256):
        want = _ref_ids(ref.lib.qwref_trie_collect_by_first_char, ref.trie, c)
        assert np.array_equal(ours.collect_by_first_char(c), want), c


def test_collect_by_prefix(tries):
    vocab, ref, ours = tries
    rng = np.random.default_rng(3)
    queries = [(b"", 0), (b"t", 0), (b"true", 0), (b"xtrue", 1), (b"true", 9), (b'{"ab', 0), (b'{"abc', 0),
               (b"\xff\x00", 0), (b"<|endoftext|>", 0)]
    for _ in range(3000):
        s = vocab[int(rng.integers(0, len(vocab)))]
        if not s:
            continue
        q = s + bytes(rng.integers(0, 256, int(rng.integers(0, 3)), dtype=np.uint8))
        queries.append((q, int(rng.integers(0, len(q) + 1))))
    for q, off in queries:
        want = _ref_ids(ref.lib.qwref_trie_collect_by_prefix, ref.trie, q, len(q), off)
        got = ours.collect_by_prefix(q, off)
        assert np.array_equal(got, want), (q, off, got[:8], want[:8])


def test_char_classes(tries):
    vocab, ref, ours = tries
    rng = np.random.default_rng(4)
    classes = [(b'"\\', True), (b"0123456789", False), (b" \t\n", False), (b"", True), (b"", False),
               (bytes(range(256)), False), (bytes(range(128, 256)), True)]
    for _ in range(60):
        classes.append((bytes(rng.integers(0, 256, int(rng.integers(1, 40)), dtype=np.uint8)), bool(rng.random() < .5)))
    for chars, neg in classes:
        c = np.frombuffer(chars, np.uint8).copy() if chars else np.zeros(1, np.uint8)
        want = _ref_ids(ref.lib.qwref_trie_collect_by_char_class, ref.trie, O._ptr(c), len(chars), int(neg))
        assert np.array_equal(ours.collect_by_char_class(list(chars), neg), want), (chars[:8], neg)
        mk = np.zeros(len(vocab), np.uint8)
        ref.lib.qwref_trie_mark_char_class(ref.trie, O._ptr(c), len(chars), int(neg), len(vocab), O._ptr(mk))
        assert np.array_equal(ours.mark_char_class(list(chars), neg), mk.astype(bool)), (chars[:8], neg)


def test_full_config3_vocabulary_is_small_and_fast():
    """The config-3 vocabulary (151,936 byte-level tokens): the reference's
    256-pointer nodes take about 29 s and 2.1 GB to build on it; the compact
    trie is a few MB."""
    vocab = W.config3_vocab()
    t0 = time.perf_counter()
    t = qsamp.TokenTrie(vocab)
    el = time.perf_counter() - t0
    total = sum(len(s) for s in vocab)
    assert t.token_count() == sum(1 for s in vocab if s)
    assert t.memory_bytes() < total + 9 * len(vocab) + 4096
    assert el < 10.0
    # a query the JSON grammar makes at a string value: every token whose
    # first byte is not '"' or '\'
    m = t.mark_char_class(['"', "\\"], True)
    first = np.array([s[0] if s else 256 for s in vocab])
    assert np.array_equal(m, (first != ord('"')) & (first != ord("\\")) & (first != 256))


def test_grammar_valid_sets_with_compact_trie(tmp_path):
    """The reference's GrammarVocab with the drop-in token-trie.h attached
    (oracle/_ref/trie_grammar_check, built through symbolic links so that the
    grammar's own #include resolves to the drop-in): on random walks of the
    config-3 JSON grammar over the config-3 vocabulary, every state's valid set
    equals the brute-force scan's (grammar_vocab.cpp:713-747)."""
    import os
    import struct
    import subprocess

    exe = os.path.join(os.path.dirname(O.HERE), "oracle", "_ref", "trie_grammar_check")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/trie_grammar_check not built (needs the reference sources)")
    vocab = W.config3_vocab()
    vf, gf = tmp_path / "vocab.bin", tmp_path / "json.gbnf"
    with open(vf, "wb") as f:
        f.write(struct.pack("<I", len(vocab)))
        for s in vocab:
            f.write(struct.pack("<I", len(s)))
            f.write(s)
    gf.write_text(W.JSON_GBNF)
    states = 0
    for seed in range(12):
        r = subprocess.run([exe, str(gf), str(vf), "60", str(seed)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
        states += int(r.stdout.split()[0])
    assert states >= 60
