"""Grammar char classes (TokenTrie::mark_char_class, token-trie.cpp:93-116):
the first-byte table and 256-bit class of qsamp_char_class_masks, against
the reference's own marks (the compiled trie) on the C3 vocabulary."""
import numpy as np
import pytest

from qwenium_b200 import qsamp
from qwenium_b200 import workloads as W


def marks_from_table(table, bits):
    """What qs_char_class_kernel computes: bit i = class[first byte of i]."""
    allowed = np.unpackbits(bits.view(np.uint8), bitorder="little").astype(bool)
    allowed = np.concatenate([allowed, [False]])  # index 256: empty token
    return allowed[table]


def test_first_byte_table():
    strs = [b"", b"a", b"\xff\x00", "{\"", b" x"]
    t = qsamp.first_byte_table(strs)
    assert t.tolist() == [256, ord("a"), 0xFF, ord("{"), ord(" ")]


def test_class_bits():
    b = qsamp.char_class_bits(['"', "\\"], negated=True)
    allowed = np.unpackbits(b.view(np.uint8), bitorder="little").astype(bool)
    assert not allowed[ord('"')] and not allowed[ord("\\")] and allowed.sum() == 254
    b = qsamp.char_class_bits([ord(c) for c in "0123456789"], negated=False)
    assert np.unpackbits(b.view(np.uint8), bitorder="little").sum() == 10


def test_marks_match_reference_trie(ref_mod):
    vocab = W.config3_vocab()
    vocab[5] = b""  # an empty token: never marked
    table = qsamp.first_byte_table(vocab)
    rv = ref_mod.RefVocab(vocab)
    lib = ref_mod.ref_lib("strict")
    rng = np.random.default_rng(3)
    V = len(vocab)
    classes = [('"\\', True), ("0123456789", False), (" \t\n", False), ("abc", True), ("", True), ("\x80\xff", False)]
    for _ in range(6):
        chars = bytes(rng.choice(256, size=int(rng.integers(1, 40)), replace=False).astype(np.uint8))
        classes.append((chars, bool(rng.integers(0, 2))))
    for chars, neg in classes:
        cb = chars.encode("latin-1") if isinstance(chars, str) else chars
        arr = np.frombuffer(cb, np.uint8).copy() if cb else np.zeros(1, np.uint8)
        out = np.zeros(V, np.uint8)
        lib.qwref_trie_mark_char_class(rv.trie, ref_mod._ptr(arr), len(cb), int(neg), V, ref_mod._ptr(out))
        mine = marks_from_table(table, qsamp.char_class_bits(list(cb), neg))
        assert np.array_equal(mine, out.astype(bool)), (chars, neg)
