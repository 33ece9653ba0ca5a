"""qsamp_char_class_masks on the GPU: the allow-bits of B grammar char
classes at once, against the first-byte construction pinned to the
reference's TokenTrie::mark_char_class (tests/test_char_class.py) and, where
the compiled reference harness is present, against the reference directly."""
import numpy as np
import pytest

from qwenium_b200 import qsamp
from qwenium_b200 import workloads as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return qsamp.Context(0)


def packed(marks):
    V = marks.shape[-1]
    words = (V + 31) // 32
    pad = np.zeros(marks.shape[:-1] + (words * 32,), np.uint8)
    pad[..., :V] = marks
    return np.packbits(pad, axis=-1, bitorder="little").view(np.uint32)


def run(ctx, table, classes, V, init=None, or_into=False, table_offset=0):
    import torch

    B = classes.shape[0]
    words = (V + 31) // 32
    tt = np.zeros(V + table_offset, np.uint16)
    tt[table_offset:] = table
    dt = torch.from_numpy(tt.view(np.int16)).cuda()[table_offset:]
    dc = torch.from_numpy(classes.view(np.int32)).cuda()
    m0 = init if init is not None else np.zeros((B, words), np.uint32)
    dm = torch.from_numpy(m0.view(np.int32).copy()).cuda()
    ctx.char_class_masks(dt, dc, dm, or_into=or_into)
    torch.cuda.synchronize()
    return dm.cpu().numpy().view(np.uint32)


def classes_for(rng, B):
    out = np.zeros((B, 8), np.uint32)
    for b in range(B):
        chars = list(rng.choice(256, size=int(rng.integers(0, 60)), replace=False))
        out[b] = qsamp.char_class_bits(chars, bool(rng.integers(0, 2)))
    out[0] = qsamp.char_class_bits(['"', "\\"], True)  # the JSON string body
    return out


@pytest.mark.parametrize("V", [1, 31, 32, 33, 1000, W.V_QWEN])
def test_char_class_masks(ctx, V):
    rng = np.random.default_rng(V)
    vocab = W.config3_vocab(V=max(V, 256))[:V] if V >= 256 else [bytes([c]) for c in rng.integers(0, 256, V)]
    vocab = list(vocab)
    vocab[V // 2] = b""
    table = qsamp.first_byte_table(vocab)
    cls = classes_for(rng, 24)
    allowed = np.unpackbits(cls.view(np.uint8), axis=1, bitorder="little").astype(bool)
    allowed = np.concatenate([allowed, np.zeros((24, 1), bool)], axis=1)
    want = packed(allowed[:, table])
    assert np.array_equal(run(ctx, table, cls, V), want)
    # OR into existing bits, and a table that is not 16-byte aligned
    init = rng.integers(0, 2**32, size=want.shape, dtype=np.uint64).astype(np.uint32)
    assert np.array_equal(run(ctx, table, cls, V, init=init, or_into=True), init | want)
    assert np.array_equal(run(ctx, table, cls, V, table_offset=3), want)


def test_char_class_against_reference(ctx, ref_mod):
    vocab = W.config3_vocab()
    table = qsamp.first_byte_table(vocab)
    rv = ref_mod.RefVocab(vocab)
    lib = ref_mod.ref_lib("strict")
    V = len(vocab)
    specs = [(b'"\\', True), (b"0123456789", False), (b" \t\n", False), (b"}", True)]
    cls = np.stack([qsamp.char_class_bits(list(c), n) for c, n in specs])
    got = run(ctx, table, cls, V)
    for b, (c, n) in enumerate(specs):
        arr = np.frombuffer(c, np.uint8).copy()
        out = np.zeros(V, np.uint8)
        lib.qwref_trie_mark_char_class(rv.trie, ref_mod._ptr(arr), len(c), int(n), V, ref_mod._ptr(out))
        assert np.array_equal(got[b], packed(out.astype(np.uint8))), (c, n)
