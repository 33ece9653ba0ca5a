"""TEST INFRASTRUCTURE ONLY: ctypes access to the checker libraries.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
module. It loads

* ``oracle/_build/libqsamp_oracle.so`` -- the C restatement of the reference's
  token selection (qsamp_oracle.c), and
* ``oracle/_ref/libqwref_{strict,release}.so`` -- the reference's own
  ``src/sampling`` sources compiled unmodified (ref_harness.cpp shims).

Nothing here is used by the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libqsamp_oracle.so")
REF_SO = {
    "strict": os.path.join(HERE, "_ref", "libqwref_strict.so"),
    "release": os.path.join(HERE, "_ref", "libqwref_release.so"),
}

# Same layout as qsamp_row_params (include/qsamp.h) and qso_row_params.
ROW_PARAMS = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_k", "<i4"),
        ("top_p", "<f4"),
        ("repetition_penalty", "<f4"),
        ("repetition_lookback", "<i4"),
        ("frequency_penalty", "<f4"),
        ("presence_penalty", "<f4"),
        ("softcap", "<f4"),
        ("force_token", "<i4"),
        ("flags", "<i4"),
        ("seed", "<u8"),
    ],
    align=True,
)
assert ROW_PARAMS.itemsize == 48

RESULT = np.dtype(
    [
        ("token", "<i4"),
        ("position", "<i4"),
        ("n_keep", "<i4"),
        ("drew", "<i4"),
        ("sum_exp", "<f4"),
        ("sum_keep", "<f4"),
        ("max_logit", "<f4"),
        ("prob", "<f4"),
    ]
)
assert RESULT.itemsize == 32

_P = ctypes.c_void_p
_lib_cache: dict = {}


def build(quiet: bool = True) -> None:
    """Compile the checker libraries (oracle/Makefile)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_P)


def oracle_lib():
    if "oracle" not in _lib_cache:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.qso_sample_batch.restype = ctypes.c_int
        lib.qso_sample_batch.argtypes = [
            _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _P, _P, ctypes.c_int,
            _P, _P, ctypes.c_int64, _P, _P, _P, _P, ctypes.c_int, _P, ctypes.c_int,
        ]
        lib.qso_expf.restype = ctypes.c_float
        lib.qso_expf.argtypes = [ctypes.c_float]
        lib.qso_softcap.restype = ctypes.c_float
        lib.qso_softcap.argtypes = [ctypes.c_float, ctypes.c_float]
        _lib_cache["oracle"] = lib
    return _lib_cache["oracle"]


def ref_available(kind: str = "strict") -> bool:
    return os.path.exists(REF_SO[kind])


def ref_lib(kind: str = "strict"):
    key = "ref_" + kind
    if key not in _lib_cache:
        lib = ctypes.CDLL(REF_SO[kind])
        lib.qwref_temperature_sample.restype = ctypes.c_int
        lib.qwref_temperature_sample.argtypes = [
            _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
            ctypes.c_int, ctypes.c_float, ctypes.c_uint32, _P, _P, _P,
        ]
        lib.qwref_greedy_sample.restype = ctypes.c_int
        lib.qwref_greedy_sample.argtypes = [
            _P, ctypes.c_int, _P, ctypes.c_int, ctypes.c_float, ctypes.c_int, _P,
        ]
        lib.qwref_temperature_sample_batch.restype = ctypes.c_int
        lib.qwref_temperature_sample_batch.argtypes = [
            _P, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _P, _P, _P, _P, _P, _P, ctypes.c_int,
            _P, _P, _P, ctypes.c_int,
        ]
        lib.qwref_first_uniform.restype = ctypes.c_double
        lib.qwref_first_uniform.argtypes = [ctypes.c_uint32]
        lib.qwref_vocab_new.restype = _P
        lib.qwref_vocab_new.argtypes = [_P, _P, ctypes.c_int]
        lib.qwref_vocab_free.argtypes = [_P]
        lib.qwref_trie_new.restype = _P
        lib.qwref_trie_new.argtypes = [_P]
        lib.qwref_trie_free.argtypes = [_P]
        lib.qwref_grammar_parse.restype = _P
        lib.qwref_grammar_parse.argtypes = [ctypes.c_char_p]
        lib.qwref_grammar_free.argtypes = [_P]
        lib.qwref_grammar_set_trie.argtypes = [_P, _P]
        lib.qwref_grammar_valid.restype = ctypes.c_int
        lib.qwref_grammar_valid.argtypes = [_P, _P, _P, ctypes.c_int]
        lib.qwref_grammar_accept.argtypes = [_P, ctypes.c_int32, _P]
        lib.qwref_grammar_accepting.restype = ctypes.c_int
        lib.qwref_grammar_accepting.argtypes = [_P]
        lib.qwref_grammar_reset.argtypes = [_P]
        lib.qwref_spec_verify.restype = None
        lib.qwref_spec_verify.argtypes = [_P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P, _P, _P]
        lib.qwref_trie_mark_char_class.restype = None
        lib.qwref_trie_mark_char_class.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        lib.qwref_trie_collect_by_prefix.restype = ctypes.c_int
        lib.qwref_trie_collect_by_prefix.argtypes = [_P, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _P,
                                                     ctypes.c_int]
        lib.qwref_trie_collect_by_char_class.restype = ctypes.c_int
        lib.qwref_trie_collect_by_char_class.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int]
        lib.qwref_trie_collect_by_first_char.restype = ctypes.c_int
        lib.qwref_trie_collect_by_first_char.argtypes = [_P, ctypes.c_uint8, _P, ctypes.c_int]
        lib.qwref_trie_token_count.restype = ctypes.c_longlong
        lib.qwref_trie_token_count.argtypes = [_P]
        lib.qwref_sampler_sample_full.restype = ctypes.c_int
        lib.qwref_sampler_sample_full.argtypes = [
            ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            _P, _P, ctypes.c_int32, _P, ctypes.c_int, _P, ctypes.c_int, _P, ctypes.c_int,
            ctypes.c_uint32, _P, _P,
        ]
        _lib_cache[key] = lib
    return _lib_cache[key]


# ---------------------------------------------------------------------------
# oracle (C restatement)
# ---------------------------------------------------------------------------
def oracle_sample(logits, params, hist=None, hist_len=None, masks=None, u=None, top_cap=0,
                  want_logits=False, n_threads=None, bf16=False):
    """Run the C restatement over a batch.

    logits: [B, V] float32, or uint16 bf16 bits when ``bf16``.
    Returns (results[B] of RESULT, top_ids, top_probs, logits_after or None).
    """
    lib = oracle_lib()
    logits = np.ascontiguousarray(logits)
    B, V = logits.shape
    params = np.ascontiguousarray(params, dtype=ROW_PARAMS)
    assert params.shape == (B,)
    if hist is not None:
        hist = np.ascontiguousarray(hist, dtype=np.int32)
        hist_len = np.ascontiguousarray(hist_len, dtype=np.int32)
        hstride = hist.shape[1]
    else:
        hstride = 0
    mstride = 0
    if masks is not None:
        masks = np.ascontiguousarray(masks, dtype=np.uint32)
        mstride = masks.shape[1] if masks.ndim == 2 else 0
    if u is not None:
        u = np.ascontiguousarray(u, dtype=np.float64)
    out = np.zeros(B, dtype=RESULT)
    top_ids = np.full((B, max(top_cap, 1)), -1, np.int32) if top_cap else None
    top_probs = np.zeros((B, max(top_cap, 1)), np.float32) if top_cap else None
    lo = np.empty((B, V), np.float32) if want_logits else None
    nt = n_threads or max(1, os.cpu_count() or 1)
    rc = lib.qso_sample_batch(
        _ptr(logits), 1 if bf16 else 0, B, V, V, _ptr(params), _ptr(hist), hstride, _ptr(hist_len),
        _ptr(masks), mstride, _ptr(u), _ptr(out), _ptr(top_ids), _ptr(top_probs), top_cap, _ptr(lo), nt,
    )
    if rc != 0:
        raise RuntimeError(f"qso_sample_batch failed: {rc}")
    return out, top_ids, top_probs, lo


# ---------------------------------------------------------------------------
# reference (unmodified sources)
# ---------------------------------------------------------------------------
def ref_temperature_sample(logits_row, hist_row, T, rep, lookback, k, p, seed, kind="strict",
                           want_logits=False):
    lib = ref_lib(kind)
    x = np.ascontiguousarray(logits_row, dtype=np.float32)
    h = np.ascontiguousarray(hist_row if hist_row is not None else np.zeros(0, np.int32), dtype=np.int32)
    u = ctypes.c_double()
    drew = ctypes.c_int()
    lo = np.empty_like(x) if want_logits else None
    tok = lib.qwref_temperature_sample(
        _ptr(x), x.size, _ptr(h), h.size, T, rep, lookback, k, p, seed, ctypes.byref(u),
        ctypes.byref(drew), _ptr(lo),
    )
    return tok, u.value, drew.value, lo


def ref_greedy_sample(logits_row, hist_row, rep, lookback, kind="strict", want_logits=False):
    lib = ref_lib(kind)
    x = np.ascontiguousarray(logits_row, dtype=np.float32)
    h = np.ascontiguousarray(hist_row if hist_row is not None else np.zeros(0, np.int32), dtype=np.int32)
    lo = np.empty_like(x) if want_logits else None
    tok = lib.qwref_greedy_sample(_ptr(x), x.size, _ptr(h), h.size, rep, lookback, _ptr(lo))
    return tok, lo


def ref_first_uniform(seed, kind="strict"):
    return ref_lib(kind).qwref_first_uniform(seed)


class RefVocab:
    """A reference std::vector<std::string> vocabulary (plus optional trie)."""

    def __init__(self, strs, kind="strict", trie=True):
        self.lib = ref_lib(kind)
        bs = [s.encode("latin-1") if isinstance(s, str) else bytes(s) for s in strs]
        self._bufs = [ctypes.create_string_buffer(b, len(b) + 1) for b in bs]
        arr = (ctypes.c_void_p * len(bs))(*[ctypes.addressof(b) for b in self._bufs])
        lens = np.array([len(b) for b in bs], np.int32)
        self.V = len(bs)
        self.handle = self.lib.qwref_vocab_new(ctypes.cast(arr, _P), _ptr(lens), len(bs))
        self.trie = self.lib.qwref_trie_new(self.handle) if trie else None

    def close(self):
        if self.trie:
            self.lib.qwref_trie_free(self.trie)
            self.trie = None
        if self.handle:
            self.lib.qwref_vocab_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefGrammar:
    """The reference GrammarVocab (GBNF pushdown grammar) behind a handle."""

    def __init__(self, gbnf: str, vocab: RefVocab, kind="strict"):
        self.lib = ref_lib(kind)
        self.vocab = vocab
        self.handle = self.lib.qwref_grammar_parse(gbnf.encode())
        if not self.handle:
            raise ValueError("GBNF parse failed")
        if vocab.trie:
            self.lib.qwref_grammar_set_trie(self.handle, vocab.trie)

    def valid_tokens(self):
        out = np.empty(self.vocab.V, np.int32)
        n = self.lib.qwref_grammar_valid(self.handle, self.vocab.handle, _ptr(out), out.size)
        return out[:n].copy()

    def accept(self, tok):
        self.lib.qwref_grammar_accept(self.handle, int(tok), self.vocab.handle)

    def accepting(self) -> bool:
        return bool(self.lib.qwref_grammar_accepting(self.handle))

    def reset(self):
        self.lib.qwref_grammar_reset(self.handle)

    def close(self):
        if self.handle:
            self.lib.qwref_grammar_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Philox4x32-10 (production RNG mode; no reference counterpart)
# ---------------------------------------------------------------------------
_PHILOX_M0, _PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
_PHILOX_W0, _PHILOX_W1 = 0x9E3779B9, 0xBB67AE85
_M32 = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Philox4x32 with 10 rounds, the published counter-based generator of
    Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1,
    2, 3" (SC'11): per round, two 32x32->64 multiplies of counter words 0 and
    2 by M0 / M1, the high halves XORed with the other counter words and the
    key, the key bumped by the Weyl constants W0 / W1 between rounds.
    ctr: 4 uint32, key: 2 uint32 -> 4 uint32."""
    c0, c1, c2, c3 = (int(v) & _M32 for v in ctr)
    k0, k1 = (int(v) & _M32 for v in key)
    for _ in range(10):
        p0 = _PHILOX_M0 * c0
        p1 = _PHILOX_M1 * c2
        hi0, lo0 = p0 >> 32, p0 & _M32
        hi1, lo1 = p1 >> 32, p1 & _M32
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        k0 = (k0 + _PHILOX_W0) & _M32
        k1 = (k1 + _PHILOX_W1) & _M32
    return c0, c1, c2, c3


def philox_uniform(seed: int, offset: int, row: int) -> float:
    """The uniform the library's u == NULL mode draws for `row`: Philox4x32-10
    with key = seed (low word first) and counter = (row, 0, offset low,
    offset high); the first two output words g1, g2 become
    (g1 + g2 * 2^32) / 2^64 rounded once to double (the form
    std::generate_canonical<double,53> gives two 32-bit draws), kept below 1."""
    seed, offset = int(seed), int(offset)
    g = philox4x32_10((row & _M32, 0, offset & _M32, (offset >> 32) & _M32), (seed & _M32, (seed >> 32) & _M32))
    s = float(g[0]) + float(g[1]) * 4294967296.0
    u = s * 5.421010862427522e-20
    if u >= 1.0:
        u = float(np.nextafter(1.0, 0.0))
    return u


def reference_root():
    """The reference source tree, where it is present: $QWENIUM_REF, else a
    `reference` directory beside this repository's checkout. None when
    neither exists (the GPU box: the checker libraries travel prebuilt)."""
    cand = os.environ.get("QWENIUM_REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(os.path.join(cand, "src", "sampling")) else None
