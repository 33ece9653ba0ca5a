"""Python host binding of the qsamp C ABI (include/qsamp.h).

Loads the in-tree ``libqsamp.so`` (built by ``qwenium_b200/build.py``) through
ctypes. There is no fallback: if the library or a CUDA device is missing, the
calls raise.

The host-side classes mirror the reference's sampler API
(src/sampling/sampling.h:15-93): ``GreedySampler`` / ``TemperatureSampler``
with the same constructor arguments and defaults, ``sample(logits,
last_tokens, token_strs)``, ``set_grammar``, ``set_pruned_vocab`` and
``set_eos_token_id``; ``sample`` raises on empty logits like
sampling.cpp:101,140. ``Context.sample_batch`` is the batched device entry.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqsamp.so")

# qsamp_row_params (include/qsamp.h): 48 bytes, naturally aligned.
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

# qsamp_row_result: 32 bytes.
ROW_RESULT = np.dtype(
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
assert ROW_RESULT.itemsize == 32

QSAMP_F32, QSAMP_BF16 = 0, 1
STATUS = {0: "OK", 1: "INVALID_ARG", 2: "CUDA", 3: "UNSUPPORTED", 4: "DEVICE", 5: "NO_MEMORY", 6: "IO", 7: "TIMEOUT",
          8: "COMM"}

EXPORTS = (
    "qsamp_create", "qsamp_destroy", "qsamp_last_error", "qsamp_sample", "qsamp_sample_host",
    "qsamp_pack_ids", "qsamp_grammar_mask", "qsamp_find_eos_string", "qsamp_keep_list_mask",
    "qsamp_mask_and", "qsamp_shard_topk", "qsamp_merge_topk", "qsamp_get_counters", "qsamp_set_kernel_timing",
    "qsamp_sample_static", "qsamp_first_byte_table", "qsamp_char_class_masks", "qsamp_verify_greedy",
    "qsamp_poll_status", "qsamp_set_limits", "qsamp_get_limits",
    "qsamp_trie_build", "qsamp_trie_free", "qsamp_trie_token_count", "qsamp_trie_memory_bytes",
    "qsamp_trie_collect_by_prefix", "qsamp_trie_collect_by_char_class", "qsamp_trie_collect_by_first_char",
    "qsamp_trie_mark_char_class",
)

_P = ctypes.c_void_p


class QsampError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"qsamp {STATUS.get(status, status)}: {msg}")
        self.status = status


class _Batch(ctypes.Structure):
    _fields_ = [
        ("logits", _P),
        ("dtype", ctypes.c_int),
        ("B", ctypes.c_int32),
        ("V", ctypes.c_int32),
        ("row_stride", ctypes.c_int64),
        ("params", _P),
        ("hist", _P),
        ("hist_stride", ctypes.c_int32),
        ("hist_len", _P),
        ("masks", _P),
        ("mask_stride", ctypes.c_int64),
        ("u", _P),
        ("rng_offset", ctypes.c_uint64),
        ("out_ids", _P),
        ("out_results", _P),
        ("out_top_ids", _P),
        ("out_top_probs", _P),
        ("top_cap", ctypes.c_int32),
    ]


class _Counters(ctypes.Structure):
    _fields_ = [
        ("calls", ctypes.c_uint64),
        ("rows", ctypes.c_uint64),
        ("logit_bytes", ctypes.c_uint64),
        ("gather_rounds", ctypes.c_uint64),
        ("last_call_us", ctypes.c_double),
        ("kernel_launches", ctypes.c_uint64),
        ("last_stream_kernel_ms", ctypes.c_double),
        ("last_rows_kernel_ms", ctypes.c_double),
        ("last_merge_kernel_ms", ctypes.c_double),
        ("last_stream_rows", ctypes.c_int32),
        ("last_cluster_rows", ctypes.c_int32),
        ("last_cluster_size", ctypes.c_int32),
        ("last_clusters", ctypes.c_int32),
        ("last_hist_rows", ctypes.c_int32),
        ("last_hist_handed_on", ctypes.c_int32),
        ("last_hist_kernel_ms", ctypes.c_double),
        ("last_live_candidates", ctypes.c_int32),
        ("last_live_rows", ctypes.c_int32),
        ("last_live_returned", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("last_live_kernel_ms", ctypes.c_double),
    ]


class _Limits(ctypes.Structure):
    _fields_ = [
        ("max_rounds", ctypes.c_int32),
        ("drop_ready_from", ctypes.c_int32),
        ("ready_wait_ns", ctypes.c_int64),
        ("hist_path", ctypes.c_int32),
        ("live_path", ctypes.c_int32),
    ]


_lib = None


def load(path: str = LIB_PATH):
    """Load libqsamp.so; raises if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python qwenium_b200/build.py`")
    lib = ctypes.CDLL(path)
    lib.qsamp_create.restype = ctypes.c_int
    lib.qsamp_create.argtypes = [ctypes.c_int32, ctypes.POINTER(_P)]
    lib.qsamp_destroy.restype = None
    lib.qsamp_destroy.argtypes = [_P]
    lib.qsamp_last_error.restype = ctypes.c_char_p
    lib.qsamp_last_error.argtypes = [_P]
    lib.qsamp_sample.restype = ctypes.c_int
    lib.qsamp_sample.argtypes = [_P, ctypes.POINTER(_Batch), _P]
    lib.qsamp_sample_host.restype = ctypes.c_int
    lib.qsamp_sample_host.argtypes = [_P, ctypes.POINTER(_Batch)]
    lib.qsamp_pack_ids.restype = ctypes.c_int
    lib.qsamp_pack_ids.argtypes = [_P, ctypes.c_int64, ctypes.c_int32, _P]
    lib.qsamp_grammar_mask.restype = ctypes.c_int
    lib.qsamp_grammar_mask.argtypes = [_P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _P, _P]
    lib.qsamp_find_eos_string.restype = ctypes.c_int32
    lib.qsamp_find_eos_string.argtypes = [_P, _P, ctypes.c_int32]
    lib.qsamp_keep_list_mask.restype = ctypes.c_int
    lib.qsamp_keep_list_mask.argtypes = [ctypes.c_char_p, ctypes.c_int32, _P]
    lib.qsamp_mask_and.restype = ctypes.c_int
    lib.qsamp_mask_and.argtypes = [_P, _P, ctypes.c_int64, _P]
    lib.qsamp_shard_topk.restype = ctypes.c_int
    lib.qsamp_shard_topk.argtypes = [_P, ctypes.POINTER(_Batch), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                     _P, _P, _P]
    lib.qsamp_merge_topk.restype = ctypes.c_int
    lib.qsamp_merge_topk.argtypes = [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, _P, _P, _P,
                                     ctypes.c_uint64, _P, _P, _P]
    lib.qsamp_get_counters.restype = ctypes.c_int
    lib.qsamp_get_counters.argtypes = [_P, ctypes.POINTER(_Counters)]
    lib.qsamp_verify_greedy.restype = ctypes.c_int
    lib.qsamp_verify_greedy.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                        ctypes.c_int32, _P, _P, ctypes.c_int32, _P, _P, _P, _P]
    lib.qsamp_first_byte_table.restype = ctypes.c_int
    lib.qsamp_first_byte_table.argtypes = [_P, _P, ctypes.c_int32, _P]
    lib.qsamp_char_class_masks.restype = ctypes.c_int
    lib.qsamp_char_class_masks.argtypes = [_P, _P, ctypes.c_int32, ctypes.c_int32, _P, _P, ctypes.c_int64,
                                           ctypes.c_int32, _P]
    lib.qsamp_set_kernel_timing.restype = ctypes.c_int
    lib.qsamp_set_kernel_timing.argtypes = [_P, ctypes.c_int32]
    lib.qsamp_sample_static.restype = ctypes.c_int
    lib.qsamp_sample_static.argtypes = [ctypes.POINTER(_Batch), _P, ctypes.c_char_p, ctypes.c_size_t]
    lib.qsamp_poll_status.restype = ctypes.c_int
    lib.qsamp_poll_status.argtypes = [_P]
    lib.qsamp_set_limits.restype = ctypes.c_int
    lib.qsamp_set_limits.argtypes = [_P, ctypes.POINTER(_Limits)]
    lib.qsamp_get_limits.restype = ctypes.c_int
    lib.qsamp_get_limits.argtypes = [_P, ctypes.POINTER(_Limits)]
    lib.qsamp_trie_build.restype = ctypes.c_int
    lib.qsamp_trie_build.argtypes = [_P, _P, ctypes.c_int32, ctypes.POINTER(_P)]
    lib.qsamp_trie_free.restype = None
    lib.qsamp_trie_free.argtypes = [_P]
    for f in ("qsamp_trie_token_count", "qsamp_trie_memory_bytes"):
        getattr(lib, f).restype = ctypes.c_int64
        getattr(lib, f).argtypes = [_P]
    lib.qsamp_trie_collect_by_prefix.restype = ctypes.c_int64
    lib.qsamp_trie_collect_by_prefix.argtypes = [_P, ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32, _P,
                                                 ctypes.c_int64]
    lib.qsamp_trie_collect_by_char_class.restype = ctypes.c_int64
    lib.qsamp_trie_collect_by_char_class.argtypes = [_P, _P, ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_int64]
    lib.qsamp_trie_collect_by_first_char.restype = ctypes.c_int64
    lib.qsamp_trie_collect_by_first_char.argtypes = [_P, ctypes.c_uint8, _P, ctypes.c_int64]
    lib.qsamp_trie_mark_char_class.restype = ctypes.c_int
    lib.qsamp_trie_mark_char_class.argtypes = [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P]
    _lib = lib
    return lib


def _np_ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _dev_ptr(t):
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return int(t)


# ---------------------------------------------------------------- masks
def words_for(V: int) -> int:
    return (V + 31) // 32


def pack_ids(ids, V: int) -> np.ndarray:
    """Allow-bits for ids (qsamp_pack_ids)."""
    lib = load()
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.zeros(words_for(V), np.uint32)
    rc = lib.qsamp_pack_ids(_np_ptr(ids), ids.size, V, _np_ptr(out))
    if rc:
        raise QsampError(rc, "qsamp_pack_ids")
    return out


def grammar_mask(valid_ids, accepting: bool, eos_string_id: int, eos_token_id: int, V: int):
    """(mask, force_token) per Sampler::apply_grammar_constraints."""
    lib = load()
    ids = np.ascontiguousarray(valid_ids, np.int32)
    out = np.zeros(words_for(V), np.uint32)
    force = ctypes.c_int32(-1)
    rc = lib.qsamp_grammar_mask(_np_ptr(ids), ids.size, int(bool(accepting)), eos_string_id, eos_token_id, V,
                                _np_ptr(out), ctypes.addressof(force))
    if rc:
        raise QsampError(rc, "qsamp_grammar_mask")
    return out, force.value


def find_eos_string(strs: Sequence) -> int:
    lib = load()
    bs = [s.encode("latin-1") if isinstance(s, str) else bytes(s) for s in strs]
    bufs = [ctypes.create_string_buffer(b, len(b) + 1) for b in bs]
    arr = (ctypes.c_void_p * len(bs))(*[ctypes.addressof(b) for b in bufs])
    lens = np.array([len(b) for b in bs], np.int32)
    return lib.qsamp_find_eos_string(ctypes.cast(arr, _P), _np_ptr(lens), len(bs))


def first_byte_table(strs: Sequence) -> np.ndarray:
    """qsamp_first_byte_table: first byte of each token (256: empty token)."""
    lib = load()
    bs = [s.encode("latin-1") if isinstance(s, str) else bytes(s) for s in strs]
    bufs = [ctypes.create_string_buffer(b, len(b) + 1) for b in bs]
    arr = (ctypes.c_void_p * len(bs))(*[ctypes.addressof(b) for b in bufs])
    lens = np.array([len(b) for b in bs], np.int32)
    out = np.empty(len(bs), np.uint16)
    rc = lib.qsamp_first_byte_table(ctypes.cast(arr, _P), _np_ptr(lens), len(bs), _np_ptr(out))
    if rc:
        raise QsampError(rc, "qsamp_first_byte_table")
    return out


def char_class_bits(chars, negated: bool) -> np.ndarray:
    """The 256-bit allowed set of a grammar char class (8 uint32 words), as
    TokenTrie::mark_char_class builds its lookup table (token-trie.cpp:96-104):
    the class's bytes, or their complement for a negated class."""
    allowed = np.zeros(256, bool)
    idx = np.array([int(c) if isinstance(c, (int, np.integer)) else ord(c) for c in chars], np.int64) & 0xFF
    allowed[idx] = True
    if negated:
        allowed = ~allowed
    return np.packbits(allowed, bitorder="little").view(np.uint32).copy()


def keep_list_mask(path: str, V: int) -> np.ndarray:
    lib = load()
    out = np.zeros(words_for(V), np.uint32)
    rc = lib.qsamp_keep_list_mask(path.encode(), V, _np_ptr(out))
    if rc:
        raise QsampError(rc, f"keep list {path!r}")
    return out


def mask_and(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    lib = load()
    a = np.ascontiguousarray(a, np.uint32)
    b = np.ascontiguousarray(b, np.uint32)
    out = np.empty_like(a)
    rc = lib.qsamp_mask_and(_np_ptr(a), _np_ptr(b), a.size, _np_ptr(out))
    if rc:
        raise QsampError(rc, "qsamp_mask_and")
    return out


# ---------------------------------------------------------------- context
class Context:
    """A qsamp_ctx bound to one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = _P()
        rc = self.lib.qsamp_create(int(device), ctypes.byref(h))
        if rc:
            raise QsampError(rc, f"qsamp_create(device={device})")
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self.lib.qsamp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str):
        if rc:
            raise QsampError(rc, f"{what}: {self.lib.qsamp_last_error(self.h).decode(errors='replace')}")

    def set_kernel_timing(self, on: bool):
        """Bracket each selection kernel with CUDA events (see counters())."""
        self._check(self.lib.qsamp_set_kernel_timing(self.h, 1 if on else 0), "qsamp_set_kernel_timing")

    def poll_status(self) -> None:
        """qsamp_poll_status: raises QsampError (DEVICE) when the last
        asynchronous call's kernels hit a device-side limit; call it after
        synchronising that call's stream."""
        self._check(self.lib.qsamp_poll_status(self.h), "qsamp_poll_status")

    def limits(self) -> dict:
        lim = _Limits()
        self._check(self.lib.qsamp_get_limits(self.h, ctypes.byref(lim)), "qsamp_get_limits")
        return {f: getattr(lim, f) for f, _ in lim._fields_}

    def set_limits(self, max_rounds=None, ready_wait_ns=None, drop_ready_from=None, hist_path=None,
                   live_path=None) -> None:
        """qsamp_set_limits; arguments left None keep their current value."""
        cur = self.limits()
        lim = _Limits()
        lim.max_rounds = cur["max_rounds"] if max_rounds is None else int(max_rounds)
        lim.ready_wait_ns = cur["ready_wait_ns"] if ready_wait_ns is None else int(ready_wait_ns)
        lim.drop_ready_from = cur["drop_ready_from"] if drop_ready_from is None else int(drop_ready_from)
        lim.hist_path = cur["hist_path"] if hist_path is None else int(hist_path)
        lim.live_path = cur["live_path"] if live_path is None else int(live_path)
        self._check(self.lib.qsamp_set_limits(self.h, ctypes.byref(lim)), "qsamp_set_limits")

    def verify_greedy(self, logits, row_off, drafts, eos_token: int = -1, stream=None):
        """qsamp_verify_greedy on CUDA tensors: logits [n_rows][V] (fp32, or
        bf16 bits as int16/bfloat16), row_off int32 [B+1], drafts int32
        [n_rows]. Returns (accepted, bonus, has_bonus) int32 [B] tensors."""
        import torch

        n_rows, V = int(logits.shape[0]), int(logits.shape[1])
        B = int(row_off.shape[0]) - 1
        dtype = QSAMP_BF16 if logits.dtype in (torch.bfloat16, torch.int16, torch.uint16) else QSAMP_F32
        acc = torch.empty(B, dtype=torch.int32, device=row_off.device)
        bonus = torch.empty_like(acc)
        has = torch.empty_like(acc)
        if stream is None:
            stream = torch.cuda.current_stream(row_off.device).cuda_stream
        self._check(self.lib.qsamp_verify_greedy(self.h, _dev_ptr(logits), dtype, V, int(logits.stride(0)), n_rows, B,
                                                 _dev_ptr(row_off), _dev_ptr(drafts), int(eos_token), _dev_ptr(acc),
                                                 _dev_ptr(bonus), _dev_ptr(has), ctypes.c_void_p(stream)),
                    "qsamp_verify_greedy")
        return acc, bonus, has

    def char_class_masks(self, table, classes, masks, or_into: bool = False, stream=None):
        """qsamp_char_class_masks on CUDA tensors: table uint16 [V] (as int16),
        classes uint32 [B][8] (as int32), masks uint32 [B][stride] (as int32)."""
        import torch

        V = int(table.shape[0])
        B = int(classes.shape[0])
        if stream is None:
            stream = torch.cuda.current_stream(masks.device).cuda_stream
        self._check(self.lib.qsamp_char_class_masks(self.h, _dev_ptr(table), V, B, _dev_ptr(classes), _dev_ptr(masks),
                                                    int(masks.stride(0)), 1 if or_into else 0,
                                                    ctypes.c_void_p(stream)), "qsamp_char_class_masks")
        return masks

    def counters(self) -> dict:
        c = _Counters()
        self._check(self.lib.qsamp_get_counters(self.h, ctypes.byref(c)), "qsamp_get_counters")
        return {f: getattr(c, f) for f, _ in c._fields_}

    @staticmethod
    def _batch(logits_ptr, dtype, B, V, row_stride, params, hist_ptr, hist_stride, hist_len, masks_ptr,
               mask_stride, u, rng_offset, out_ids_ptr, out_res_ptr, top_ids_ptr, top_probs_ptr, top_cap):
        b = _Batch()
        b.logits = logits_ptr
        b.dtype = dtype
        b.B = B
        b.V = V
        b.row_stride = row_stride
        b.params = _np_ptr(params)
        b.hist = hist_ptr
        b.hist_stride = hist_stride
        b.hist_len = _np_ptr(hist_len)
        b.masks = masks_ptr
        b.mask_stride = mask_stride
        b.u = _np_ptr(u)
        b.rng_offset = rng_offset
        b.out_ids = out_ids_ptr
        b.out_results = out_res_ptr
        b.out_top_ids = top_ids_ptr
        b.out_top_probs = top_probs_ptr
        b.top_cap = top_cap
        return b

    def sample_batch(self, logits, params, hist=None, hist_len=None, masks=None, u=None, rng_offset=0,
                     out_ids=None, out_results=None, top_cap=0, out_top_ids=None, out_top_probs=None,
                     stream=None):
        """Device entry (qsamp_sample). logits/hist/masks/out_* are CUDA
        tensors (torch) or raw device pointers; params/hist_len/u are host
        numpy arrays. Asynchronous on `stream` (default: torch's current)."""
        import torch

        B, V = int(logits.shape[0]), int(logits.shape[1])
        dtype = QSAMP_BF16 if logits.dtype in (torch.bfloat16, torch.int16, torch.uint16) else QSAMP_F32
        params = np.ascontiguousarray(params, ROW_PARAMS)
        if hist_len is not None:
            hist_len = np.ascontiguousarray(hist_len, np.int32)
        if u is not None:
            u = np.ascontiguousarray(u, np.float64)
        if out_results is None:
            out_results = torch.empty((B, ROW_RESULT.itemsize), dtype=torch.uint8, device=logits.device)
        if stream is None:
            stream = torch.cuda.current_stream(logits.device).cuda_stream
        mstride = 0
        if masks is not None and masks.dim() == 2:
            mstride = int(masks.stride(0))
        b = self._batch(
            logits.data_ptr(), dtype, B, V, int(logits.stride(0)), params, _dev_ptr(hist),
            int(hist.stride(0)) if hist is not None else 0, hist_len, _dev_ptr(masks), mstride, u, rng_offset,
            _dev_ptr(out_ids), _dev_ptr(out_results), _dev_ptr(out_top_ids), _dev_ptr(out_top_probs), top_cap,
        )
        self._check(self.lib.qsamp_sample(self.h, ctypes.byref(b), ctypes.c_void_p(stream)), "qsamp_sample")
        return out_results

    def shard_topk(self, local_logits, params, v_offset: int, V_total: int, k: int, hist=None, hist_len=None,
                   masks=None, cand_vals=None, cand_ids=None, stream=None):
        """Vocab-sharded step 1 (qsamp_shard_topk): this rank's logits
        [B][V_local] hold global ids [v_offset, v_offset + V_local). Returns
        (cand_vals [B][k] float32, cand_ids [B][k] int32 global ids, -1 for
        padding) on the logits' device. hist holds global ids; masks cover
        the local slice (bit i <-> global id v_offset + i)."""
        import torch

        B = int(local_logits.shape[0])
        if cand_vals is None:
            cand_vals = torch.empty((B, k), dtype=torch.float32, device=local_logits.device)
        if cand_ids is None:
            cand_ids = torch.empty((B, k), dtype=torch.int32, device=local_logits.device)
        dtype = QSAMP_BF16 if local_logits.dtype in (torch.bfloat16, torch.int16, torch.uint16) else QSAMP_F32
        params = np.ascontiguousarray(params, ROW_PARAMS)
        if hist_len is not None:
            hist_len = np.ascontiguousarray(hist_len, np.int32)
        if stream is None:
            stream = torch.cuda.current_stream(local_logits.device).cuda_stream
        mstride = int(masks.stride(0)) if masks is not None and masks.dim() == 2 else 0
        b = self._batch(
            local_logits.data_ptr(), dtype, B, int(local_logits.shape[1]), int(local_logits.stride(0)), params,
            _dev_ptr(hist), int(hist.stride(0)) if hist is not None else 0, hist_len, _dev_ptr(masks), mstride, None,
            0, None, None, None, None, 0,
        )
        self._check(self.lib.qsamp_shard_topk(self.h, ctypes.byref(b), int(v_offset), int(V_total), int(k),
                                              _dev_ptr(cand_vals), _dev_ptr(cand_ids), ctypes.c_void_p(stream)),
                    "qsamp_shard_topk")
        return cand_vals, cand_ids

    def merge_topk(self, all_vals, all_ids, params, u=None, rng_offset=0, out_ids=None, out_results=None,
                   stream=None):
        """Vocab-sharded step 2 (qsamp_merge_topk): all_vals / all_ids are the
        all-gathered candidates [n_ranks][B][k] (CUDA tensors)."""
        import torch

        n_ranks, B, k = (int(x) for x in all_vals.shape)
        params = np.ascontiguousarray(params, ROW_PARAMS)
        if u is not None:
            u = np.ascontiguousarray(u, np.float64)
        if out_results is None:
            out_results = torch.empty((B, ROW_RESULT.itemsize), dtype=torch.uint8, device=all_vals.device)
        if stream is None:
            stream = torch.cuda.current_stream(all_vals.device).cuda_stream
        self._check(self.lib.qsamp_merge_topk(self.h, n_ranks, B, k, _dev_ptr(all_vals), _dev_ptr(all_ids),
                                              _np_ptr(params), _np_ptr(u), int(rng_offset), _dev_ptr(out_ids),
                                              _dev_ptr(out_results), ctypes.c_void_p(stream)), "qsamp_merge_topk")
        return out_results

    def sample_host(self, logits: np.ndarray, params, hist=None, hist_len=None, masks=None, u=None, rng_offset=0,
                    top_cap=0, bf16=False, status_out=None):
        """Host-memory entry (qsamp_sample_host): numpy in, numpy out.
        With status_out (a list), a device-side status (QSAMP_ERR_DEVICE) is
        appended to it instead of raised, and the outputs are returned."""
        logits = np.ascontiguousarray(logits)
        B, V = logits.shape
        params = np.ascontiguousarray(params, ROW_PARAMS)
        hist_ptr, hstride = None, 0
        if hist is not None:
            hist = np.ascontiguousarray(hist, np.int32)
            hist_ptr, hstride = _np_ptr(hist), hist.shape[1]
            hist_len = np.ascontiguousarray(hist_len if hist_len is not None else np.full(B, hstride), np.int32)
        mptr, mstride = None, 0
        if masks is not None:
            masks = np.ascontiguousarray(masks, np.uint32)
            mptr = _np_ptr(masks)
            mstride = masks.shape[1] if masks.ndim == 2 else 0
        if u is not None:
            u = np.ascontiguousarray(u, np.float64)
        ids = np.empty(B, np.int32)
        res = np.zeros(B, ROW_RESULT)
        top_ids = np.empty((B, max(top_cap, 1)), np.int32) if top_cap else None
        top_probs = np.empty((B, max(top_cap, 1)), np.float32) if top_cap else None
        b = self._batch(_np_ptr(logits), QSAMP_BF16 if bf16 else QSAMP_F32, B, V, V, params, hist_ptr, hstride,
                        hist_len, mptr, mstride, u, rng_offset, _np_ptr(ids), _np_ptr(res), _np_ptr(top_ids),
                        _np_ptr(top_probs), top_cap)
        rc = self.lib.qsamp_sample_host(self.h, ctypes.byref(b))
        if status_out is not None and rc == 4:
            status_out.append((rc, self.lib.qsamp_last_error(self.h).decode(errors="replace")))
        else:
            self._check(rc, "qsamp_sample_host")
        return ids, res, top_ids, top_probs


# ---------------------------------------------------------------- reference-shaped API
class Sampler:
    """Mirror of qwenium::Sampler (sampling.h:15-51) over the CUDA path."""

    def __init__(self, device: int = 0):
        self._ctx = Context(device)
        self._grammar = None
        self._pruned = None
        self._eos_token_id = -1
        self._eos_string = None

    def set_grammar(self, grammar):
        """grammar: an object with get_valid_tokens(vocab) and
        is_accepting_state() (the GrammarVocab interface, grammar_vocab.h)."""
        self._grammar = grammar

    def set_pruned_vocab(self, ids):
        self._pruned = None if ids is None else np.asarray(sorted(ids), np.int32)

    def set_eos_token_id(self, token_id: int):
        self._eos_token_id = int(token_id)

    def _params(self) -> np.ndarray:
        raise NotImplementedError

    def sample(self, logits, last_tokens=(), token_strs=()) -> int:
        x = np.ascontiguousarray(logits, np.float32).reshape(1, -1)
        if x.size == 0:
            raise RuntimeError("Cannot sample from empty logits")
        V = x.shape[1]
        p = self._params()
        mask = None
        if self._pruned is not None:
            mask = pack_ids(self._pruned, V)
        if self._grammar is not None and len(token_strs):
            if self._eos_string is None:
                self._eos_string = find_eos_string(token_strs)
            valid = self._grammar.get_valid_tokens(token_strs)
            gm, force = grammar_mask(valid, self._grammar.is_accepting_state(), self._eos_string,
                                     self._eos_token_id, V)
            p["force_token"] = force
            mask = gm if mask is None else mask_and(mask, gm)
        hist = np.ascontiguousarray(last_tokens, np.int32).reshape(1, -1) if len(last_tokens) else None
        u = self._next_u()
        ids, _, _, _ = self._ctx.sample_host(x, p, hist=hist, hist_len=None if hist is None else [hist.shape[1]],
                                             masks=mask, u=u)
        return int(ids[0])

    def _next_u(self):
        return None


class GreedySampler(Sampler):
    """GreedySampler(repetition_penalty=1.2, repetition_lookback=32), sampling.h:53-69."""

    def __init__(self, repetition_penalty: float = 1.2, repetition_lookback: int = 32, device: int = 0):
        super().__init__(device)
        self.repetition_penalty = repetition_penalty
        self.repetition_lookback = repetition_lookback

    def _params(self):
        p = np.zeros(1, ROW_PARAMS)
        p["temperature"] = 0.0
        p["repetition_penalty"] = self.repetition_penalty
        p["repetition_lookback"] = self.repetition_lookback
        p["force_token"] = -1
        return p


class TemperatureSampler(Sampler):
    """TemperatureSampler(temperature=0.7, repetition_penalty=1.1,
    repetition_lookback=64, top_k=40, top_p=0.95), sampling.h:71-93. The
    draw uses u from `uniform` (a callable) when given -- e.g. the
    reference engine's stream -- else the device Philox stream keyed by seed."""

    def __init__(self, temperature: float = 0.7, repetition_penalty: float = 1.1, repetition_lookback: int = 64,
                 top_k: int = 40, top_p: float = 0.95, device: int = 0, seed: int = 0, uniform=None):
        super().__init__(device)
        self.temperature = temperature
        self.repetition_penalty = repetition_penalty
        self.repetition_lookback = repetition_lookback
        self.top_k = top_k
        self.top_p = top_p
        self.seed = seed
        self.uniform = uniform
        self.step = 0

    def _params(self):
        p = np.zeros(1, ROW_PARAMS)
        p["temperature"] = self.temperature
        p["top_k"] = self.top_k
        p["top_p"] = self.top_p
        p["repetition_penalty"] = self.repetition_penalty
        p["repetition_lookback"] = self.repetition_lookback
        p["force_token"] = -1
        p["seed"] = self.seed
        return p

    def _next_u(self):
        if self.uniform is None:
            return None
        return np.array([self.uniform()], np.float64)


STATIC_MAX_ROWS = 4096  # QSAMP_STATIC_MAX_ROWS in include/qsamp.h


def sample_static(logits, params, hist=None, hist_len=None, masks=None, u=None, rng_offset=0, out_ids=None,
                  out_results=None, stream=None):
    """qsamp_sample_static: the allocation-free entry point (no context).
    Same arguments as Context.sample_batch; every output must be supplied."""
    import torch

    lib = load()
    B, V = int(logits.shape[0]), int(logits.shape[1])
    dtype = QSAMP_BF16 if logits.dtype in (torch.bfloat16, torch.int16, torch.uint16) else QSAMP_F32
    params = np.ascontiguousarray(params, ROW_PARAMS)
    if hist_len is not None:
        hist_len = np.ascontiguousarray(hist_len, np.int32)
    if u is not None:
        u = np.ascontiguousarray(u, np.float64)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    mstride = int(masks.stride(0)) if masks is not None and masks.dim() == 2 else 0
    b = Context._batch(logits.data_ptr(), dtype, B, V, int(logits.stride(0)), params, _dev_ptr(hist),
                       int(hist.stride(0)) if hist is not None else 0, hist_len, _dev_ptr(masks), mstride, u,
                       rng_offset, _dev_ptr(out_ids), _dev_ptr(out_results), None, None, 0)
    err = ctypes.create_string_buffer(512)
    rc = lib.qsamp_sample_static(ctypes.byref(b), ctypes.c_void_p(stream), err, len(err))
    if rc:
        raise QsampError(rc, "qsamp_sample_static: " + err.value.decode(errors="replace"))


# ---------------------------------------------------------------- compact token trie
class TokenTrie:
    """The reference's TokenTrie queries (src/sampling/token-trie.h:20-64) over
    the library's compact trie (qsamp_trie_*): build(vocab), then
    collect_by_prefix / collect_by_char_class / collect_by_first_char return
    id arrays in the reference's order, mark_char_class a bool array."""

    def __init__(self, vocab: Optional[Sequence] = None):
        self.lib = load()
        self.h = None
        self.V = 0
        if vocab is not None:
            self.build(vocab)

    def build(self, vocab: Sequence) -> None:
        self.close()
        bs = [s.encode("latin-1") if isinstance(s, str) else bytes(s) for s in vocab]
        bufs = [ctypes.create_string_buffer(b, len(b) + 1) for b in bs]
        arr = (ctypes.c_void_p * len(bs))(*[ctypes.addressof(b) for b in bufs])
        lens = np.array([len(b) for b in bs], np.int32)
        h = _P()
        rc = self.lib.qsamp_trie_build(ctypes.cast(arr, _P), _np_ptr(lens), len(bs), ctypes.byref(h))
        if rc:
            raise QsampError(rc, "qsamp_trie_build")
        self.h = h
        self.V = len(bs)

    def close(self):
        if getattr(self, "h", None):
            self.lib.qsamp_trie_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def token_count(self) -> int:
        return int(self.lib.qsamp_trie_token_count(self.h))

    def memory_bytes(self) -> int:
        return int(self.lib.qsamp_trie_memory_bytes(self.h))

    def _collect(self, fn, *args) -> np.ndarray:
        n = fn(self.h, *args, None, 0)
        if n < 0:
            raise QsampError(1, "qsamp_trie query: invalid argument")
        out = np.empty(max(n, 1), np.int32)
        fn(self.h, *args, _np_ptr(out), n)
        return out[:n]

    def collect_by_prefix(self, prefix, offset: int = 0) -> np.ndarray:
        b = prefix.encode("latin-1") if isinstance(prefix, str) else bytes(prefix)
        return self._collect(self.lib.qsamp_trie_collect_by_prefix, b, len(b), int(offset))

    @staticmethod
    def _chars(chars) -> np.ndarray:
        return np.array([c if isinstance(c, (int, np.integer)) else ord(c) for c in chars], np.uint8)

    def collect_by_char_class(self, chars, negated: bool) -> np.ndarray:
        c = self._chars(chars)
        return self._collect(self.lib.qsamp_trie_collect_by_char_class, _np_ptr(c), c.size, int(bool(negated)))

    def collect_by_first_char(self, c) -> np.ndarray:
        return self._collect(self.lib.qsamp_trie_collect_by_first_char, int(c if isinstance(c, int) else ord(c)))

    def mark_char_class(self, chars, negated: bool) -> np.ndarray:
        c = self._chars(chars)
        out = np.zeros(self.V, np.uint8)
        rc = self.lib.qsamp_trie_mark_char_class(self.h, _np_ptr(c), c.size, int(bool(negated)), self.V, _np_ptr(out))
        if rc:
            raise QsampError(rc, "qsamp_trie_mark_char_class")
        return out.astype(bool)
