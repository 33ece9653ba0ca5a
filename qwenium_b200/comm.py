"""Python binding of libqsamp_comm.so (include/qsamp_comm.h): the candidate
exchange of vocab-sharded selection over a non-blocking NCCL communicator
whose every wait has a deadline. An asynchronous NCCL error or a deadline
that passes (a rank that never joins, a peer that died) aborts the
communicator and raises CommError (TIMEOUT or COMM); the communicator is
then dead and is replaced by a new one. Raises if the library is missing
(there is no fallback)."""
from __future__ import annotations

import ctypes
import os
from typing import Optional

from .qsamp import STATUS

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqsamp_comm.so")
ID_BYTES = 128
EXPORTS = ("qsamp_comm_unique_id", "qsamp_comm_create", "qsamp_comm_allgather_candidates", "qsamp_comm_wait",
           "qsamp_comm_status", "qsamp_comm_last_error", "qsamp_comm_destroy", "qsamp_comm_selftest")

_lib = None
_P = ctypes.c_void_p


class CommError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"qsamp_comm {STATUS.get(status, status)}: {msg}")
        self.status = status


def load(path: str = LIB_PATH):
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python qwenium_b200/build.py`")
    lib = ctypes.CDLL(path)
    lib.qsamp_comm_unique_id.restype = ctypes.c_int
    lib.qsamp_comm_unique_id.argtypes = [ctypes.c_char_p]
    lib.qsamp_comm_create.restype = ctypes.c_int
    lib.qsamp_comm_create.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p, ctypes.c_int32, ctypes.c_int64,
                                      ctypes.POINTER(_P), ctypes.c_char_p, ctypes.c_size_t]
    lib.qsamp_comm_allgather_candidates.restype = ctypes.c_int
    lib.qsamp_comm_allgather_candidates.argtypes = [_P, _P, _P, ctypes.c_int64, _P, _P, _P]
    lib.qsamp_comm_wait.restype = ctypes.c_int
    lib.qsamp_comm_wait.argtypes = [_P, _P]
    lib.qsamp_comm_status.restype = ctypes.c_int
    lib.qsamp_comm_status.argtypes = [_P]
    lib.qsamp_comm_last_error.restype = ctypes.c_char_p
    lib.qsamp_comm_last_error.argtypes = [_P]
    lib.qsamp_comm_destroy.restype = None
    lib.qsamp_comm_destroy.argtypes = [_P]
    lib.qsamp_comm_selftest.restype = ctypes.c_int
    lib.qsamp_comm_selftest.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)]
    _lib = lib
    return lib


def unique_id() -> bytes:
    """A new communicator id (rank 0 makes it; every rank passes it on)."""
    lib = load()
    buf = ctypes.create_string_buffer(ID_BYTES)
    rc = lib.qsamp_comm_unique_id(buf)
    if rc:
        raise CommError(rc, "qsamp_comm_unique_id")
    return buf.raw


def selftest(scenario: int, timeout_ms: int):
    """The deadline logic against a fake collective (no GPU): (status, aborted)."""
    lib = load()
    ab = ctypes.c_int32(0)
    rc = lib.qsamp_comm_selftest(scenario, timeout_ms, ctypes.byref(ab))
    return rc, ab.value


class Comm:
    """Rank `rank` of `nranks` on CUDA device `device`; every wait gives up
    after timeout_ms."""

    def __init__(self, nranks: int, rank: int, uid: bytes, device: int, timeout_ms: int = 10000):
        self.lib = load()
        if len(uid) != ID_BYTES:
            raise ValueError(f"uid: expected {ID_BYTES} bytes, got {len(uid)}")
        h = _P()
        err = ctypes.create_string_buffer(512)
        rc = self.lib.qsamp_comm_create(nranks, rank, uid, device, timeout_ms, ctypes.byref(h), err, 512)
        if rc:
            raise CommError(rc, err.value.decode(errors="replace"))
        self.h = h
        self.nranks, self.rank = nranks, rank

    def _check(self, rc: int, what: str):
        if rc:
            raise CommError(rc, f"{what}: {self.lib.qsamp_comm_last_error(self.h).decode(errors='replace')}")

    def allgather_candidates(self, vals, ids, stream=None):
        """vals [B][k] float32 and ids [B][k] int32 CUDA tensors of this rank
        -> [nranks][B][k] each (rank-major), enqueued on `stream` (default:
        torch's current); call wait() before reading them on the host."""
        import torch

        vals, ids = vals.contiguous(), ids.contiguous()
        out_v = torch.empty((self.nranks,) + tuple(vals.shape), dtype=vals.dtype, device=vals.device)
        out_i = torch.empty((self.nranks,) + tuple(ids.shape), dtype=ids.dtype, device=ids.device)
        st = torch.cuda.current_stream(vals.device).cuda_stream if stream is None else stream
        self._check(self.lib.qsamp_comm_allgather_candidates(self.h, vals.data_ptr(), ids.data_ptr(), vals.numel(),
                                                             out_v.data_ptr(), out_i.data_ptr(), st),
                    "qsamp_comm_allgather_candidates")
        return out_v, out_i

    def wait(self, stream=None, device: Optional[int] = None):
        import torch

        st = torch.cuda.current_stream(device).cuda_stream if stream is None else stream
        self._check(self.lib.qsamp_comm_wait(self.h, st), "qsamp_comm_wait")

    def alive(self) -> bool:
        return self.lib.qsamp_comm_status(self.h) == 0

    def close(self):
        if getattr(self, "h", None):
            self.lib.qsamp_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
