"""libqsamp_comm.so on CPU: it loads and exports every entry point
include/qsamp_comm.h declares, rejects bad arguments with a message, and its
deadline logic -- run against a fake collective, so nothing waits on a GPU or
a peer -- gives up on time and aborts: a collective that never completes
(TIMEOUT), one whose communicator reports an asynchronous error (COMM), and
one that completes (OK, no abort)."""
import ctypes
import os
import re
import time

import pytest

from qwenium_b200 import comm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OK, INVALID_ARG, TIMEOUT, COMM = 0, 1, 7, 8


def test_exports_every_declared_entry_point():
    lib = comm.load()
    hdr = open(os.path.join(ROOT, "include", "qsamp_comm.h")).read()
    declared = set(re.findall(r"\b(qsamp_comm_\w+)\s*\(", hdr))
    assert declared == set(comm.EXPORTS), declared ^ set(comm.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


@pytest.mark.parametrize("scenario,want,aborted", [(0, TIMEOUT, 1), (1, COMM, 1), (2, OK, 0)])
def test_deadline_logic_against_a_fake_collective(scenario, want, aborted):
    t0 = time.monotonic()
    rc, ab = comm.selftest(scenario, 300)
    el = time.monotonic() - t0
    assert rc == want and ab == aborted, (rc, ab)
    if scenario == 0:
        assert 0.3 <= el < 5.0, el  # gave up at its deadline, not before, not much after
    else:
        assert el < 0.3, el  # the error / the completion ends the wait at once


def test_create_rejects_bad_arguments():
    lib = comm.load()
    uid = b"\0" * comm.ID_BYTES
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    cases = [((0, 0, uid, 0, 1000), "nranks"), ((2, 2, uid, 0, 1000), "rank"), ((2, -1, uid, 0, 1000), "rank"),
             ((2, 0, None, 0, 1000), "id"), ((2, 0, uid, 0, 0), "timeout_ms")]
    for args, name in cases:
        rc = lib.qsamp_comm_create(*args, ctypes.byref(h), err, 256)
        assert rc == INVALID_ARG, (args, rc)
        assert err.value.decode().startswith(name), err.value
        assert not h.value
    with pytest.raises(ValueError):
        comm.Comm(2, 0, b"short", 0)
