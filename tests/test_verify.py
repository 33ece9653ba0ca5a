"""The numpy restatement of greedy draft verification against the
reference's own SpeculativeDecoder::try_speculative_step (compiled harness)."""
import ctypes

import numpy as np
import pytest

from verify_cases import make_cases, verify_one


@pytest.mark.parametrize("seed,V", [(1, 7), (2, 64), (3, 1000), (4, 2)])
def test_restatement_matches_reference(ref_mod, seed, V):
    lib = ref_mod.ref_lib("strict")
    x, drafts, off, eos = make_cases(seed, 40, V)
    for b in range(40):
        r0, r1 = off[b], off[b + 1]
        K = r1 - r0
        if K == 0:
            continue
        rows = np.ascontiguousarray(x[r0:r1])
        d = np.ascontiguousarray(drafts[r0:r1])
        a, bo, h = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        lib.qwref_spec_verify(ref_mod._ptr(rows), int(K), V, ref_mod._ptr(d), eos, ctypes.byref(a), ctypes.byref(bo),
                              ctypes.byref(h))
        assert (a.value, bo.value, h.value) == verify_one(rows, d, eos), (seed, V, b)
