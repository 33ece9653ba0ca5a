"""Philox4x32-10, the generator of the library's production RNG mode
(qsamp_batch.u == NULL), against the published known-answer vectors of
Salmon et al., "Parallel random numbers: as easy as 1, 2, 3" (SC'11), as
distributed with their Random123 library (philox4x32, 10 rounds)."""
import numpy as np

import oracle as O

KAT = [
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
     (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


def test_philox_known_answers():
    for ctr, key, want in KAT:
        assert O.philox4x32_10(ctr, key) == want


def test_philox_uniform_range_and_spread():
    # the u of distinct rows / offsets / seeds: in [0, 1), distinct, and
    # roughly uniform (mean of 4096 draws within 5 standard errors of 1/2)
    us = np.array([O.philox_uniform(seed, off, row) for seed in (0, 7, 2**40 + 3) for off in (0, 1, 2**33)
                   for row in range(456)])
    assert us.min() >= 0.0 and us.max() < 1.0
    assert len(np.unique(us)) == len(us)
    assert abs(us.mean() - 0.5) < 5 * np.sqrt(1 / 12 / len(us))
