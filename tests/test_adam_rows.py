"""The selective Adam kernel finds the row of element e of a group with D
elements per row as floor(e * M / 2^64) with M = ceil(2^64 / D) (adam.cu,
row_of): exact for every e < 2^32. Checked here in exact integer arithmetic on
the boundaries of every row and on random elements."""

import numpy as np


def magic(D):
    return 0 if D <= 1 else (2**64 - 1) // D + 1  # ~0ull / D + 1 in the kernel's host code


def row_of(e, m):
    return e if m == 0 else (e * m) >> 64


def test_row_of_matches_division():
    rng = np.random.default_rng(0)
    for D in list(range(1, 70)) + [128, 192, 1000, 4096, 65537]:
        m = magic(D)
        assert m < 2**64
        last = 2**32 - 1
        probes = [0, 1, D - 1, D, D + 1, last, last - 1, (last // D) * D, (last // D) * D - 1]
        probes += [int(x) for x in rng.integers(0, 2**32, size=2000, dtype=np.uint64)]
        probes += [k * D + r for k in (1, 7, 1234567) for r in (0, D - 1) if k * D + r < 2**32]
        for e in probes:
            assert row_of(e, m) == e // D, (D, e)
