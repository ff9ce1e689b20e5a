"""The GEMM epilogues divide row and tile indices by launch constants d (the
band count, the number of column tiles) as umulhi(x, ceil(2^32 / d)); the
host enables it only where x * d < 2^32, the bound under which it is exact.
Checked here exhaustively for the bench's d = 62 and at the edges for others."""
import numpy as np


def umulhi_div(x, d):
    m = ((1 << 32) + d - 1) // d
    return (x.astype(np.uint64) * np.uint64(m)) >> np.uint64(32)


def test_band_count_exhaustive():
    d = 62
    lim = (1 << 32) // d
    for lo in range(0, lim, 1 << 24):
        x = np.arange(lo, min(lo + (1 << 24), lim), dtype=np.uint64)
        assert np.array_equal(umulhi_div(x, d), x // np.uint64(d))


def test_edges_other_divisors():
    for d in list(range(2, 130)) + [1000, 4096, 65535]:
        lim = ((1 << 32) - 1) // d
        k = np.arange(0, lim // d + 1, max(1, lim // d // 5000), dtype=np.uint64)
        x = np.concatenate([k * np.uint64(d), k * np.uint64(d) + np.uint64(d - 1),
                            np.array([lim, lim - 1], dtype=np.uint64)])
        x = x[x <= np.uint64(lim)]
        assert np.array_equal(umulhi_div(x, d), x // np.uint64(d)), d
