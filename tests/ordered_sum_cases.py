"""Inputs for the ordered-sum tests: non-negative fp32 vectors with the
rounding cases of a running fp32 sum (exact ties on the sum's grid, binade
crossings, zeros, subnormals, huge terms, inf, NaN), and the sequential sum
they must give.

The sequential fp32 sum is np.cumsum(a, dtype=float32)[-1]: numpy's cumsum
adds in order, one rounding per term (np.sum does not: it sums pairwise)."""
import numpy as np


def sequential(a: np.ndarray) -> np.float32:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return np.float32(0.0) if a.size == 0 else np.cumsum(a, dtype=np.float32)[-1]


def cases(seed: int = 0):
    """(name, float32 array) pairs."""
    rng = np.random.default_rng(seed)
    out = []
    for n in (1, 31, 33, 256, 2048, 3072, 4096, 8192):
        x = rng.standard_normal(n).astype(np.float32)
        out.append((f"squares_n{n}", x * x))
    for n in (2048, 8192):
        # magnitudes over 40 decades: many binade crossings, tiny terms below a
        # big sum, subnormal squares
        x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-25, 15, n)).astype(np.float32)
        out.append((f"wide_n{n}", x * x))
        # a large first term, then small ones (the sum sits in one binade)
        a = (rng.random(n).astype(np.float32) * np.float32(1e-3))
        a[0] = np.float32(1e6)
        out.append((f"big_first_n{n}", a))
        # growing geometrically: a crossing every few terms (the round limit)
        out.append((f"geometric_n{n}", (np.float32(1.0001) ** np.arange(n)).astype(np.float32)))
    # exact ties: once s is in [1, 2), u = 2^-23 and a term of 2^-24 is half a
    # unit; sums land on both parities
    a = np.full(2048, np.float32(2.0 ** -24))
    a[:40] = np.float32(1.0 / 32)
    out.append(("ties_half_unit", a))
    a = rng.integers(0, 8, 2048).astype(np.float32) * np.float32(2.0 ** -24)
    a[:33] = np.float32(0.05)
    out.append(("ties_mixed", a))
    # three-halves units and odd multiples of half a unit
    a = (rng.integers(0, 64, 2048) * 2 + 1).astype(np.float32) * np.float32(2.0 ** -25)
    a[:32] = np.float32(0.03)
    out.append(("ties_odd_halves", a))
    # a few exact ties among ordinary squares, each planted where the running
    # sum's grid makes the term exactly an odd number of half units
    x = rng.standard_normal(2048).astype(np.float32)
    a = x * x
    for j in (200, 555, 901, 1400, 2000):
        prev = np.cumsum(a[:j], dtype=np.float32)[-1]
        e = int(prev.view(np.uint32)) >> 23
        u = np.float32(2.0 ** (e - 150))
        a[j] = np.float32(int(rng.integers(0, 40)) * 2 + 1) * (u / np.float32(2))
    out.append(("planted_ties", a))
    # zeros: all, leading, and interleaved
    out.append(("zeros", np.zeros(2048, np.float32)))
    a = rng.random(2048).astype(np.float32)
    a[:100] = 0.0
    out.append(("leading_zeros", a))
    a = rng.random(2048).astype(np.float32)
    a[::3] = 0.0
    out.append(("some_zeros", a))
    # subnormal terms only, and subnormal then normal
    a = (rng.random(2048) * 1e-40).astype(np.float32)
    out.append(("subnormal", a))
    a = (rng.random(2048) * 1e-40).astype(np.float32)
    a[1000:] = rng.random(1048).astype(np.float32)
    out.append(("subnormal_then_normal", a))
    # overflow to inf, an inf term, a NaN term
    a = np.full(2048, np.float32(3e37))
    out.append(("to_inf", a))
    a = rng.random(2048).astype(np.float32)
    a[700] = np.inf
    out.append(("inf_term", a))
    a = rng.random(2048).astype(np.float32)
    a[1500] = np.nan
    out.append(("nan_term", a))
    # terms just below and at the binade limit of the running sum
    a = rng.random(2048).astype(np.float32)
    a[500] = np.float32(4096.0)
    a[501] = np.float32(np.nextafter(np.float32(8192.0), np.float32(0)))
    out.append(("near_limit", a))
    return out
