"""The air-side dense solver of k_dense (dense_team: one thread per matrix
row, the matrix in shared memory) against a restatement of the reference's partial-pivot
Gaussian elimination (complete_port/csim/sb_fdm.c:9-38, as the oracle's
gauss_solve in oracle/sbo_sim.c), bit for bit: random systems, systems with
tied magnitudes and zero multipliers, a singular system (the elimination
stops), a NaN off the pivot path, rows scaled over 600 decades (overflowing
and subnormal intermediates), and sizes across the warp boundaries."""
import ctypes

import numpy as np
import pytest


def _gauss_reference(M, b):
    """sb_fdm.c:9-38 in Python floats (IEEE double, no contraction)."""
    k = len(b)
    M = [list(map(float, row)) for row in M]
    b = list(map(float, b))
    for c in range(k):
        piv, best = c, abs(M[c][c])
        for r in range(c + 1, k):
            v = abs(M[r][c])
            if v > best:
                best, piv = v, r
        if best == 0.0:
            return b
        if piv != c:
            for j in range(c, k):
                M[c][j], M[piv][j] = M[piv][j], M[c][j]
            b[c], b[piv] = b[piv], b[c]
        d = M[c][c]
        for r in range(c + 1, k):
            f = M[r][c] / d
            if f == 0.0:
                continue
            for j in range(c, k):
                M[r][j] -= f * M[c][j]
            b[r] -= f * b[c]
    for r in range(k - 1, -1, -1):
        acc = b[r]
        for j in range(r + 1, k):
            acc -= M[r][j] * b[j]
        b[r] = acc / M[r][r]
    return b


def _cases(k, rng):
    out = []
    A = rng.standard_normal((k, k)) + np.eye(k) * 0.5
    out.append((A, rng.standard_normal(k)))
    T = rng.integers(-2, 3, size=(k, k)).astype(np.float64)   # ties and zero multipliers
    T[np.arange(k), np.arange(k)] = rng.choice([-2.0, 2.0], size=k)
    out.append((T, rng.integers(-3, 4, size=k).astype(np.float64)))
    if k >= 3:
        Z = rng.standard_normal((k, k))
        Z[:, k // 2] = 0.0                                         # the elimination stops
        out.append((Z, rng.standard_normal(k)))
        N = rng.standard_normal((k, k)) + np.eye(k) * 4.0
        N[k - 1, 0] = np.nan                                       # never a pivot; propagates
        out.append((N, rng.standard_normal(k)))
        X = (rng.standard_normal((k, k)) + np.eye(k) * 2.0) * (10.0 ** rng.uniform(-300, 300, size=(k, 1)))
        out.append((X, rng.standard_normal(k) * 1e-300))          # rows over 600 decades, subnormal sums
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 2, 5, 31, 32, 33, 64, 81, 83, 84, 100, 128])
def test_dense_solver_matches_reference(built, k):
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    lib.sb_dense_check.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    rng = np.random.default_rng(k)
    cases = _cases(k, rng)
    M = np.ascontiguousarray(np.stack([c[0] for c in cases]))
    b = np.ascontiguousarray(np.stack([c[1] for c in cases]))
    out = np.zeros_like(b)
    assert lib.sb_dense_check(k, len(cases), M.ctypes.data, b.ctypes.data, out.ctypes.data) == 0, \
        lib.sb_last_error()
    for i, (A, rhs) in enumerate(cases):
        ref = np.array(_gauss_reference(A, rhs))
        # NaN positions agree (payload bits differ between CPU and GPU); every
        # other value bit for bit
        nan = np.isnan(ref)
        np.testing.assert_array_equal(np.isnan(out[i]), nan, err_msg=f"case {i}: NaN positions")
        np.testing.assert_array_equal(out[i][~nan].view(np.uint64), ref[~nan].view(np.uint64), err_msg=f"case {i}")


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 5, 33, 81, 128])
def test_tolerant_solver_agrees_to_rounding(built, k):
    """The corrected and folded builds' dense solver (fused multiply-add row
    updates, back substitution in descending column order with one barrier
    per position) against the exact one: the same pivots here, so the
    solutions agree to rounding (1e-12 relative on systems whose condition
    keeps the reordering's effect small); a stopped elimination (singular
    system) returns the right side as eliminated, again to rounding."""
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    lib.sb_dense_check_mode.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int]
    rng = np.random.default_rng(100 + k)
    A = rng.standard_normal((4, k, k)) + np.eye(k) * (2.0 * np.sqrt(k))   # well conditioned
    if k >= 3:
        A[3, :, k // 2] = 0.0                                                 # the elimination stops
    b = rng.standard_normal((4, k))
    A, b = np.ascontiguousarray(A), np.ascontiguousarray(b)
    exact, fast = np.zeros_like(b), np.zeros_like(b)
    assert lib.sb_dense_check_mode(k, 4, A.ctypes.data, b.ctypes.data, exact.ctypes.data, 0) == 0
    assert lib.sb_dense_check_mode(k, 4, A.ctypes.data, b.ctypes.data, fast.ctypes.data, 1) == 0
    scale = np.maximum(np.abs(exact).max(axis=1, keepdims=True), 1e-300)
    assert (np.abs(fast - exact) <= 1e-12 * scale).all()
