"""The allocation-free dense solve (sb_dense_solve_noalloc) against the
allocating one (sb_dense_check), through the C ABI (GPU).

Some callers cannot call cudaMalloc: a host program whose device memory
belongs to another allocator, or code running where allocation is not
allowed. sb_dense_solve_noalloc serves them from one fixed device array. This
test gives it device buffers it did not allocate and checks its solutions
against sb_dense_check's bit for bit (the tolerance every dense-solve test here
uses is zero), on several calls in a row that reuse the array with different
sizes, and checks that a batch beyond the array is refused. The file name
makes pytest collect it last."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_DOUBLES = 1 << 19


def _systems(k, n, seed):
    rng = np.random.default_rng(seed)
    M = rng.standard_normal((n, k, k)) + np.eye(k)[None] * 0.5
    M[::3] = rng.integers(-2, 3, size=M[::3].shape)          # ties and zero multipliers
    M[1::5, :, k // 2] = 0.0                                 # some eliminations stop
    b = rng.standard_normal((n, k))
    return np.ascontiguousarray(M), np.ascontiguousarray(b)


def _check(lib, k, n, M, b):
    out = np.zeros((n, k))
    d = ctypes.POINTER(ctypes.c_double)
    assert lib.sb_dense_check(k, n, M.ctypes.data_as(d), b.ctypes.data_as(d), out.ctypes.data_as(d)) == 0
    return out


def test_noalloc_matches_allocating_solve(built):
    import torch

    from neurips2026_smart_building_challenge_b200 import env_lib

    lib = env_lib()
    lib.sb_dense_solve_noalloc.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p]
    lib.sb_dense_check.argtypes = [ctypes.c_int, ctypes.c_int] + [ctypes.POINTER(ctypes.c_double)] * 3
    # consecutive calls share the array: a large batch, a smaller one, the first again
    for k, n, seed in [(81, 79, 1), (33, 300, 2), (81, 79, 1), (128, 32, 3)]:
        assert n * k * k <= SCRATCH_DOUBLES
        M, b = _systems(k, n, seed)
        ref = _check(lib, k, n, M, b)
        Md = torch.from_numpy(M).cuda()
        bd = torch.from_numpy(b).cuda()
        out = torch.full((n, k), 7.0, dtype=torch.float64, device="cuda")
        torch.cuda.synchronize()
        assert lib.sb_dense_solve_noalloc(k, n, Md.data_ptr(), bd.data_ptr(), out.data_ptr()) == 0, \
            lib.sb_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint64), ref.view(np.uint64)), f"k={k} n={n}"


def test_noalloc_after_a_smaller_check(built):
    """A check with a small k, then a no-alloc solve with a large k: the kernel's
    shared-memory limit set for one entry point must serve the other."""
    import torch

    from neurips2026_smart_building_challenge_b200 import env_lib

    lib = env_lib()
    lib.sb_dense_solve_noalloc.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p]
    lib.sb_dense_check.argtypes = [ctypes.c_int, ctypes.c_int] + [ctypes.POINTER(ctypes.c_double)] * 3
    Ms, bs = _systems(8, 4, 5)
    _check(lib, 8, 4, Ms, bs)
    for k, n, seed in [(81, 40, 6), (128, 16, 7)]:
        M, b = _systems(k, n, seed)
        Md = torch.from_numpy(M).cuda()
        bd = torch.from_numpy(b).cuda()
        out = torch.zeros((n, k), dtype=torch.float64, device="cuda")
        torch.cuda.synchronize()
        assert lib.sb_dense_solve_noalloc(k, n, Md.data_ptr(), bd.data_ptr(), out.data_ptr()) == 0, \
            lib.sb_last_error()
        torch.cuda.synchronize()
        ref = _check(lib, k, n, M, b)
        assert np.array_equal(out.cpu().numpy().view(np.uint64), ref.view(np.uint64)), f"k={k} n={n}"
        _check(lib, 8, 4, Ms, bs)


def test_noalloc_rejects_batches_beyond_its_array(built):
    import torch

    from neurips2026_smart_building_challenge_b200 import env_lib

    lib = env_lib()
    lib.sb_dense_solve_noalloc.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p]
    k = 128
    n = SCRATCH_DOUBLES // (k * k) + 1
    buf = torch.zeros(8, dtype=torch.float64, device="cuda")
    p = buf.data_ptr()
    assert lib.sb_dense_solve_noalloc(k, n, p, p, p) == -1
    assert b"exceeds the fixed scratch" in lib.sb_last_error()
    assert lib.sb_dense_solve_noalloc(129, 1, p, p, p) == -1
