"""The device solve schedule (host-built, streamed chunk by chunk into shared
memory) replayed on the CPU: executing it with the kernel's semantics -- every
task of a chunk reads the vector as it was when the chunk started -- must give
bit for bit the reference's column-push replay (complete_port/csim/sb_lu.c:38-63)."""
import ctypes
import struct

import numpy as np
import pytest

from sbb_read import Blob


def _schedule(lib, blob, sweep):
    used = ctypes.c_size_t()
    nch = ctypes.c_uint32()
    lib.sb_solve_schedule.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_uint32)]
    assert lib.sb_solve_schedule(str(blob).encode(), sweep, None, 0, ctypes.byref(used), ctypes.byref(nch)) == 1
    buf = (ctypes.c_uint8 * used.value)()
    assert lib.sb_solve_schedule(str(blob).encode(), sweep, buf, used.value, ctypes.byref(used),
                                 ctypes.byref(nch)) == 0
    return bytes(buf), nch.value


def _chunks(raw, nch):
    pos, out, sizes = 0, [], []
    for _ in range(nch):
        ntask, nval, nxt, check = struct.unpack_from("<4I", raw, pos)
        assert check == (ntask ^ (nval << 12) ^ 0x5B5B0000) & 0xFFFFFFFF
        size = (16 + 8 * ntask + 10 * nval + 15) & ~15
        assert size <= 4096
        tasks = np.frombuffer(raw, dtype=np.dtype([("row", "<u2"), ("lo", "u1"), ("hi", "u1"), ("off", "<u4")]),
                              count=ntask, offset=pos + 16)
        vals = np.frombuffer(raw, dtype="<f8", count=nval, offset=pos + 16 + 8 * ntask)
        cols = np.frombuffer(raw, dtype="<u2", count=nval, offset=pos + 16 + 8 * ntask + 8 * nval)
        out.append((tasks, vals, cols, nxt))
        sizes.append(size)
        pos += size
    assert pos == len(raw)
    for c, (_, _, _, nxt) in enumerate(out):   # next_bytes = size of the chunk six later
        assert nxt == (sizes[c + 6] if c + 6 < nch else 0)
    return out


def _run(chunks, x, backward, n):
    x = x.copy()
    final = np.zeros(n, bool)
    if not backward:
        final[:] = True   # rows without L terms are final from the start; corrected below
        has = np.zeros(n, bool)
        for tasks, _, _, _ in chunks:
            has[tasks["row"]] = True
        final[has] = False
    for tasks, vals, cols, _ in chunks:
        snap = x.copy()
        newv = {}
        rows = [int(r) for r in tasks["row"]]
        assert len(set(rows)) == len(rows), "a row appears twice in one chunk"
        for t in tasks:
            row, nt = int(t["row"]), int(t["lo"]) | ((int(t["hi"]) & 0x0F) << 8)
            off, fin = int(t["off"]), bool(t["hi"] & 0x80)
            acc = snap[row]
            for q in range(nt):
                c = int(cols[off + q])
                assert final[c], "a term reads a row that is not final yet"
                acc = acc - vals[off + q] * snap[c]
            if fin:
                acc = acc / vals[off + nt]
            newv[row] = (acc, fin or not backward)
        for row, (v, f) in newv.items():
            x[row] = v
        # forward rows become final after their last task; track via remaining terms
        for t in tasks:
            row = int(t["row"])
            if backward and (t["hi"] & 0x80):
                final[row] = True
        if not backward:
            for row in newv:
                final[row] = _fwd_done(row)
    return x


_FWD_LEFT = {}


def _fwd_done(row):
    _FWD_LEFT[row] -= 1
    return _FWD_LEFT[row] == 0


def _push_reference(L, U, b):
    n = len(b)
    w = b.copy().tolist()
    Lc = L.tocsc()
    for j in range(n):
        yj = w[j]
        for p in range(Lc.indptr[j], Lc.indptr[j + 1]):
            i = Lc.indices[p]
            if i != j:
                w[i] = w[i] - Lc.data[p] * yj
    Uc = U.tocsc()
    diag = Uc.diagonal()
    for j in range(n - 1, -1, -1):
        zj = w[j] / diag[j]
        w[j] = zj
        for p in range(Uc.indptr[j], Uc.indptr[j + 1]):
            i = Uc.indices[p]
            if i != j:
                w[i] = w[i] - Uc.data[p] * zj
    return np.array(w)


@pytest.mark.parametrize("config,index", [(1, 0), (2, 23)])
def test_schedule_replays_reference_solve(built, tmp_path, config, index):
    import neurips2026_smart_building_challenge_b200 as pkg

    blob = pkg.write_scenario(tmp_path / "s.sbb", pkg.preset(config, index, n_steps=10))
    b = Blob(blob)
    L, U = b.csc("lu_L"), b.csc("lu_U")
    n = L.shape[0]
    lib = pkg.env_lib()
    fwd = _chunks(*_schedule(lib, blob, 0))
    bwd = _chunks(*_schedule(lib, blob, 1))
    # number of forward tasks per row (a row is final after its last one)
    _FWD_LEFT.clear()
    for tasks, _, _, _ in fwd:
        for r in tasks["row"]:
            _FWD_LEFT[int(r)] = _FWD_LEFT.get(int(r), 0) + 1
    rng = np.random.default_rng(index)
    rhs = rng.standard_normal(n) * 300.0
    y = _run(fwd, rhs, False, n)
    z = _run(bwd, y, True, n)
    ref = _push_reference(L, U, rhs)
    assert np.array_equal(z, ref)
    # every off-diagonal term appears exactly once
    assert sum(len(c[2]) for c in fwd) == L.nnz - n
    assert sum(len(c[2]) for c in bwd) == U.nnz   # terms + one diagonal per row
