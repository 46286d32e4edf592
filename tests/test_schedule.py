"""The solve kernel's sweep programs (built on the host by csrc/sweep_sched.cpp),
executed on the CPU with the kernel's semantics under several interleavings of
the 16 warps. Every row must receive exactly the reference's terms in the
reference's order (the column push of complete_port/csim/sb_lu.c:38-63), no
bundle may read a row that is not final yet (a bundle starts only when the
rows it waits for are published), no interleaving may deadlock, and the solve
must equal the column-push replay bit for bit."""
import ctypes
import struct

import numpy as np
import pytest

from sbb_read import Blob

NW, STAGE, MAX_BUNDLE = 16, 512, 960
END, SKIP, FIN_NEVER = 0x8000, 0x4000, 0xFF


def _programs(lib, blob, sweep, ring_stages):
    used = ctypes.c_size_t()
    stages = (ctypes.c_uint32 * NW)()
    lib.sb_solve_schedule.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_uint32)]
    b = str(blob).encode()
    assert lib.sb_solve_schedule(b, sweep, ring_stages, None, 0, ctypes.byref(used), stages) == 1
    buf = (ctypes.c_uint8 * used.value)()
    assert lib.sb_solve_schedule(b, sweep, ring_stages, buf, used.value, ctypes.byref(used), stages) == 0
    raw, out, pos = bytes(buf), [], 0
    for w in range(NW):
        size = stages[w] * STAGE
        out.append(raw[pos:pos + size])
        pos += size
    assert pos == len(raw)
    return out


def _parse(stream, n, backward, ring_stages):
    """Bundles of one warp stream. A bundle never wraps around the warp's ring
    (ring_stages x 512 bytes): a skip header moves the stream to the ring's
    start (zero bytes)."""
    RING = ring_stages * STAGE
    pos, bundles = 0, []
    while True:
        hdr = stream[pos:pos + 16]
        assert len(hdr) == 16, "stream ends without an end marker"
        rows = struct.unpack_from("<4H", hdr)
        nblk, flags = struct.unpack_from("<HH", hdr, 8)
        fin = list(hdr[12:16])
        if flags & END:
            pos += 16
            break
        if flags & SKIP:
            ro = pos % RING
            assert not any(stream[pos + 16:pos + RING - ro])
            pos += RING - ro
            continue
        assert flags & 0x3000 == 0
        assert all(r <= n for r in rows)
        assert all(f == FIN_NEVER or f <= nblk for f in fin)
        npre = (flags >> 8) & 0xF
        size = 16 + 16 * npre + (32 if flags & 0xF0 else 0) + 160 * nblk
        assert size <= MAX_BUNDLE and pos % RING + size <= RING, "bundle too large or wraps the ring"
        off = pos + 16
        pre = list(struct.unpack_from(f"<{8 * npre}H", stream, off)) if npre else []
        off += 16 * npre
        diag = [1.0] * 4
        if flags & 0xF0:
            diag = list(struct.unpack_from("<4d", stream, off))
            off += 32
        assert bool(flags & 0xF0) == (backward and any(f != FIN_NEVER for f in fin))
        blocks = []
        for _ in range(nblk):
            vals = np.frombuffer(stream, "<f8", 16, off).reshape(4, 4)
            cols = np.frombuffer(stream, "<u2", 16, off + 128).reshape(4, 4)
            blocks.append((vals, cols))
            off += 160
        bundles.append(dict(rows=rows, flags=flags, fin=fin, pre=pre, diag=diag, blocks=blocks))
        pos = off
    assert not any(stream[pos:]), "bytes after the end marker"
    assert len(stream) % STAGE == 0
    return bundles


class _Warp:
    def __init__(self, bundles):
        self.bundles, self.bi, self.b, self.acc, self.done = bundles, 0, -1, [0.0] * 4, [False] * 4

    def finished(self):
        return self.bi >= len(self.bundles)


def _execute(programs, x, n, backward, pick, expect, ring_stages):
    """Runs the warps' bundles block by block in the order pick() chooses."""
    x = list(x) + [0.0]
    final = [False] * (n + 1)
    final[n] = True
    if not backward:
        for i in range(n):
            final[i] = not expect[i]
    ready = [False] * n + [True]
    got = [[] for _ in range(n)]
    warps = [_Warp(_parse(p, n, backward, ring_stages)) for p in programs]

    def finish(wp, B, g):
        r = B["rows"][g]
        acc = wp.acc[g]
        if (B["flags"] >> (4 + g)) & 1:
            acc = acc / B["diag"][g]
        x[r], wp.acc[g], wp.done[g] = acc, acc, True
        final[r] = True
        if (B["flags"] >> g) & 1:
            ready[r] = True

    def step(wp):
        """One unit of warp wp; False if it is blocked."""
        B = wp.bundles[wp.bi]
        if wp.b < 0:   # bundle start: pre-waits, accumulators
            if not all(ready[r] for r in B["pre"]):
                return False
            for g in range(4):
                wp.acc[g], wp.done[g] = x[B["rows"][g]], False
                if B["fin"][g] == 0:
                    finish(wp, B, g)
            wp.b = 0
        elif wp.b < len(B["blocks"]):
            vals, cols = B["blocks"][wp.b]
            for g in range(4):
                r = B["rows"][g]
                for s in range(4):
                    c, v = int(cols[g, s]), float(vals[g, s])
                    assert final[c], f"row {r} reads row {c} before it is final"
                    wp.acc[g] = wp.acc[g] - v * x[c]
                    if c != n:
                        got[r].append((c, v))
                    else:
                        assert v == 0.0
                if B["fin"][g] == wp.b + 1:
                    finish(wp, B, g)
            wp.b += 1
        else:          # bundle end
            for g in range(4):
                if not wp.done[g]:
                    x[B["rows"][g]] = wp.acc[g]
            wp.bi, wp.b = wp.bi + 1, -1
        return True

    while True:
        live = [w for w in warps if not w.finished()]
        if not live:
            break
        order = pick(live)
        assert any(step(w) for w in order), "deadlock: every unfinished warp waits"
    for i in range(n):
        assert got[i] == expect[i], f"row {i}: terms differ from the reference's push order"
        assert final[i]
    return np.array(x[:n])


def _terms(M, backward):
    """(column, value) per row in the order the reference's column push delivers them."""
    Mc = M.tocsc()
    n = Mc.shape[0]
    out = [[] for _ in range(n)]
    cols = range(n - 1, -1, -1) if backward else range(n)
    for j in cols:
        for p in range(Mc.indptr[j], Mc.indptr[j + 1]):
            i = int(Mc.indices[p])
            if i != j:
                out[i].append((j, float(Mc.data[p])))
    return out


def _push_reference(L, U, b):
    n = len(b)
    w = b.copy().tolist()
    Lc, Uc = L.tocsc(), U.tocsc()
    for j in range(n):
        yj = w[j]
        for p in range(Lc.indptr[j], Lc.indptr[j + 1]):
            i = Lc.indices[p]
            if i != j:
                w[i] = w[i] - Lc.data[p] * yj
    diag = Uc.diagonal()
    for j in range(n - 1, -1, -1):
        zj = w[j] / diag[j]
        w[j] = zj
        for p in range(Uc.indptr[j], Uc.indptr[j + 1]):
            i = Uc.indices[p]
            if i != j:
                w[i] = w[i] - Uc.data[p] * zj
    return np.array(w)


def _pickers(seed):
    rng = np.random.default_rng(seed)

    def shuffled(live):
        return [live[k] for k in rng.permutation(len(live))]

    def greedy(live):      # one warp as far as it goes: reads race ahead of producers
        return live

    def laggard(live):     # the warp with the least progress first
        return sorted(live, key=lambda w: (w.bi, w.b))

    return [shuffled, greedy, laggard]


@pytest.mark.parametrize("config,index,ring", [(1, 0, 4), (2, 23, 6), (2, 5, 8)])
def test_schedule_replays_reference_solve(built, tmp_path, config, index, ring):
    import neurips2026_smart_building_challenge_b200 as pkg

    blob = pkg.write_scenario(tmp_path / "s.sbb", pkg.preset(config, index, n_steps=10))
    b = Blob(blob)
    L, U = b.csc("lu_L"), b.csc("lu_U")
    n = L.shape[0]
    lib = pkg.env_lib()
    fwd, bwd = _programs(lib, blob, 0, ring), _programs(lib, blob, 1, ring)
    tl, tu = _terms(L, False), _terms(U, True)
    rhs = np.random.default_rng(index).standard_normal(n) * 300.0
    ref = _push_reference(L, U, rhs)
    for k, pick in enumerate(_pickers(index)):
        y = _execute(fwd, rhs, n, False, pick, tl, ring)
        z = _execute(bwd, y, n, True, pick, tu, ring)
        assert np.array_equal(z, ref), f"interleaving {k}"


def test_schedule_stats(built, tmp_path):
    """The statistics export agrees with the streams; bad arguments are errors."""
    import neurips2026_smart_building_challenge_b200 as pkg

    blob = pkg.write_scenario(tmp_path / "s.sbb", pkg.preset(1, 0, n_steps=10))
    lib = pkg.env_lib()
    lib.sb_sweep_stats.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
    L = Blob(blob).csc("lu_L")
    n = L.shape[0]
    st = (ctypes.c_double * 8)()
    for sweep in (0, 1):
        assert lib.sb_sweep_stats(str(blob).encode(), sweep, 5, st) == 0
        progs = _programs(lib, blob, sweep, 5)
        bundles = [B for p in progs for B in _parse(p, n, sweep == 1, 5)]
        assert st[0] == L.nnz - n
        assert st[1] == len(bundles)
        assert st[2] == sum(len(B["blocks"]) for B in bundles)
        assert st[3] == sum(int(r != n) for B in bundles for r in B["rows"])
        assert st[4] <= sum(len(B["pre"]) for B in bundles)
        assert st[7] == sum(len(p) for p in progs)
    assert lib.sb_sweep_stats(str(blob).encode(), 0, 0, st) == 0          # default depth
    assert lib.sb_sweep_stats(str(blob).encode(), 2, 5, st) == -1         # no such sweep
    assert lib.sb_sweep_stats(str(blob).encode(), 0, 3, st) == -1         # ring too shallow
    assert b"ring" in lib.sb_last_error()
