"""TEST INFRASTRUCTURE: a CPU model of the solve kernel's per-warp stage ring
(StageRing and the record cursor of run_sweep / run_block in
csrc/k_solve.cuh). It walks a warp program the way the kernel does and checks
the ring protocol: a stage is read only after it has landed and while its
slot holds it, a slot is refilled only after its previous copy has landed,
and every wait is on a stage that was issued."""
import struct

REC, STAGE = 160, 1440   # nine records per ring stage (csrc/sbenv_dev.h)
C_NEXT, C_END, C_BLOCK = 1, 2, 4
NEXT_CTRL = 0x8000


def walk(stream, R):
    nst = len(stream) // STAGE
    assert nst > 0
    slot_stage = [-1] * R
    st = {"head": 0, "landed": 0}
    for s in range(min(R, nst)):
        slot_stage[s] = s

    def land(t):
        assert t < min(st["head"] + R, nst), f"wait on stage {t} that was not issued"
        while st["landed"] <= t:
            assert slot_stage[st["landed"] % R] == st["landed"]
            st["landed"] += 1

    def consume(t):
        if st["head"] >= t:
            return
        assert t <= st["head"] + R, "consume beyond the ring"
        land(t - 1)
        while st["head"] < t:
            h = st["head"]
            assert st["landed"] > h, "slot refilled before its copy landed"
            if h + R < nst:
                slot_stage[h % R] = h + R
            st["head"] += 1

    def read(off, nbytes):
        for b in (off, off + nbytes - 1):
            s = b // STAGE
            assert st["head"] <= s < st["landed"] and slot_stage[s % R] == s, f"read of stage {s} not in the ring"

    land(0)
    rec, ctrl = 0, True
    while True:
        off = rec * REC
        read(off, REC)
        if not ctrl:
            ctrl = bool(struct.unpack_from("<H", stream, off + 128)[0] & NEXT_CTRL)
        else:
            flags = stream[off + 13]
            if flags & C_BLOCK:   # its values are read from the value region, not the ring
                assert flags & C_NEXT
                ctrl = True
                rec += 1
                if rec % (STAGE // REC) == 0:
                    consume(st["head"] + 1)
                    assert st["head"] < nst
                    land(st["head"])
                continue
            if flags & C_END:
                break
            ctrl = bool(flags & C_NEXT)
        rec += 1
        if rec % (STAGE // REC) == 0:
            consume(st["head"] + 1)
            assert st["head"] < nst
            land(st["head"])
    # in-flight copies at the end
    end = min(st["head"] + R, nst)
    land(end - 1)
    return rec
