"""TEST INFRASTRUCTURE: minimal SBB1 reader (format: 52-byte header, 56-byte
directory entries; see neurips2026_smart_building_challenge_b200/csrc/sbb.h)."""
from __future__ import annotations

import struct

import numpy as np

_DT = {0: np.float64, 1: np.float32, 2: np.int64, 3: np.int32, 4: np.int8, 5: np.uint8, 6: np.uint32, 7: np.uint8}


class Blob:
    def __init__(self, path):
        self.raw = open(path, "rb").read()
        magic, ver, nsec, dir_off, names_off, names_len, total, _ = struct.unpack_from("<4sII5Q", self.raw, 0)
        assert magic == b"SBB1" and ver == 1
        self.sec = {}
        for i in range(nsec):
            name_off, dt, ndim, _r, s0, s1, s2, s3, off = struct.unpack_from("<IIII5Q", self.raw, dir_off + 56 * i)
            end = self.raw.index(b"\0", names_off + name_off)
            name = self.raw[names_off + name_off:end].decode()
            shape = (s0, s1, s2, s3)[:ndim]
            self.sec[name] = (dt, shape, off)

    def __contains__(self, name):
        return name in self.sec

    def get(self, name):
        dt, shape, off = self.sec[name]
        n = int(np.prod(shape)) if shape else 1
        return np.frombuffer(self.raw, dtype=_DT[dt], count=n, offset=off).reshape(shape)

    def csc(self, prefix):
        import scipy.sparse as sp

        shape = tuple(int(x) for x in self.get(prefix + "_shape"))
        return sp.csc_matrix((self.get(prefix + "_data"), self.get(prefix + "_indices"), self.get(prefix + "_indptr")),
                             shape=shape)
