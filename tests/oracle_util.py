"""TEST INFRASTRUCTURE: ctypes access to the CPU oracle libraries (oracle/sbo.h).

PORT = this repository's C restatement (oracle/liboracle.so, always built);
REF  = the reference's own C core behind the same ABI (oracle/_ref/libcsimref.so,
       present only where the reference tree was available at build time).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
PORT = ROOT / "oracle" / "liboracle.so"
REF = ROOT / "oracle" / "_ref" / "libcsimref.so"

_cache: dict[str, ctypes.CDLL] = {}


def lib(path: Path) -> ctypes.CDLL:
    key = str(path)
    if key not in _cache:
        l = ctypes.CDLL(key)
        l.sbo_create.restype = ctypes.c_void_p
        l.sbo_create.argtypes = [ctypes.c_char_p, ctypes.c_int]
        for fn in ["sbo_destroy", "sbo_dims", "sbo_reset", "sbo_step", "sbo_get_temp", "sbo_get_mass",
                   "sbo_step_index", "sbo_reseed", "sbo_visible"]:
            getattr(l, fn).argtypes = None
        l.sbo_set_episode.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_int]
        l.sbo_episode_offset.argtypes = [ctypes.c_void_p]
        _cache[key] = l
    return _cache[key]


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class OracleEnv:
    """One reference-CPU-env instance (reset/step order of complete_port/pufferlib_cpu_env.h)."""

    def __init__(self, blob: str | Path, max_steps: int = 0, path: Path = PORT):
        self.l = lib(path)
        self.h = ctypes.c_void_p(self.l.sbo_create(str(blob).encode(), max_steps))
        if not self.h.value:
            raise RuntimeError(f"oracle could not load {blob}")
        d = (ctypes.c_int * 10)()
        self.l.sbo_dims(self.h, d)
        (self.ncv, self.n, self.k, self.nz, self.nv, self.na, self.nact, self.n_cont, self.n_disc,
         self.obs_len) = list(d)
        self.obs = np.zeros(1024, np.float32)

    def set_episode(self, first_len: int, start_rng: int = 0, random_start: bool = False) -> None:
        """The device env's episode options for this env: first-episode length
        (desync) and random-start stream (oracle/sbo.h sbo_set_episode)."""
        self.l.sbo_set_episode(self.h, int(first_len), int(start_rng), 1 if random_start else 0)

    def episode_offset(self) -> int:
        return int(self.l.sbo_episode_offset(self.h))

    def reset(self) -> np.ndarray:
        self.l.sbo_reset(self.h, _p(self.obs))
        return self.obs.copy()

    def step(self, act: np.ndarray):
        act = np.ascontiguousarray(act, dtype=np.float32)
        r, t, rd = ctypes.c_float(), ctypes.c_float(), ctypes.c_double()
        parts, log8 = np.zeros(12), np.zeros(8)
        self.l.sbo_step(self.h, _p(act), _p(self.obs), ctypes.byref(r), ctypes.byref(t), ctypes.byref(rd),
                        _p(parts), _p(log8))
        return self.obs.copy(), r.value, t.value, rd.value, parts, log8

    def temp(self) -> np.ndarray:
        out = np.zeros(self.ncv)
        self.l.sbo_get_temp(self.h, _p(out))
        return out

    def mass(self) -> np.ndarray:
        out = np.zeros(self.n)
        self.l.sbo_get_mass(self.h, _p(out))
        return out

    def visible(self) -> np.ndarray:
        """Snapshot fields after the last step (oracle/sbo_env.c sbo_visible)."""
        out = np.zeros(self.ncv + 4 * self.nz + 4 * self.nv + 3 * self.na + self.nact + 3)
        self.l.sbo_visible.restype = ctypes.c_int
        if self.l.sbo_visible(self.h, _p(out)) != len(out):
            raise RuntimeError("this oracle build does not export the visible state")
        return out

    def close(self):
        if self.h.value:
            self.l.sbo_destroy(self.h)
            self.h = ctypes.c_void_p(0)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def actions(rng: np.random.Generator, n_env: int, n_cont: int, n_disc: int, wild: bool = True,
            alpha=None, beta=None) -> np.ndarray:
    """Seeded action batch: continuous heads 2x-1 with x ~ Beta(alpha, beta) (the
    trainer's Beta-head contract, complete_port/patches/pufferlib_core.diff:2556),
    a few out-of-range values to exercise the clamp, discrete run bits mostly on."""
    a = np.zeros((n_env, 272), np.float32)
    al = 2.0 if alpha is None else alpha
    be = 2.0 if beta is None else beta
    a[:, :n_cont] = 2.0 * rng.beta(al, be, size=(n_env, n_cont)) - 1.0
    if wild:
        m = rng.random((n_env, n_cont)) < 0.02
        a[:, :n_cont][m] = 3.0 * rng.standard_normal(m.sum())
    a[:, 256:256 + n_disc] = (rng.random((n_env, n_disc)) < 0.9).astype(np.float32)
    return a
