"""Generates the golden fixtures in this directory (run where the reference tree exists).

ref_small.npz: the reference's own C core (complete_port/csim, compiled unmodified
into oracle/_ref/libcsimref.so by oracle/Makefile) stepping one small synthetic
scenario for 90 steps with seeded actions: reset observation, every step's
observation / reward (f32 and f64) / terminal / 12 reward diagnostics, and the
temperature field and interior mass at a few steps. The blob's sha256 is stored
too, so a generator change that would silently move the fixture is caught.

ref_month.npz: the same compiled reference core stepping BASELINE configuration 1
(one 64x48 / 41-zone building, Monday 16 January 00:00 onward) for its whole
8,640-step month plus 24 steps after the in-step restart, with Beta(2,2) actions
drawn with seed 0: a 64-bit BLAKE2b digest of every step's observation, every
step's reward (f32 and f64) and terminal, a digest of the temperature field and
interior mass every simulated hour, and the full field and mass at the end. The
month crosses four weekends, the January-February roll of the gas price and
every occupancy arrival and departure window.

mt19937.npz: numpy's legacy RandomState stream (random_sample, randint) for a few
seeds -- the stream the reference's occupancy and convection draw from.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE.parent))

SMALL = dict(notch_rows=3, notch_cols=4, n_steps=40, start_hour=7, conv_p=0.5)
STEPS = 90
TEMP_AT = (0, 39, 40, 89)


def small_blob(path: Path) -> Path:
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    return write_scenario(path, preset(1, 0, **SMALL))


MONTH_STEPS = 8640 + 24
MONTH_HOUR = 12


def digest(a: np.ndarray) -> np.uint64:
    return np.frombuffer(hashlib.blake2b(np.ascontiguousarray(a).tobytes(), digest_size=8).digest(), np.uint64)[0]


def month_blob(path: Path) -> Path:
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    return write_scenario(path, preset(1, 0))


def month_actions(n_cont: int, n_disc: int):
    """Configuration 1's action stream: every continuous head 2x - 1 with
    x ~ Beta(2, 2), seed 0; run bits on. One batch per step (a generator)."""
    rng = np.random.default_rng(0)
    for _ in range(MONTH_STEPS):
        a = np.zeros(272, np.float32)
        a[:n_cont] = 2.0 * rng.beta(2.0, 2.0, size=n_cont) - 1.0
        a[256:256 + n_disc] = 1.0
        yield a


def record_month(env) -> dict:
    """Steps an oracle env through the month; returns the fixture's arrays."""
    obs_d, r32, r64, term, t_d, m_d = [digest(env.reset())], [], [], [], [], []
    for s, a in enumerate(month_actions(env.n_cont, env.n_disc)):
        o, r, t, rd, _, _ = env.step(a)
        obs_d.append(digest(o))
        r32.append(r)
        r64.append(rd)
        term.append(t)
        if s % MONTH_HOUR == MONTH_HOUR - 1:
            t_d.append(digest(env.temp()))
            m_d.append(digest(env.mass()))
    return dict(obs_digest=np.array(obs_d, np.uint64), rew32=np.array(r32, np.float32), rew64=np.array(r64),
                term=np.array(term, np.float32), temp_digest=np.array(t_d, np.uint64),
                mass_digest=np.array(m_d, np.uint64), temp_end=env.temp(), mass_end=env.mass())


def action_stream(n_cont: int, n_disc: int) -> np.ndarray:
    from oracle_util import actions

    rng = np.random.default_rng(20261201)
    return np.stack([actions(rng, 1, n_cont, n_disc)[0] for _ in range(STEPS)])


def main() -> None:
    from neurips2026_smart_building_challenge_b200 import build
    from oracle_util import REF, OracleEnv

    build.build_all()
    if not REF.exists():
        raise SystemExit("oracle/_ref/libcsimref.so is missing: the reference tree is needed")
    tmp = HERE / "_small.sbb"
    small_blob(tmp)
    sha = hashlib.sha256(tmp.read_bytes()).hexdigest()
    env = OracleEnv(tmp, path=REF)
    acts = action_stream(env.n_cont, env.n_disc)
    L = env.obs_len
    obs = [env.reset()[:L]]
    rew32, rew64, term, parts, temps, mass = [], [], [], [], [], []
    for s in range(STEPS):
        o, r, t, rd, p12, _ = env.step(acts[s])
        obs.append(o[:L])
        rew32.append(r)
        rew64.append(rd)
        term.append(t)
        parts.append(p12)
        if s in TEMP_AT:
            temps.append(env.temp())
            mass.append(env.mass())
    np.savez_compressed(HERE / "ref_small.npz", sha256=np.array(sha), obs=np.array(obs, np.float32),
                        rew32=np.array(rew32, np.float32), rew64=np.array(rew64), term=np.array(term, np.float32),
                        parts=np.array(parts), temp=np.array(temps), mass=np.array(mass),
                        temp_at=np.array(TEMP_AT), actions=acts)
    tmp.unlink()
    mb = month_blob(HERE / "_month.sbb")
    month = record_month(OracleEnv(mb, path=REF))
    np.savez_compressed(HERE / "ref_month.npz", sha256=np.array(hashlib.sha256(mb.read_bytes()).hexdigest()),
                        **month)
    mb.unlink()
    mt = {}
    for seed in (0, 5, 17321, 4294967295):
        rs = np.random.RandomState(seed)
        mt[f"sample_{seed}"] = rs.random_sample(2000)
        mt[f"randint_{seed}"] = np.array([rs.randint(0, hi + 1) for hi in (0, 1, 5, 7, 8, 100, 1023, 1 << 20)
                                          for _ in range(50)], dtype=np.int64)
    np.savez_compressed(HERE / "mt19937.npz", **mt)
    print("golden fixtures written:", sha)


if __name__ == "__main__":
    main()
