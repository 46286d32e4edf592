"""Generates the golden fixtures in this directory (run where the reference tree exists).

ref_small.npz: the reference's own C core (complete_port/csim, compiled unmodified
into oracle/_ref/libcsimref.so by oracle/Makefile) stepping one small synthetic
scenario for 90 steps with seeded actions: reset observation, every step's
observation / reward (f32 and f64) / terminal / 12 reward diagnostics, and the
temperature field and interior mass at a few steps. The blob's sha256 is stored
too, so a generator change that would silently move the fixture is caught.

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
