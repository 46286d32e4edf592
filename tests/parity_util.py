"""TEST INFRASTRUCTURE: the device env stepped beside CPU oracle envs, compared
after every step (observations as f32 bit patterns, rewards as f32 and f64,
terminals, the 8 log terms; the temperature field and interior mass every
`temp_every` steps). Used by the GPU parity tests.

The oracle is the reference's own C core (oracle/_ref/libcsimref.so) when
`oracle` is "reference" and that library exists, else this repository's
restatement (oracle/liboracle.so, pinned to the reference by
tests/test_oracle.py). The reference core cannot form the gas term of the log
(it is internal to its reward), so against it that term is not compared.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle_util import PORT, REF, OracleEnv, actions


def oracle_path(kind: str = "port") -> Path:
    return REF if kind == "reference" and REF.exists() else PORT


def vec(n, blob_dir, **kw):
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec

    return SmartBuildingsVec(n, blob_dir=str(blob_dir), **kw)


def scenario_paths(blob_dir: Path) -> list[Path]:
    """Scenario index -> blob path, in the env's own building-first round-robin order."""
    names = sorted(p.name for p in Path(blob_dir).glob("*.sbb"))
    blds, keys = [], []
    for nm in names:
        b = nm.split("__")[0]
        keys.append(b)
        if b not in blds:
            blds.append(b)
    used = [False] * len(names)
    order = []
    while len(order) < len(names):
        for b in blds:
            for i, nm in enumerate(names):
                if not used[i] and keys[i] == b:
                    order.append(Path(blob_dir) / nm)
                    used[i] = True
                    break
    return order


def pre_stage_diff(env, orc, e):
    """Which pre-stage quantity differs (air conductances, supply temperatures,
    per-zone cell heat, boiler/pump scalars) -- localises a field mismatch."""
    import ctypes

    g, o = np.zeros(1024), np.zeros(1024)
    ng = env.lib.sb_debug_state(e, g.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), 1024)
    orc.l.sbo_debug.restype = ctypes.c_int
    no = orc.l.sbo_debug(orc.h, o.ctypes.data_as(ctypes.c_void_p))
    if ng != no or ng < 0:
        return f"pre-stage export sizes {ng} vs {no}"
    k, nz = orc.k, orc.nz
    out = []
    for name, a, b in [("air_g", 0, k), ("air_T", k, 2 * k), ("zone q", 2 * k, 2 * k + nz),
                       ("scalars", 2 * k + nz, 2 * k + nz + 5)]:
        d = np.nonzero(g[a:b] != o[a:b])[0]
        if len(d):
            out.append(f"{name} differs at {d[:6].tolist()}: {g[a:b][d[:3]].tolist()} vs {o[a:b][d[:3]].tolist()}")
    return "pre-stage: " + ("; ".join(out) if out else "identical")


# Tolerances of the folded build (solve_exact = 0), the north star's contract:
# temperatures within 1e-9 relative (the field and interior mass, every check),
# rewards within 1e-9 relative, observations equal up to the float32 rounding of
# a value that moved by that much (1e-4 of the field's scale).
TOL_FIELD = 1e-9
TOL_REWARD = 1e-9
TOL_OBS = 1e-4


def run_parity(blob_dir, n, steps, max_steps=0, seed=0, temp_every=10, groups=0, beta_mix=False,
               oracle="port", wild=True, env_kw=None, tolerant=False, on_step=None):
    """Steps n device envs and n oracle envs with the same seeded actions and
    compares them bit for bit after every step (tolerant: within the folded
    build's tolerances above; the largest differences seen are returned).
    With the episode options desync / random_start in env_kw, each oracle env
    gets the device env's first-episode length and random-start stream. on_step
    (if given) is called as on_step(step, env, oracles) after the comparisons."""
    import torch

    from neurips2026_smart_building_challenge_b200 import SB_NUM_ATNS

    env = vec(n, blob_dir, max_steps=max_steps, groups=groups, **(env_kw or {}))
    path = oracle_path(oracle)
    against_ref = path == REF
    worst = {"field_rel": 0.0, "field_abs_K": 0.0, "reward_rel": 0.0, "obs_abs": 0.0, "obs_fields_differing": 0}
    try:
        paths = scenario_paths(blob_dir)
        orc = [OracleEnv(paths[int(env.scenario[e])], max_steps=max_steps, path=path) for e in range(n)]
        kw = env_kw or {}
        if kw.get("desync") or kw.get("random_start"):
            fl, sr = env.episode_options()
            for e in range(n):
                orc[e].set_episode(int(fl[e]), int(sr[e]), bool(kw.get("random_start")))
        env.reset()
        env.synchronize()
        obs = env.obs.cpu().numpy()
        for e in range(n):
            o = orc[e].reset()
            np.testing.assert_array_equal(obs[e].view(np.uint32), o.view(np.uint32), err_msg=f"reset obs env {e}")
        rng = np.random.default_rng(seed)
        if beta_mix:
            al = rng.uniform(0.5, 12.0, size=(n, 256))
            be = rng.uniform(0.5, 12.0, size=(n, 256))
        for s in range(steps):
            a = np.zeros((n, SB_NUM_ATNS), np.float32)
            for e in range(n):
                bkw = dict(alpha=al[e, :orc[e].n_cont], beta=be[e, :orc[e].n_cont]) if beta_mix else {}
                a[e] = actions(rng, 1, orc[e].n_cont, orc[e].n_disc, wild=wild, **bkw)[0]
            env.step(torch.from_numpy(a).to(env.device))
            env.synchronize()
            obs = env.obs.cpu().numpy()
            rew = env.rewards.cpu().numpy()
            term = env.terminals.cpu().numpy()
            rd, parts = env.reward_f64()
            for e in range(n):
                o, r, t, r64, p12, log8 = orc[e].step(a[e])
                where = f"step {s} env {e} scenario {int(env.scenario[e])}"
                bad = []
                if term[e] != t:
                    bad.append("terminal")
                cmp = slice(0, 7) if against_ref else slice(0, 8)
                if tolerant:
                    do = np.abs(obs[e].astype(np.float64) - o.astype(np.float64))
                    worst["obs_abs"] = max(worst["obs_abs"], float(do.max()))
                    worst["obs_fields_differing"] += int(np.count_nonzero(do))
                    if (do > TOL_OBS * np.maximum(1.0, np.abs(o))).any():
                        bad.append(f"obs fields {np.nonzero(do > TOL_OBS)[0][:8].tolist()} differ by {do.max():.3e}")
                    rel = abs(rd[e] - r64) / max(abs(r64), 1e-2)
                    worst["reward_rel"] = max(worst["reward_rel"], rel)
                    if rel > TOL_REWARD:
                        bad.append(f"reward {rd[e]!r} vs {r64!r}")
                    pr = np.abs(parts[e][cmp] - log8[cmp]) / np.maximum(np.abs(log8[cmp]), 1e-2)
                    if (pr > TOL_REWARD).any():
                        bad.append(f"log terms {np.nonzero(pr > TOL_REWARD)[0].tolist()}")
                else:
                    if not np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)):
                        bad.append(f"obs fields {np.nonzero(obs[e] != o)[0][:8].tolist()}")
                    if rew[e] != np.float32(r) or rd[e] != r64:
                        bad.append(f"reward {rd[e]!r} vs {r64!r}")
                    if not np.array_equal(parts[e][cmp], log8[cmp]):
                        bad.append(f"log terms {np.nonzero(parts[e][cmp] != log8[cmp])[0].tolist()}")
                if bad or s % temp_every == 0 or s == steps - 1:
                    To, Mo = orc[e].temp(), orc[e].mass()
                    dT = env.temp(e, orc[e].ncv) - To
                    dM = env.mass(e, orc[e].n) - Mo
                    if tolerant:
                        scale = max(np.abs(To).max(), np.abs(Mo).max())
                        worst["field_abs_K"] = max(worst["field_abs_K"], float(np.abs(dT).max()), float(np.abs(dM).max()))
                        worst["field_rel"] = max(worst["field_rel"], worst["field_abs_K"] / scale)
                        if np.abs(dT).max() > TOL_FIELD * scale or np.abs(dM).max() > TOL_FIELD * scale:
                            bad.append(f"field differs by {np.abs(dT).max():.3e} K, mass by {np.abs(dM).max():.3e} K")
                    else:
                        if dT.any():
                            bad.append(f"T differs at {np.count_nonzero(dT)} cells, max {np.abs(dT).max():.3e}")
                        if dM.any():
                            bad.append(f"M differs at {np.count_nonzero(dM)} cells, max {np.abs(dM).max():.3e}")
                if bad and not against_ref and not tolerant:
                    bad.append(pre_stage_diff(env, orc[e], e))
                assert not bad, f"{where} ({path.name}): " + "; ".join(bad)
            if on_step is not None:
                on_step(s, env, orc)
        assert env.status() == 0
        return worst
    finally:
        env.close()
