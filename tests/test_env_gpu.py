"""Device env vs the CPU oracle, bit for bit (GPU).

The oracle is this repository's C restatement of the reference CPU core
(oracle/, pinned to the reference's own csim by tests/test_oracle.py). Every
comparison is exact: observations as f32 bit patterns, rewards as f32 and f64,
the temperature field and interior mass as f64. The north star allows 1e-9
relative per step; the device path replays the reference's operation order, so
the tolerance used here is zero.
"""
import numpy as np
import pytest

from oracle_util import OracleEnv, actions

pytestmark = pytest.mark.gpu


def _vec(n, blob_dir, **kw):
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec

    return SmartBuildingsVec(n, blob_dir=str(blob_dir), **kw)


def _run_parity(blob_dir, n, steps, max_steps=0, seed=0, temp_every=10, groups=0, beta_mix=False):
    import torch

    from neurips2026_smart_building_challenge_b200 import SB_NUM_ATNS

    env = _vec(n, blob_dir, max_steps=max_steps, groups=groups)
    try:
        blobs = sorted(blob_dir.glob("*.sbb"))
        from neurips2026_smart_building_challenge_b200.__init__ import SB_OBS  # noqa: F401
        # the env's own scenario assignment decides which blob each env runs
        lib_paths = _scenario_paths(env, blob_dir)
        orc = [OracleEnv(lib_paths[int(env.scenario[e])], max_steps=max_steps) for e in range(n)]
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
                kw = dict(alpha=al[e, :orc[e].n_cont], beta=be[e, :orc[e].n_cont]) if beta_mix else {}
                a[e] = actions(rng, 1, orc[e].n_cont, orc[e].n_disc, **kw)[0]
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
                if not np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)):
                    bad.append(f"obs fields {np.nonzero(obs[e] != o)[0][:8].tolist()}")
                if rew[e] != np.float32(r) or rd[e] != r64:
                    bad.append(f"reward {rd[e]!r} vs {r64!r}")
                if term[e] != t:
                    bad.append("terminal")
                if not np.array_equal(parts[e], log8):
                    bad.append(f"log terms {np.nonzero(parts[e] != log8)[0].tolist()} {parts[e]} vs {log8}")
                if bad or s % temp_every == 0 or s == steps - 1:
                    dT = env.temp(e, orc[e].ncv) - orc[e].temp()
                    dM = env.mass(e, orc[e].n) - orc[e].mass()
                    if dT.any():
                        bad.append(f"T differs at {np.count_nonzero(dT)} cells, max {np.abs(dT).max():.3e}")
                    if dM.any():
                        bad.append(f"M differs at {np.count_nonzero(dM)} cells, max {np.abs(dM).max():.3e}")
                if bad:
                    bad.append(_pre_stage_diff(env, orc[e], e))
                assert not bad, f"{where}: " + "; ".join(bad)
        assert env.status() == 0
        return env
    finally:
        env.close()


def _pre_stage_diff(env, orc, e):
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


def _scenario_paths(env, blob_dir):
    """Scenario index -> blob path, in the env's own (round-robin) order."""
    from neurips2026_smart_building_challenge_b200 import env_lib  # noqa: F401

    names = sorted(p.name for p in blob_dir.glob("*.sbb"))
    # building-first round robin of the native loader
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
                    order.append(blob_dir / nm)
                    used[i] = True
                    break
    return order


def test_config1_parity(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache)
    _run_parity(d, n=4, steps=120, max_steps=50, seed=1)


def test_config2_mix_parity(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    # 60 envs over the 30 scenarios: two per scenario, six solver groups
    _run_parity(d, n=60, steps=30, seed=2, temp_every=15, groups=30, beta_mix=True)


def test_notch_and_restart_parity(scenario_cache):
    """Unsolved (exterior) cells, strong convection, several in-step restarts."""
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    d = scenario_cache / "notch"
    d.mkdir(exist_ok=True)
    p = d / "notch__w0.sbb"
    if not p.exists():
        write_scenario(p, preset(1, 0, notch_rows=3, notch_cols=4, n_steps=60, start_hour=7, conv_p=0.5))
    _run_parity(d, n=3, steps=130, seed=3, temp_every=7)


def test_config3_parity(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(3, scenario_cache, n_steps=200)
    _run_parity(d, n=2, steps=12, seed=4, temp_every=4)


def test_mask_and_shapes(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import SB_MASK_WIDTH, config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    env = _vec(64, d, groups=30)
    try:
        m = env.mask().cpu().numpy()
        assert m.shape == (64, SB_MASK_WIDTH)
        for e in range(64):
            orc = OracleEnv(_scenario_paths(env, d)[int(env.scenario[e])])
            assert m[e, :orc.n_cont].all() and not m[e, orc.n_cont:256].any()
            assert m[e, 256:256 + 2 * orc.n_disc].all() and not m[e, 256 + 2 * orc.n_disc:].any()
        env.reset()
        env.synchronize()
        obs = env.obs.cpu().numpy()
        for e in range(64):
            assert not obs[e, env.obs_len[e]:].any()
    finally:
        env.close()


def test_config2_full_batch_sample(scenario_cache):
    """The bench configuration itself (960 envs, slabs of 6-7 envs, six dense classes):
    a sample of envs spread over the batch against the oracle, bit for bit."""
    import torch

    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    n, steps = 960, 6
    sample = [0, 1, 31, 159, 160, 479, 481, 700, 959]
    env = _vec(n, d, groups=30)
    try:
        paths = _scenario_paths(env, d)
        orc = {e: OracleEnv(paths[int(env.scenario[e])]) for e in sample}
        env.reset()
        env.synchronize()
        obs = env.obs.cpu().numpy()
        for e in sample:
            o = orc[e].reset()
            np.testing.assert_array_equal(obs[e].view(np.uint32), o.view(np.uint32), err_msg=f"reset env {e}")
        rng = np.random.default_rng(21)
        for s in range(steps):
            a = np.zeros((n, 272), np.float32)
            a[:, :256] = 2.0 * rng.beta(2.0, 2.0, size=(n, 256)) - 1.0
            a[:, 256:] = (rng.random((n, 16)) < 0.9).astype(np.float32)
            env.step(torch.from_numpy(a).to(env.device))
            env.synchronize()
            obs = env.obs.cpu().numpy()
            rd, _ = env.reward_f64()
            for e in sample:
                o, _, _, r64, _, _ = orc[e].step(a[e])
                assert np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)), f"step {s} env {e}"
                assert rd[e] == r64, f"step {s} env {e} reward"
        for e in sample:
            assert not (env.temp(e, orc[e].ncv) - orc[e].temp()).any(), f"field env {e}"
        assert env.status() == 0
    finally:
        env.close()
