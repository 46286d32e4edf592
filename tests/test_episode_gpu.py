"""Episode options, logs and resets of the device env against the CPU oracle (GPU).

The reference's GPU backend adds episode options its CPU env lacks
(complete_port/gpu/smart_buildings.cu:2583-2608, 2806-2816, 1636-1657,
1936-2050): desync (each env's first episode cut at a step drawn from its
index, the cut episodes kept out of the log), random_start (every episode
starting on a day drawn from a per-env SplitMix64 stream) and the learning-
reward normalisations rew_norm / rew_center. The oracle envs are given the
device env's per-env choices (oracle/sbo.h sbo_set_episode) and must agree
bit for bit. The Log records and the live log are recomputed from the
oracle's per-step outputs in the device's own arithmetic (float32 sums in
step order; double sums compared to 1e-12, their atomic order being free).
"""

import numpy as np
import pytest

from oracle_util import OracleEnv, actions
from parity_util import run_parity, scenario_paths, vec

pytestmark = pytest.mark.gpu


def test_desync_parity(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache, n_steps=60)
    seen = {}

    def check(s, env, orc):
        if s == 0:
            fl, _ = env.episode_options()
            seen["first"] = fl
            assert (fl >= 1).all() and (fl <= 60).all() and len(set(fl.tolist())) > 1
        if s == 199:
            env.synchronize()
            assert all(int(r.max_steps) == 60 for r in env.records)

    run_parity(d, n=8, steps=200, seed=11, temp_every=9, oracle="reference", env_kw={"desync": 1}, on_step=check)


def test_random_start_parity(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache, n_steps=300, random_start_days=7)
    days = set()

    def check(s, env, orc):
        env.synchronize()
        for e, o in enumerate(orc):
            assert int(env.records[e].start_offset) == o.episode_offset(), (s, e)
            days.add(o.episode_offset() // 288)

    # desync is ignored under random_start: every first episode is whole
    run_parity(d, n=6, steps=700, seed=12, temp_every=25, oracle="reference",
               env_kw={"random_start": 1, "random_start_seed": 7, "desync": 1}, on_step=check)
    assert len(days) >= 3


def test_random_start_needs_its_blob(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache, n_steps=60)
    with pytest.raises(RuntimeError, match="random_start"):
        vec(2, d, random_start=1)


def _f32(x):
    return np.float32(x)


def test_logs_and_live_log_against_oracle(scenario_cache):
    """Short desynchronised episodes run to completion: every Log field of
    every env, the live log's keys, and the truncated first episodes' absence."""
    import torch

    from neurips2026_smart_building_challenge_b200 import LOG_FIELDS, config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    n, steps, L = 12, 90, 25
    env = vec(n, d, groups=6, max_steps=L, desync=1)
    try:
        paths = scenario_paths(d)
        fl, _ = env.episode_options()
        orc = [OracleEnv(paths[int(env.scenario[e])], max_steps=L) for e in range(n)]
        for e in range(n):
            orc[e].set_episode(int(fl[e]))
            orc[e].reset()
        env.reset()
        env.live_log()   # clears the window
        rng = np.random.default_rng(13)
        log = {f: np.zeros(n, np.float32) for f in LOG_FIELDS}
        ep_ret = np.zeros(n, np.float32)
        ep_part = np.zeros((n, 8), np.float32)
        ep_worst = np.zeros(n, np.float32)
        step = np.zeros(n, np.int64)
        live = np.zeros(10)
        scn_sum = {}
        ep_scores = {}
        epret_d = np.zeros(n)
        for s in range(steps):
            a = np.zeros((n, 272), np.float32)
            for e in range(n):
                a[e] = actions(rng, 1, orc[e].n_cont, orc[e].n_disc)[0]
            env.step(torch.from_numpy(a).to(env.device))
            for e in range(n):
                _, r, t, rd, _, log8 = orc[e].step(a[e])
                r32 = _f32(r)
                step[e] += 1
                ep_ret[e] = _f32(ep_ret[e] + r32)
                epret_d[e] += rd
                for q in range(8):
                    ep_part[e, q] = _f32(ep_part[e, q] + _f32(log8[q]))
                if _f32(log8[4]) > ep_worst[e]:
                    ep_worst[e] = _f32(log8[4])
                live += np.concatenate([[1.0, float(r32)], log8])
                sc = int(env.scenario[e])
                acc = scn_sum.setdefault(sc, np.zeros(4))
                acc += [float(r32), log8[3], 1.0, float(r32) ** 2]
                if t:
                    assert step[e] == (fl[e] if s < fl[e] else L), (s, e)
                    st = _f32(step[e])
                    if step[e] >= L:   # whole episodes only
                        mean = _f32(ep_ret[e] / st)
                        ep_scores.setdefault(sc, []).append(epret_d[e] / step[e])
                        for f, v in [("perf", mean), ("score", mean), ("episode_return", ep_ret[e]),
                                     ("episode_length", st), ("productivity", _f32(ep_part[e, 0] / st)),
                                     ("energy_cost_norm", _f32(ep_part[e, 1] / st)),
                                     ("carbon_norm", _f32(ep_part[e, 2] / st)),
                                     ("comfort_dev_K", _f32(ep_part[e, 3] / st)), ("worst_dev_K", ep_worst[e]),
                                     ("out_of_band_frac", _f32(ep_part[e, 5] / st)), ("elec_kwh", ep_part[e, 6]),
                                     ("gas_kwh", ep_part[e, 7]), ("n", _f32(1.0))]:
                            log[f][e] = _f32(log[f][e] + v)
                    ep_ret[e] = 0.0
                    ep_part[e] = 0.0
                    ep_worst[e] = 0.0
                    step[e] = 0
                    epret_d[e] = 0.0
        env.synchronize()
        for e in range(n):
            for f in LOG_FIELDS:
                got = np.float32(getattr(env.records[e].log, f))
                assert got == log[f][e], f"env {e} Log.{f}: {got} vs {log[f][e]}"
        assert any(fl[e] < L for e in range(n)), "no truncated first episode in the sample"
        total = env.log()
        for f in LOG_FIELDS:
            assert abs(total[f] - float(np.sum(log[f], dtype=np.float64))) <= 1e-3 * max(1.0, abs(total[f])), f
        got = env.live_log()
        c = live[0]
        dt = 300.0
        want = {"live/reward": live[1] / c, "live/productivity": live[2] / c, "live/energy_cost_norm": live[3] / c,
                "live/carbon_norm": live[4] / c, "live/comfort_dev_K": live[5] / c, "live/worst_dev_K": live[6] / c,
                "live/out_of_band_frac": live[7] / c, "live/elec_kw": live[8] / c * 3600.0 / dt,
                "live/gas_kw": live[9] / c * 3600.0 / dt}
        names = {int(env.scenario[e]): paths[int(env.scenario[e])].stem for e in range(n)}
        for sc, acc in scn_sum.items():
            want[f"scenario/{names[sc]}/reward"] = acc[0] / acc[2]
            want[f"scenario/{names[sc]}/comfort_dev_K"] = acc[1] / acc[2]
        for sc, v in ep_scores.items():
            want[f"scenario/{names[sc]}/episode_score"] = -float(np.mean(v))
        for k, v in want.items():
            assert k in got, k
            assert abs(got[k] - v) <= 1e-12 * max(1.0, abs(v)), f"{k}: {got[k]} vs {v}"
        assert got["env/episode_score_n_scen"] == 6.0
    finally:
        env.close()


@pytest.mark.parametrize("mode", ["rew_norm", "rew_center"])
def test_reward_normalisation(scenario_cache, mode):
    """rewards[] = (r - mean) * inv_std per scenario in float32; the statistics
    move towards each puf_live_log window (0.1 for rew_norm, center_beta for
    rew_center), starting at mean 0 and variance 0.217 (rew_norm) or 1."""
    import torch

    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    n = 12
    kw = {mode: 1, "center_beta": 0.25}
    env = vec(n, d, groups=6, **kw)
    try:
        env.reset()
        G = 6
        mu = np.zeros(G)
        var = np.full(G, 0.217 if mode == "rew_norm" else 1.0)
        rng = np.random.default_rng(14)
        for window in range(3):
            acc = np.zeros((G, 4))
            for s in range(5):
                a = np.zeros((n, 272), np.float32)
                a[:, :256] = 2.0 * rng.beta(2.0, 2.0, size=(n, 256)) - 1.0
                a[:, 256:] = 1.0
                env.step(torch.from_numpy(a).to(env.device))
                env.synchronize()
                rd, _ = env.reward_f64()
                got = env.rewards.cpu().numpy()
                for e in range(n):
                    sc = int(env.scenario[e])
                    r32 = np.float32(rd[e])
                    inv = np.float32(1.0) if mode == "rew_center" else np.float32(1.0 / np.sqrt(max(var[sc], 1e-12)))
                    want = np.float32(np.float32(r32 - np.float32(mu[sc])) * inv)
                    # window 0 is exact; later windows' statistics come from double sums
                    # whose atomic order is free, so they may differ in the last float bit
                    tol = 0.0 if window == 0 else 4e-7 * max(1.0, abs(float(want)))
                    assert abs(float(got[e]) - float(want)) <= tol, (window, s, e, got[e], want)
                    acc[sc] += [float(r32), 0.0, 1.0, float(r32) ** 2]
            out = env.live_log()
            b = 0.25 if mode == "rew_center" else 0.1
            for sc in range(G):
                if acc[sc, 2] > 0:
                    mw = acc[sc, 0] / acc[sc, 2]
                    mu[sc] = (1 - b) * mu[sc] + b * mw
                    if mode == "rew_norm":
                        var[sc] = (1 - b) * var[sc] + b * max(acc[sc, 3] / acc[sc, 2] - mw * mw, 1e-12)
            assert abs(out["norm/reward_mean"] - mu.mean()) < 1e-6
            if mode == "rew_norm":
                assert "live/rew_z_gt1_frac" in out
    finally:
        env.close()


def test_second_reset_matches_oracle(scenario_cache):
    """puf_reset in the middle of an episode: the random inputs produced one step
    ahead and never consumed are undone, so the restarted envs continue exactly
    as the reference's envs do after their reset."""
    import torch

    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache, n_steps=300)
    n = 3
    env = vec(n, d)
    try:
        path = scenario_paths(d)[0]
        orc = [OracleEnv(path) for _ in range(n)]
        rng = np.random.default_rng(15)
        for phase, steps in enumerate((37, 30, 11)):
            env.reset()
            env.synchronize()
            obs = env.obs.cpu().numpy()
            for e in range(n):
                o = orc[e].reset()
                assert np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)), (phase, e)
            for s in range(steps):
                a = np.concatenate([actions(rng, 1, orc[e].n_cont, orc[e].n_disc) for e in range(n)])
                env.step(torch.from_numpy(a).to(env.device))
                env.synchronize()
                obs = env.obs.cpu().numpy()
                rd, _ = env.reward_f64()
                for e in range(n):
                    o, _, _, r64, _, _ = orc[e].step(a[e])
                    assert np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)), (phase, s, e)
                    assert rd[e] == r64, (phase, s, e)
            for e in range(n):
                assert np.array_equal(env.temp(e, orc[e].ncv), orc[e].temp()), (phase, e)
        assert env.status() == 0
    finally:
        env.close()


@pytest.mark.parametrize("wide", [0, 1], ids=["slabs", "wide"])
def test_bounded_wait_runs_out_and_reports(scenario_cache, wide):
    """A sweep wait that can never be satisfied (sb_test_stall: warp 0 waits for
    a row no warp publishes, under a short spin limit) ends with status 5 and
    no fault or hang; after puf_reset the env steps exactly as the oracle does.
    Both first solves: the slabs' ready-flag waits (wide = 0) and the wide
    tiles' ready-count waits (wide = 1), whose other warps and program producer
    then leave their own waits."""
    import torch

    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache, n_steps=60)
    n = 2
    env = vec(n, d, wide=wide)
    try:
        path = scenario_paths(d)[0]
        rng = np.random.default_rng(16)
        # the oracle envs step beside the device env throughout, so their random
        # streams are where the device env's are when both restart
        orc = [OracleEnv(path) for _ in range(n)]

        def act():
            return np.concatenate([actions(rng, 1, orc[e].n_cont, orc[e].n_disc) for e in range(n)])

        env.reset()
        for e in range(n):
            orc[e].reset()
        for stalled in (False, True):
            if stalled:
                assert env.lib.sb_test_stall(1, 1 << 12) == 0
            a = act()
            env.step(torch.from_numpy(a).to(env.device))
            env.synchronize()
            for e in range(n):
                orc[e].step(a[e])
            assert env.status() == (5 if stalled else 0)
        assert env.lib.sb_test_stall(0, 0) == 0
        env.reset()
        assert env.status() == 0
        env.synchronize()
        obs = env.obs.cpu().numpy()
        for e in range(n):
            assert np.array_equal(obs[e].view(np.uint32), orc[e].reset().view(np.uint32))
        for s in range(5):
            a = act()
            env.step(torch.from_numpy(a).to(env.device))
            env.synchronize()
            obs = env.obs.cpu().numpy()
            for e in range(n):
                o = orc[e].step(a[e])[0]
                assert np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)), (s, e)
        assert env.status() == 0
    finally:
        env.close()
