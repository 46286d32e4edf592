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

from oracle_util import OracleEnv
from parity_util import run_parity as _run_parity, scenario_paths, vec as _vec

pytestmark = pytest.mark.gpu


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
            orc = OracleEnv(scenario_paths(d)[int(env.scenario[e])])
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
        paths = scenario_paths(d)
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


@pytest.mark.parametrize("wide", [0, 1], ids=["slabs", "wide"])
def test_config4_multiwave_sample(scenario_cache, wide):
    """Configuration 4's per-GPU batch (7,680 envs over the config-2 mix): the
    first solve on about 960 slabs, several waves of CTAs, or on 240 wide
    tiles of 32 envs; a sample of envs from every group and wave position
    against the oracle, bit for bit."""
    import torch

    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, scenario_cache, n_steps=400)
    n, steps = 7680, 5
    sample = [0, 1, 255, 256, 1279, 1280, 2561, 3839, 4000, 5119, 6400, 7679]
    env = _vec(n, d, groups=30, wide=wide)
    try:
        if wide:
            assert env.shape[6] == n // 32, "one wide tile per 32 envs of a group"
        else:
            assert env.shape[6] > 2 * 148, "expected several waves of slabs"
        paths = scenario_paths(d)
        orc = {e: OracleEnv(paths[int(env.scenario[e])]) for e in sample}
        env.reset()
        env.synchronize()
        obs = env.obs.cpu().numpy()
        for e in sample:
            assert np.array_equal(obs[e].view(np.uint32), orc[e].reset().view(np.uint32)), f"reset env {e}"
        rng = np.random.default_rng(22)
        for s in range(steps):
            a = np.zeros((n, 272), np.float32)
            a[:, :256] = 2.0 * rng.beta(2.0, 2.0, size=(n, 256)) - 1.0
            a[:, 256:] = 1.0
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
