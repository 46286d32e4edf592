"""Policy-in-loop rollouts on the GPU.

The action sampler (`sb_beta_actions`) is checked against the distributions it
draws from: per-head means and variances of the Beta draws against the closed
forms, a pooled probability-integral-transform KS test, categorical
frequencies, the mask rules and the counter/seed contract. The rollout (policy
GEMMs + sampler + env step, captured in a CUDA graph) is checked against the
CPU oracle: the actions the sampler wrote each step are fed to the oracle and
the observations must agree bit for bit, and the captured step must produce
the same trajectory as the same steps run eagerly.
"""
import numpy as np
import pytest

from oracle_util import OracleEnv
from parity_util import scenario_paths

pytestmark = pytest.mark.gpu

WIDTH = 288


def _lib():
    from neurips2026_smart_building_challenge_b200 import env_lib

    return env_lib()


def _sample(raw, n, floor_c=1.0, cap=12.0, seed=0, call=0, mask=None):
    import torch

    lib = _lib()
    act = torch.full((n, 272), 7.0, dtype=torch.float32, device="cuda:0")
    c = torch.tensor([call], dtype=torch.int64, device="cuda:0")
    mp = mask.data_ptr() if mask is not None else None
    assert lib.sb_beta_actions(raw.data_ptr(), mp, act.data_ptr(), n, floor_c, cap, seed, c.data_ptr()) == 0
    torch.cuda.synchronize()
    return act.cpu().numpy()


def _softplus_inv(y):
    return np.where(y > 20, y, np.log(np.expm1(np.maximum(y, 1e-30))))


def _shapes(n, floor_c, a_t, b_t):
    """raw logits whose concentrations are a_t, b_t per continuous head."""
    import torch

    raw = np.zeros((2, n, WIDTH), np.float32)
    raw[0, :, :256] = _softplus_inv(a_t - floor_c)
    raw[1, :, :256] = _softplus_inv(b_t - floor_c)
    return torch.from_numpy(raw).to("cuda:0")


def _capped(a, b, cap):
    s = a + b
    k = np.where((cap > 0) & (s > cap), cap / s, 1.0)
    return a * k, b * k


@pytest.mark.parametrize("floor_c,cap,lo,hi", [(1.0, 12.0, 1.0, 10.0), (1.0, 0.0, 1.0, 30.0),
                                               (0.25, 0.0, 0.3, 3.0)])
def test_beta_moments(built, floor_c, cap, lo, hi):
    from scipy import stats

    n = 4096
    h = np.arange(256)
    a_t = lo + (hi - lo) * (h % 16) / 15.0
    b_t = lo + (hi - lo) * (h // 16) / 15.0
    raw = _shapes(n, floor_c, a_t, b_t)
    x = (_sample(raw, n, floor_c, cap)[:, :256].astype(np.float64) + 1.0) / 2.0
    a, b = _capped(a_t, b_t, cap)
    m, v, _, kurt = stats.beta.stats(a, b, moments="mvsk")
    mu4 = (np.asarray(kurt) + 3.0) * v * v
    z_mean = (x.mean(0) - m) / np.sqrt(v / n)
    z_var = (x.var(0) - v) / np.sqrt((mu4 - v * v) / n)
    assert np.abs(z_mean).max() < 5.5, np.abs(z_mean).max()
    assert np.abs(z_var).max() < 5.5, np.abs(z_var).max()
    assert 0.6 < (z_mean ** 2).mean() < 1.5
    # pooled probability integral transform (shapes >= 1 only: below 1 the
    # clamp into [1e-6, 1 - 1e-6] holds visible mass at the ends)
    if lo >= 1.0:
        pit = stats.beta.cdf(x, a[None, :], b[None, :]).ravel()
        assert stats.kstest(pit, "uniform").pvalue > 1e-6


def test_discrete_heads_and_mask(built):
    import torch

    n = 8192
    raw = np.zeros((2, n, WIDTH), np.float32)
    l1 = np.arange(16, dtype=np.float32) - 8.0          # class-1 logit per discrete head
    raw[0, :, 257::2] = l1
    raw_d = torch.from_numpy(raw).to("cuda:0")
    act = _sample(raw_d, n)
    d = act[:, 256:]
    assert set(np.unique(d)) <= {0.0, 1.0}
    p = 1.0 / (1.0 + np.exp(-l1.astype(np.float64)))
    z = (d.mean(0) - p) / np.sqrt(p * (1 - p) / n)
    assert np.abs(z).max() < 5.5, z

    mask = np.ones((n, WIDTH), np.uint8)
    mask[:, 5] = 0                 # a masked continuous head
    mask[:, 256] = 0               # discrete head 0: class 0 masked -> always 1
    mask[:, 259] = 0               # discrete head 1: class 1 masked -> always 0
    mask[:, 260:262] = 0           # discrete head 2: padding -> 0.0
    act = _sample(raw_d, n, mask=torch.from_numpy(mask).to("cuda:0"))
    assert (act[:, 5] == 0.0).all()
    assert (act[:, 256] == 1.0).all() and (act[:, 257] == 0.0).all() and (act[:, 258] == 0.0).all()
    assert set(np.unique(act[:, 259:])) <= {0.0, 1.0}
    assert ((act[:, :256] > -1.0) & (act[:, :256] < 1.0)).all()


def test_counter_seed_and_bad_logits(built):
    import torch

    n = 256
    rng = np.random.default_rng(5)
    raw = rng.normal(0, 3, size=(2, n, WIDTH)).astype(np.float32)
    raw[0, 0, :8] = [np.nan, np.inf, -np.inf, 1e30, -1e30, np.nan, 0, 0]
    raw[1, 0, :8] = [0, np.nan, np.inf, -np.inf, 1e30, np.nan, np.inf, -np.inf]
    raw[0, 1, 256:262] = [np.nan, 0, np.inf, -np.inf, np.nan, np.nan]
    r = torch.from_numpy(raw).to("cuda:0")
    a0 = _sample(r, n, seed=3, call=11)
    assert np.array_equal(a0, _sample(r, n, seed=3, call=11))
    assert not np.array_equal(a0[:, :256], _sample(r, n, seed=3, call=12)[:, :256])
    assert not np.array_equal(a0[:, :256], _sample(r, n, seed=4, call=11)[:, :256])
    assert not np.array_equal(a0[:, :256], _sample(r, n, seed=3, call=11 + (1 << 32))[:, :256])
    assert np.isfinite(a0).all()
    assert ((a0[:, :256] > -1.0) & (a0[:, :256] < 1.0)).all()
    assert set(np.unique(a0[:, 256:])) <= {0.0, 1.0}


def test_rollout_graph_parity(scenario_cache):
    """Captured env+policy steps: the env's answer to the sampled actions is the oracle's, bit for bit."""
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec, config_dir
    from neurips2026_smart_building_challenge_b200.rollout import Rollout, ZonePolicy

    d = config_dir(2, scenario_cache, n_steps=400)
    n, steps = 12, 40
    env = SmartBuildingsVec(n, blob_dir=str(d))
    try:
        paths = scenario_paths(d)
        orc = [OracleEnv(paths[int(env.scenario[e])]) for e in range(n)]
        env.reset()
        for o in orc:
            o.reset()
        ro = Rollout(env, ZonePolicy(env.device, seed=7), seed=9, graph=True)
        for s in range(steps):
            ro.step()
            env.synchronize()
            act = env.actions.cpu().numpy()
            obs = env.obs.cpu().numpy()
            for e in range(n):
                o, *_ = orc[e].step(act[e])
                assert np.array_equal(obs[e].view(np.uint32), o.view(np.uint32)), f"step {s} env {e}"
        assert int(ro.call.item()) == steps
        assert env.status() == 0
    finally:
        env.close()


def test_rollout_graph_matches_eager(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec, config_dir
    from neurips2026_smart_building_challenge_b200.rollout import Rollout, ZonePolicy

    d = config_dir(2, scenario_cache, n_steps=400)
    out = []
    for graph in (True, False):
        env = SmartBuildingsVec(64, blob_dir=str(d))
        try:
            env.reset()
            ro = Rollout(env, ZonePolicy(env.device, seed=1), seed=2, graph=graph)
            ro.run(24)
            env.synchronize()
            out.append((env.obs.cpu().numpy().copy(), env.rewards.cpu().numpy().copy(),
                        env.actions.cpu().numpy().copy()))
            assert env.status() == 0
        finally:
            env.close()
    for a, b in zip(out[0], out[1]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
