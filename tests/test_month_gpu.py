"""Long-horizon parity of the device env (GPU): the north star's month contract.

* Configuration 1 for its whole month, 8,640 steps from Monday 16 January
  00:00 (four weekends at the weekend tariff, the January-February roll of the
  gas price, every occupancy arrival and departure window, 8,640 steps of
  accumulated state), then 24 steps into the next episode, with Beta(2,2)
  actions drawn with seed 0. Compared after every
  step with the reference's own C core (oracle/_ref/libcsimref.so, the
  restatement where it is absent) and with the digests recorded from the
  reference (tests/golden/ref_month.npz).
* Every configuration-2 scenario from Friday 27 January 18:00 for 1,300 steps:
  the evening departure window, a weekend, Monday, and the roll into February.

The exact build replays the reference's floating-point operations in order,
so every comparison is bit for bit (observations as f32 bit patterns, rewards
as f32 and f64, the field and interior mass every simulated hour).
"""
import numpy as np
import pytest

from parity_util import run_parity

pytestmark = pytest.mark.gpu

GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def test_config1_month_against_reference(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache)
    run_parity(d, n=2, steps=8640 + 24, seed=0, temp_every=12, oracle="reference", wild=False)


def test_config1_month_against_golden_digests(scenario_cache, tmp_path):
    """The device env alone against the reference's recorded month (no oracle at run time)."""
    import hashlib

    import torch

    from golden.make_golden import MONTH_HOUR, digest, month_actions, month_blob
    from parity_util import vec

    g = np.load(GOLD / "ref_month.npz")
    d = tmp_path / "month"
    d.mkdir()
    p = month_blob(d / "c1__w0.sbb")
    assert hashlib.sha256(p.read_bytes()).hexdigest() == str(g["sha256"])
    env = vec(1, d)
    try:
        env.reset()
        env.synchronize()
        ncv = len(g["temp_end"])
        assert digest(env.obs.cpu().numpy()[0]) == g["obs_digest"][0]
        h = 0
        n_cont, n_disc = int(env.records[0].n_cont), int(env.records[0].n_disc)
        for s, a in enumerate(month_actions(n_cont, n_disc)):
            env.step(torch.from_numpy(a[None]).to(env.device))
            env.synchronize()
            assert digest(env.obs.cpu().numpy()[0]) == g["obs_digest"][s + 1], f"obs step {s}"
            rd, _ = env.reward_f64()
            assert rd[0] == g["rew64"][s], f"reward step {s}"
            assert env.terminals.cpu().numpy()[0] == g["term"][s], f"terminal step {s}"
            if s % MONTH_HOUR == MONTH_HOUR - 1:
                assert digest(env.temp(0, ncv)) == g["temp_digest"][h], f"field at step {s}"
                assert digest(env.mass(0, len(g["mass_end"]))) == g["mass_digest"][h], f"mass at step {s}"
                h += 1
        np.testing.assert_array_equal(env.temp(0, ncv), g["temp_end"])
        assert env.status() == 0
    finally:
        env.close()


def test_config2_weekend_and_month_roll(scenario_cache):
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, scenario_cache, start_doy=26, start_hour=18, n_steps=1400)
    run_parity(d, n=30, steps=1300, seed=5, temp_every=12, groups=30, beta_mix=True, oracle="reference")
