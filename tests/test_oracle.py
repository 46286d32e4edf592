"""The CPU oracle, pinned: the C restatement (oracle/liboracle.so) against the
reference's own C core (golden fixtures recorded from it, and the compiled
reference itself where the reference tree is available), and MT19937 against
numpy's RandomState (the stream the reference draws from)."""
import ctypes
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle_util import PORT, REF, OracleEnv, actions, lib

GOLD = Path(__file__).resolve().parent / "golden"


def test_golden_blob_is_reproducible(built, tmp_path):
    from golden.make_golden import small_blob

    p = small_blob(tmp_path / "small.sbb")
    g = np.load(GOLD / "ref_small.npz")
    assert hashlib.sha256(p.read_bytes()).hexdigest() == str(g["sha256"])


def test_port_matches_reference_golden(built, tmp_path):
    """Bit-exact replay of the reference's recorded episode (includes an in-step restart)."""
    from golden.make_golden import small_blob

    g = np.load(GOLD / "ref_small.npz")
    env = OracleEnv(small_blob(tmp_path / "small.sbb"), path=PORT)
    L = env.obs_len
    o = env.reset()
    np.testing.assert_array_equal(o[:L].view(np.uint32), g["obs"][0].view(np.uint32))
    assert not o[L:].any()
    ti = 0
    for s in range(len(g["rew64"])):
        o, r, t, rd, p12, _ = env.step(g["actions"][s])
        np.testing.assert_array_equal(o[:L].view(np.uint32), g["obs"][s + 1].view(np.uint32), err_msg=f"step {s}")
        assert rd == g["rew64"][s] and np.float32(r) == g["rew32"][s] and t == g["term"][s]
        np.testing.assert_array_equal(p12, g["parts"][s])
        if s in g["temp_at"]:
            np.testing.assert_array_equal(env.temp(), g["temp"][ti])
            np.testing.assert_array_equal(env.mass(), g["mass"][ti])
            ti += 1
    assert ti == len(g["temp_at"])


@pytest.mark.skipif(not REF.exists(), reason="reference C core not built (reference tree absent)")
@pytest.mark.parametrize("config,index,over,steps,max_steps", [
    (1, 0, dict(n_steps=300), 160, 70),
    (2, 27, dict(n_steps=300), 60, 0),
    (2, 8, dict(n_steps=300, start_hour=6), 60, 25),
])
def test_port_matches_reference(built, tmp_path, config, index, over, steps, max_steps):
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    p = write_scenario(tmp_path / "s.sbb", preset(config, index, **over))
    a_env, b_env = OracleEnv(p, max_steps, PORT), OracleEnv(p, max_steps, REF)
    np.testing.assert_array_equal(a_env.reset().view(np.uint32), b_env.reset().view(np.uint32))
    rng = np.random.default_rng(index)
    for s in range(steps):
        a = actions(rng, 1, a_env.n_cont, a_env.n_disc)[0]
        ra, rb = a_env.step(a), b_env.step(a)
        np.testing.assert_array_equal(ra[0].view(np.uint32), rb[0].view(np.uint32), err_msg=f"obs {s}")
        assert ra[1:4] == rb[1:4], s
        np.testing.assert_array_equal(ra[4], rb[4])
        np.testing.assert_array_equal(ra[5][:7], rb[5][:7])
    np.testing.assert_array_equal(a_env.temp(), b_env.temp())
    np.testing.assert_array_equal(a_env.mass(), b_env.mass())


def test_port_matches_reference_month_golden(built, tmp_path):
    """The restatement through configuration 1's whole month (8,640 steps from
    Monday 16 January: four weekends, the month roll, every occupancy window)
    and into the next episode, against the digests recorded from the reference."""
    from golden.make_golden import MONTH_HOUR, digest, month_actions, month_blob

    g = np.load(GOLD / "ref_month.npz")
    p = month_blob(tmp_path / "month.sbb")
    assert hashlib.sha256(p.read_bytes()).hexdigest() == str(g["sha256"])
    env = OracleEnv(p, path=PORT)
    assert digest(env.reset()) == g["obs_digest"][0]
    h = 0
    for s, a in enumerate(month_actions(env.n_cont, env.n_disc)):
        o, r, t, rd, _, _ = env.step(a)
        assert digest(o) == g["obs_digest"][s + 1], f"obs step {s}"
        assert rd == g["rew64"][s] and np.float32(r) == g["rew32"][s] and t == g["term"][s], f"reward step {s}"
        if s % MONTH_HOUR == MONTH_HOUR - 1:
            assert digest(env.temp()) == g["temp_digest"][h] and digest(env.mass()) == g["mass_digest"][h], s
            h += 1
    np.testing.assert_array_equal(env.temp(), g["temp_end"])
    np.testing.assert_array_equal(env.mass(), g["mass_end"])


@pytest.mark.skipif(not REF.exists(), reason="reference C core not built (reference tree absent)")
@pytest.mark.parametrize("index", [0, 7, 14, 16, 23, 29])
def test_port_matches_reference_weekend_span(built, tmp_path, index):
    """Configuration-2 scenarios (every layout) from Friday 27 January 18:00 for
    1,300 steps: the evening departure window, a weekend at the weekend tariff,
    Monday's arrivals and departures, and the roll into February."""
    from neurips2026_smart_building_challenge_b200 import preset, write_scenario

    p = write_scenario(tmp_path / "s.sbb", preset(2, index, start_doy=26, start_hour=18, n_steps=1400))
    a_env, b_env = OracleEnv(p, 0, PORT), OracleEnv(p, 0, REF)
    np.testing.assert_array_equal(a_env.reset().view(np.uint32), b_env.reset().view(np.uint32))
    rng = np.random.default_rng(100 + index)
    al = rng.uniform(0.5, 12.0, size=a_env.n_cont)
    be = rng.uniform(0.5, 12.0, size=a_env.n_cont)
    for s in range(1300):
        a = actions(rng, 1, a_env.n_cont, a_env.n_disc, alpha=al, beta=be)[0]
        ra, rb = a_env.step(a), b_env.step(a)
        np.testing.assert_array_equal(ra[0].view(np.uint32), rb[0].view(np.uint32), err_msg=f"obs {s}")
        assert ra[1:4] == rb[1:4], s
        np.testing.assert_array_equal(ra[4], rb[4])
        if s % 12 == 11:
            np.testing.assert_array_equal(a_env.temp(), b_env.temp())
    np.testing.assert_array_equal(a_env.mass(), b_env.mass())


class _Mt(ctypes.Structure):
    _fields_ = [("s", ctypes.c_uint32 * 624), ("pos", ctypes.c_int)]


def test_mt19937_matches_numpy(built):
    l = lib(PORT)
    l.sbo_mt_sample.restype = ctypes.c_double
    l.sbo_mt_bounded.restype = ctypes.c_uint32
    l.sbo_mt_bounded.argtypes = [ctypes.POINTER(_Mt), ctypes.c_uint32]
    l.sbo_mt_seed.argtypes = [ctypes.POINTER(_Mt), ctypes.c_uint32]
    l.sbo_mt_sample.argtypes = [ctypes.POINTER(_Mt)]
    g = np.load(GOLD / "mt19937.npz")
    for seed in (0, 5, 17321, 4294967295):
        m = _Mt()
        l.sbo_mt_seed(ctypes.byref(m), seed)
        got = np.array([l.sbo_mt_sample(ctypes.byref(m)) for _ in range(2000)])
        np.testing.assert_array_equal(got, g[f"sample_{seed}"])
        his = [hi for hi in (0, 1, 5, 7, 8, 100, 1023, 1 << 20) for _ in range(50)]
        got = np.array([l.sbo_mt_bounded(ctypes.byref(m), hi) for hi in his])
        np.testing.assert_array_equal(got, g[f"randint_{seed}"])


def test_mt19937_reference_sequence(built):
    """init_genrand(5489): the published first outputs of MT19937."""
    l = lib(PORT)
    l.sbo_mt_next.restype = ctypes.c_uint32
    l.sbo_mt_next.argtypes = [ctypes.POINTER(_Mt)]
    l.sbo_mt_seed.argtypes = [ctypes.POINTER(_Mt), ctypes.c_uint32]
    m = _Mt()
    l.sbo_mt_seed(ctypes.byref(m), 5489)
    first = [l.sbo_mt_next(ctypes.byref(m)) for _ in range(5)]
    assert first == [3499211612, 581869302, 3890346734, 3586334585, 545404204]


def test_oracle_rejects_bad_blob(built, tmp_path):
    p = tmp_path / "bad.sbb"
    p.write_bytes(b"SBB1" + b"\0" * 60)
    with pytest.raises(RuntimeError):
        OracleEnv(p)
