"""SBS1 snapshots (the reference's headless viewer feed) against the CPU oracle (GPU).

After each step the snapshot of an env must carry the oracle's state bit for
bit: the field (as f32), zone means, occupancy, zone flow setpoint and flow, VAV
and AHU values, native actions, boiler setpoint and return, the reward and its
terms, and the episode return summed in f32 as the env's record does.
"""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from oracle_util import OracleEnv, actions
from parity_util import scenario_paths

pytestmark = pytest.mark.gpu


def _expected(orc, vis, reward, parts8, ep_ret):
    ncv, nz, nv, na, nact = orc.ncv, orc.nz, orc.nv, orc.na, orc.nact
    o = 0

    def take(cnt):
        nonlocal o
        a = vis[o:o + cnt]
        o += cnt
        return a

    e = {"field": take(ncv).astype(np.float32)}
    for name in ("zone_temp", "occupancy", "zone_flow_sp", "zone_flow"):
        e[name] = take(nz)
    for name in ("vav_heat_sp", "vav_cool_sp", "vav_damper", "vav_reheat"):
        e[name] = take(nv)
    e["ahu_sat"], e["ahu_flow"], e["ahu_run"] = take(na), take(na), take(na).astype(np.int32)
    e["native"] = take(nact)
    e["step"], e["boiler_setpoint"], e["boiler_return"] = int(vis[o]), vis[o + 1], vis[o + 2]
    e["reward"], e["parts"], e["episode_return"] = reward, parts8, float(np.float32(ep_ret))
    return e


def test_snapshot_matches_oracle(scenario_cache, tmp_path):
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec, config_dir
    from neurips2026_smart_building_challenge_b200.sbs import PART_NAMES, read_snapshot

    d = config_dir(2, scenario_cache, n_steps=400)
    n = 8
    env = SmartBuildingsVec(n, blob_dir=str(d), groups=30)
    try:
        paths = scenario_paths(d)
        orc = [OracleEnv(paths[int(env.scenario[e])]) for e in range(n)]
        env.reset()
        for o in orc:
            o.reset()
        rng = np.random.default_rng(11)
        ep = np.zeros(n, np.float32)
        import torch
        for s in range(6):
            a = np.zeros((n, 272), np.float32)
            for e in range(n):
                a[e] = actions(rng, 1, orc[e].n_cont, orc[e].n_disc)[0]
            env.step(torch.from_numpy(a).to(env.device))
            env.synchronize()
            for e in range(n):
                _, r, _, rd, _, log8 = orc[e].step(a[e])
                ep[e] = np.float32(ep[e] + np.float32(r))
                if (e + s) % 3:
                    continue
                f = tmp_path / f"snap_{s}_{e}.sbs"
                env.snapshot(e, f)
                got = read_snapshot(f)
                exp = _expected(orc[e], orc[e].visible(), rd, log8, ep[e])
                where = f"step {s} env {e}"
                assert os.path.basename(got["blob"]) == paths[int(env.scenario[e])].name, where
                assert (got["nz"], got["nvav"], got["nahu"], got["ncv"], got["n_action"]) == \
                    (orc[e].nz, orc[e].nv, orc[e].na, orc[e].ncv, orc[e].nact), where
                assert got["step"] == exp["step"] == s + 1, where
                assert got["field"].ravel().view(np.uint32).tolist() == exp["field"].view(np.uint32).tolist(), where
                for name in ("zone_temp", "occupancy", "zone_flow_sp", "zone_flow", "vav_heat_sp", "vav_cool_sp",
                             "vav_damper", "vav_reheat", "ahu_sat", "ahu_flow", "ahu_run", "native"):
                    assert np.array_equal(got[name], exp[name]), f"{where}: {name}"
                for name in ("boiler_setpoint", "boiler_return", "reward", "episode_return"):
                    assert got[name] == exp[name], f"{where}: {name} {got[name]!r} vs {exp[name]!r}"
                assert [got["parts"][k] for k in PART_NAMES] == list(exp["parts"]), where
        assert env.status() == 0
    finally:
        env.close()


def test_snapshot_env_variable(scenario_cache, tmp_path):
    """SB_SNAPSHOT / SB_SNAP_ENV / SB_SNAP_EVERY: puf_step writes the file itself (fresh process)."""
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(1, scenario_cache)
    out = tmp_path / "live.sbs"
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))!r})
        from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec
        from neurips2026_smart_building_challenge_b200.sbs import read_snapshot
        env = SmartBuildingsVec(3, blob_dir={str(d)!r})
        env.reset()
        for _ in range(4):
            env.step()
        env.synchronize()
        snap = read_snapshot({str(out)!r})
        assert snap["env"] == 1 and snap["step"] == 4, (snap["env"], snap["step"])
        env.close()
        print("ok")
    """)
    envv = dict(os.environ, SB_SNAPSHOT=str(out), SB_SNAP_ENV="1", SB_SNAP_EVERY="2")
    r = subprocess.run([sys.executable, "-c", code], env=envv, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
