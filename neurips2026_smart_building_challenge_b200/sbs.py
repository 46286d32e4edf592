"""SBS1 snapshot files: one env's visible state after a step.

The reference's viewer feed (complete_port/gpu/smart_buildings.cu:2205-2290,
parsed by its viewer): written by `sb_snapshot_write` / `SmartBuildingsVec.snapshot`
or, with SB_SNAPSHOT=<file> set, by puf_step. Layout (little-endian): "SBS1",
i32[12] {version 1, step, episode length, env, zones, VAVs, AHUs, rows, cols,
cells, actions, 0}, f64[12] {reward, episode return, boiler setpoint, boiler
return, 8 reward terms}, char[512] scenario path, f32 field[cells], f64 zone means,
occupancy, zone flow setpoint, zone flow [zones each], f64 VAV heating and cooling
setpoints, damper, reheat [VAVs each], f64 AHU supply temperature and flow [AHUs
each], i32 AHU run [AHUs], f64 native actions [actions].
"""
from __future__ import annotations

import os
import struct

import numpy as np

HEADER_INTS = ("version", "step", "max_steps", "env", "nz", "nvav", "nahu", "rows", "cols", "ncv", "n_action")
PART_NAMES = ("productivity", "energy_cost", "carbon", "comfort_dev_K", "worst_dev_K", "out_of_band",
              "elec_kwh", "gas_kwh")


def parse_snapshot(buf: bytes) -> dict:
    """Fields of one SBS1 record; raises ValueError on a malformed or truncated record."""
    if len(buf) < 4 + 48 + 96 + 512 or buf[:4] != b"SBS1":
        raise ValueError("not an SBS1 snapshot")
    ints = struct.unpack_from("<12i", buf, 4)
    out = dict(zip(HEADER_INTS, ints))
    if out["version"] != 1:
        raise ValueError(f"SBS1 version {out['version']}")
    sc = struct.unpack_from("<12d", buf, 52)
    out["reward"], out["episode_return"], out["boiler_setpoint"], out["boiler_return"] = sc[:4]
    out["parts"] = dict(zip(PART_NAMES, sc[4:]))
    out["blob"] = buf[148:660].split(b"\0", 1)[0].decode()
    off = 660
    nz, nv, na, ncv, nact = out["nz"], out["nvav"], out["nahu"], out["ncv"], out["n_action"]
    need = off + 4 * ncv + 8 * (4 * nz + 4 * nv + 2 * na) + 4 * na + 8 * nact
    if len(buf) != need:
        raise ValueError(f"SBS1 size {len(buf)}, expected {need}")

    def take(dtype, count):
        nonlocal off
        a = np.frombuffer(buf, dtype=dtype, count=count, offset=off).copy()
        off += a.nbytes
        return a

    out["field"] = take("<f4", ncv).reshape(out["rows"], out["cols"]) if out["rows"] * out["cols"] == ncv \
        else take("<f4", ncv)
    for name in ("zone_temp", "occupancy", "zone_flow_sp", "zone_flow"):
        out[name] = take("<f8", nz)
    for name in ("vav_heat_sp", "vav_cool_sp", "vav_damper", "vav_reheat"):
        out[name] = take("<f8", nv)
    out["ahu_sat"] = take("<f8", na)
    out["ahu_flow"] = take("<f8", na)
    out["ahu_run"] = take("<i4", na)
    out["native"] = take("<f8", nact)
    return out


def read_snapshot(path: str | os.PathLike) -> dict:
    with open(path, "rb") as f:
        return parse_snapshot(f.read())
