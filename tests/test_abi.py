"""The C-ABI libraries load and export every symbol their headers declare; the
host-only parts of the ABI (dictionary, error reporting) work without a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\([^;{]*\)\s*;", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "for", "while")))


def test_env_library_exports_header(built):
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = ctypes.CDLL(str(pkg.PKG / "libsbenv.so"))
    declared = _declared(ROOT / "include" / "sbenv.h")
    assert "puf_vec_create" in declared and "puf_step" in declared
    for sym in declared:
        assert hasattr(lib, sym), sym
    assert sorted(declared) == sorted(pkg.ENV_SYMBOLS)


def test_gen_library_exports_header(built):
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = ctypes.CDLL(str(pkg.PKG / "libsbgen.so"))
    declared = _declared(ROOT / "include" / "sbgen.h")
    assert sorted(declared) == sorted(pkg.GEN_SYMBOLS)
    for sym in declared:
        assert hasattr(lib, sym), sym


def test_dict_roundtrip(built):
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    d = lib.sb_dict_new(2)
    try:
        for i in range(40):
            lib.dict_set(d, f"k{i}".encode(), float(i))
        lib.dict_set_str(d, b"blob", b"/x/y.sbb")
        lib.dict_set(d, b"k3", 33.0)
        assert lib.dict_find(d, b"k3").contents.value == 33.0
        assert lib.dict_find(d, b"blob").contents.str == b"/x/y.sbb"
        assert not lib.dict_find(d, b"missing")
        assert pkg._dict_to_py(d)["k39"] == 39.0
    finally:
        lib.sb_dict_free(d)


def test_puf_log_writes_every_field(built):
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    log = pkg.Log(*[float(i) for i in range(len(pkg.LOG_FIELDS))])
    d = lib.sb_dict_new(4)
    try:
        lib.puf_log(ctypes.byref(log), d)
        out = pkg._dict_to_py(d)
    finally:
        lib.sb_dict_free(d)
    assert list(out) == pkg.LOG_FIELDS
    assert [out[f] for f in pkg.LOG_FIELDS] == [float(i) for i in range(len(pkg.LOG_FIELDS))]


def test_create_errors_are_reported(built, tmp_path):
    """No scenario / a corrupt blob: puf_vec_create returns NULL with a reason (never aborts)."""
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    buf = (ctypes.c_float * 4096)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    d = lib.sb_dict_new(4)
    try:
        assert not lib.puf_vec_create(4, d, p, p, p, p)
        assert b"no scenario" in lib.sb_last_error()
        bad = tmp_path / "bad.sbb"
        bad.write_bytes(b"SBB1" + b"\x01\0\0\0" + b"\xff" * 60)
        lib.dict_set_str(d, b"blob", str(bad).encode())
        assert not lib.puf_vec_create(4, d, p, p, p, p)
        assert lib.sb_last_error()
    finally:
        lib.sb_dict_free(d)


def test_env_requires_gpu_without_fallback(built):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import neurips2026_smart_building_challenge_b200 as pkg

    with pytest.raises(RuntimeError):
        pkg.SmartBuildingsVec(2, blob="/nonexistent.sbb")


def test_sampler_rejects_bad_arguments(built):
    """sb_beta_actions checks its arguments on the host, before any launch."""
    import neurips2026_smart_building_challenge_b200 as pkg

    lib = pkg.env_lib()
    buf = (ctypes.c_float * 16)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.sb_beta_actions(None, None, p, 4, 1.0, 12.0, 0, p) == -1
    assert lib.sb_beta_actions(p, None, p, 4, 1.0, 12.0, 0, None) == -1
    assert lib.sb_beta_actions(p, None, p, 0, 1.0, 12.0, 0, p) == -1
    assert lib.sb_beta_actions(p, None, p, 4, 0.0, 12.0, 0, p) == -1       # floor must be > 0
    assert lib.sb_beta_actions(p, None, p, 4, 1.0, 1.5, 0, p) == -1        # cap must exceed 2 floor
    assert b"sb_beta_actions" in lib.sb_last_error()


def test_snapshot_reader_rejects_bad_records():
    from neurips2026_smart_building_challenge_b200.sbs import parse_snapshot

    with pytest.raises(ValueError):
        parse_snapshot(b"XXXX" + bytes(700))
    import struct
    hdr = b"SBS1" + struct.pack("<12i", 1, 3, 100, 0, 1, 1, 1, 2, 2, 4, 1, 0) + struct.pack("<12d", *range(12))
    body = hdr + b"blob".ljust(512, b"\0") + bytes(4 * 4 + 8 * (4 + 4 + 2) + 4 + 8)
    snap = parse_snapshot(body)
    assert snap["step"] == 3 and snap["blob"] == "blob" and snap["field"].shape == (2, 2)
    with pytest.raises(ValueError):
        parse_snapshot(body[:-1])


def test_env_record_layout_matches_header(built, tmp_path):
    """The Python mirror of Env has the C layout (offsets and size from a probe
    compiled against include/sbenv.h), and its members follow the reference
    GPU backend's order (complete_port/gpu/smart_buildings.cu:116-143)."""
    import subprocess

    import neurips2026_smart_building_challenge_b200 as pkg

    names = [f for f, _ in pkg.EnvRecord._fields_]
    assert names[:24] == ["agents", "log", "ep_ret", "ep_part", "ep_worst", "num_agents", "tag", "boundary_reached",
                          "step", "max_steps", "start_offset", "start_day", "start_rng", "start_draws", "n_act",
                          "n_cont", "n_disc", "loaded", "rng", "seed", "cont", "disc", "native", "env_id"]
    src = tmp_path / "probe.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "sbenv.h"\nint main(void) {\n' +
                   "".join(f'  printf("%zu\\n", offsetof(Env, {n}));\n' for n in names) +
                   '  printf("%zu\\n", sizeof(Env));\n  return 0;\n}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(pkg.EnvRecord, n).offset for n in names] + [ctypes.sizeof(pkg.EnvRecord)]
    assert got == want
