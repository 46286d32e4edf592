"""In-tree build of the native libraries.

libsbenv.so  the batched env: CUDA kernels for sm_100a + host orchestration (C ABI, include/sbenv.h)
libsbgen.so  the synthetic SBB1 scenario generator (C ABI, include/sbgen.h)

Both are compiled with contraction of multiply-add disabled (-fmad=false on the
device, -ffp-contract=off on the host) because the env replays the reference
CPU core's floating-point operations in order, bit for bit.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and r.stderr.strip():
        sys.stderr.write(r.stderr)


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def build_gen(verbose: bool = False, force: bool = False) -> Path:
    out = PKG / "libsbgen.so"
    srcs = [CSRC / "synth.cpp", CSRC / "sbb.cpp", CSRC / "sbb.h", INCLUDE / "sbgen.h"]
    if force or _stale(out, srcs):
        _run([CXX, "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-Wall", "-Wextra",
              f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(out), str(CSRC / "synth.cpp"), str(CSRC / "sbb.cpp")],
             verbose)
    return out


def build_env(verbose: bool = False, force: bool = False) -> Path:
    out = PKG / "libsbenv.so"
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.cpp")) + \
        sorted(CSRC.glob("*.h")) + [INCLUDE / "sbenv.h"]
    if not (force or _stale(out, srcs)):
        return out
    BUILD.mkdir(exist_ok=True)
    host_objs = []
    for name in ["tables.cpp", "sweep_sched.cpp", "wide_sched.cpp", "sbb.cpp"]:
        obj = BUILD / (name + ".o")
        _run([CXX, "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-Wall", "-Wextra",
              f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(CSRC / name), "-o", str(obj)], verbose)
        host_objs.append(str(obj))
    cu_obj = BUILD / "env.cu.o"
    _run([NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xptxas", "-v",
          "-Xcompiler", "-fPIC,-ffp-contract=off", f"-I{INCLUDE}", f"-I{CSRC}",
          "-c", str(CSRC / "env.cu"), "-o", str(cu_obj)], verbose)
    _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(out), str(cu_obj), *host_objs,
          "-lcudart"], verbose)
    return out


def reference_csim_dir() -> Path | None:
    """The reference's C core sources: $SB_REFERENCE_DIR/complete_port/csim, else a
    checkout named `reference` beside this repository; None when neither exists
    (then oracle/_ref keeps whatever was built before)."""
    env = os.environ.get("SB_REFERENCE_DIR")
    for base in ([Path(env)] if env else []) + [ROOT.parent / "reference"]:
        d = base / "complete_port" / "csim"
        if (d / "sb_sim.c").exists():
            return d
    return None


def build_oracle(verbose: bool = False) -> None:
    """Builds the CPU checker (TEST INFRASTRUCTURE) under oracle/."""
    cmd = ["make", "-s", "-C", str(ROOT / "oracle"), "all"]
    ref = reference_csim_dir()
    if ref is not None:
        cmd.append(f"REF_DIR={ref}")
    _run(cmd, verbose)


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_gen(verbose, force)
    build_env(verbose, force)
    build_oracle(verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv, force="-f" in sys.argv)
