"""Batched Smart Buildings HVAC environment on B200.

The product is the native library ``libsbenv.so`` (CUDA kernels for sm_100a
behind the PufferLib GPU-backend C ABI declared in ``include/sbenv.h``). This
module is a thin host mirror of that interface for Python callers: it owns the
trainer-side device buffers (torch tensors, used only as device memory) and
forwards to ``puf_vec_create`` / ``puf_reset`` / ``puf_step`` / ``puf_log`` /
``puf_live_log`` / ``puf_mask_init`` (reference:
complete_port/gpu/smart_buildings.cu:2497-3323). There is no CPU fallback: if
the library or a GPU is missing, construction raises.

``write_scenario`` / ``preset`` wrap the synthetic SBB1 generator (``libsbgen.so``).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent

SB_OBS = 1024
SB_CONT = 256
SB_DISC = 16
SB_NUM_ATNS = SB_CONT + SB_DISC
SB_MASK_WIDTH = SB_CONT + 2 * SB_DISC
SB_NPARTS = 8

LOG_FIELDS = ["perf", "score", "episode_return", "episode_length", "comfort_dev_K", "worst_dev_K",
              "out_of_band_frac", "productivity", "energy_cost_norm", "carbon_norm", "elec_kwh",
              "gas_kwh", "n"]

# Every C-ABI entry point of include/sbenv.h (checked by the tests against the header).
ENV_SYMBOLS = ["sb_dict_new", "sb_dict_free", "dict_find", "dict_set", "dict_set_str", "puf_vec_create",
               "puf_bind_stream", "puf_init", "puf_reset", "puf_step", "puf_render", "puf_close", "puf_log",
               "puf_live_log", "puf_mask_init", "sb_last_error", "sb_device_status", "sb_shape",
               "sb_env_info", "sb_get_temp", "sb_get_mass", "sb_get_reward_f64", "sb_kernels_per_step",
               "sb_solve_schedule", "sb_sweep_warps", "sb_sweep_stats", "sb_debug_state", "sb_step_timed", "sb_solve_bytes",
               "sb_dense_check", "sb_dense_check_mode", "sb_beta_actions", "sb_snapshot_write", "sb_dense_solve_noalloc",
               "sb_episode_options", "sb_solve_flops", "sb_fp64_peak", "sb_scenario_stats", "sb_test_stall",
               "sb_wide_schedule", "sb_wide_warps", "sb_wide_config"]
GEN_SYMBOLS = ["sbgen_preset", "sbgen_write", "sbgen_factor_stats"]


class Log(ctypes.Structure):
    _fields_ = [(f, ctypes.c_float) for f in LOG_FIELDS]


class Agent(ctypes.Structure):
    _fields_ = [("observations", ctypes.c_void_p), ("actions", ctypes.c_void_p), ("rewards", ctypes.c_void_p),
                ("terminals", ctypes.c_void_p), ("action_mask", ctypes.c_void_p)]


class EnvRecord(ctypes.Structure):
    """include/sbenv.h Env: the reference GPU backend's member order, then `scenario`."""
    _fields_ = [("agents", Agent * 1), ("log", Log), ("ep_ret", ctypes.c_float),
                ("ep_part", ctypes.c_float * SB_NPARTS), ("ep_worst", ctypes.c_float), ("num_agents", ctypes.c_int),
                ("tag", ctypes.c_int), ("boundary_reached", ctypes.c_int), ("step", ctypes.c_int),
                ("max_steps", ctypes.c_int), ("start_offset", ctypes.c_int), ("start_day", ctypes.c_int),
                ("start_rng", ctypes.c_ulonglong), ("start_draws", ctypes.c_uint), ("n_act", ctypes.c_int),
                ("n_cont", ctypes.c_int), ("n_disc", ctypes.c_int), ("loaded", ctypes.c_int), ("rng", ctypes.c_uint),
                ("seed", ctypes.c_int), ("cont", ctypes.c_void_p), ("disc", ctypes.c_void_p),
                ("native", ctypes.c_void_p), ("env_id", ctypes.c_int), ("scenario", ctypes.c_int)]


class DictItem(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("value", ctypes.c_double), ("str", ctypes.c_char_p)]


class Dict(ctypes.Structure):
    _fields_ = [("items", ctypes.POINTER(DictItem)), ("size", ctypes.c_int), ("capacity", ctypes.c_int)]


class SbGenParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in
                ["rows", "cols", "n_rooms", "n_ahu", "notch_rows", "notch_cols", "dense_walls", "n_steps",
                 "start_doy", "start_hour", "zone_assignment", "conv_distance"]] + \
               [(n, ctypes.c_double) for n in
                ["cv_size_cm", "dt_sec", "t_mean_c", "t_amp_k", "ar_phi", "ar_sigma_k", "conv_p"]] + \
               [("layout_seed", ctypes.c_uint64), ("climate_seed", ctypes.c_uint64),
                ("occ_seed", ctypes.c_int64), ("conv_seed", ctypes.c_int64), ("random_start_days", ctypes.c_int)]


_LIBS: dict[str, ctypes.CDLL] = {}


def _load(name: str) -> ctypes.CDLL:
    if name in _LIBS:
        return _LIBS[name]
    path = PKG / name
    if not path.exists():
        raise RuntimeError(f"{path} is missing: build it with `python -m neurips2026_smart_building_challenge_b200.build`")
    lib = ctypes.CDLL(str(path))
    _LIBS[name] = lib
    return lib


def env_lib() -> ctypes.CDLL:
    lib = _load("libsbenv.so")
    if not getattr(lib, "_sb_typed", False):
        vp, ip, dp = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)
        lib.sb_dict_new.restype = ctypes.POINTER(Dict)
        lib.sb_dict_new.argtypes = [ctypes.c_int]
        lib.sb_dict_free.argtypes = [ctypes.POINTER(Dict)]
        lib.dict_find.restype = ctypes.POINTER(DictItem)
        lib.dict_find.argtypes = [ctypes.POINTER(Dict), ctypes.c_char_p]
        lib.dict_set.argtypes = [ctypes.POINTER(Dict), ctypes.c_char_p, ctypes.c_double]
        lib.dict_set_str.argtypes = [ctypes.POINTER(Dict), ctypes.c_char_p, ctypes.c_char_p]
        lib.puf_vec_create.restype = ctypes.POINTER(EnvRecord)
        lib.puf_vec_create.argtypes = [ctypes.c_int, ctypes.POINTER(Dict), vp, vp, vp, vp]
        lib.puf_bind_stream.argtypes = [vp]
        lib.puf_reset.argtypes = [vp]
        lib.puf_step.argtypes = [vp]
        lib.puf_close.argtypes = [vp]
        lib.puf_log.argtypes = [ctypes.POINTER(Log), ctypes.POINTER(Dict)]
        lib.puf_live_log.argtypes = [vp, ctypes.POINTER(Dict)]
        lib.puf_mask_init.argtypes = [vp, ctypes.c_int, ctypes.c_int]
        lib.sb_last_error.restype = ctypes.c_char_p
        lib.sb_shape.argtypes = [ip]
        lib.sb_env_info.argtypes = [ip, ip]
        lib.sb_get_temp.argtypes = [ctypes.c_int, dp, ctypes.c_int]
        lib.sb_get_mass.argtypes = [ctypes.c_int, dp, ctypes.c_int]
        lib.sb_get_reward_f64.argtypes = [dp, dp]
        lib.sb_debug_state.argtypes = [ctypes.c_int, dp, ctypes.c_int]
        lib.sb_step_timed.argtypes = [ctypes.POINTER(ctypes.c_float)]
        lib.sb_solve_bytes.argtypes = [dp]
        lib.sb_beta_actions.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                        ctypes.c_ulonglong, vp]
        lib.sb_snapshot_write.argtypes = [ctypes.c_int, ctypes.c_char_p]
        lib.sb_episode_options.argtypes = [ip, ctypes.POINTER(ctypes.c_ulonglong)]
        lib.sb_solve_flops.argtypes = [dp]
        lib.sb_fp64_peak.argtypes = [dp]
        lib.sb_scenario_stats.argtypes = [dp, ctypes.c_int]
        lib.sb_test_stall.argtypes = [ctypes.c_int, ctypes.c_uint]
        lib._sb_typed = True
    return lib


def gen_lib() -> ctypes.CDLL:
    lib = _load("libsbgen.so")
    if not getattr(lib, "_sb_typed", False):
        lib.sbgen_preset.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(SbGenParams)]
        lib.sbgen_write.argtypes = [ctypes.c_char_p, ctypes.POINTER(SbGenParams), ctypes.c_char_p, ctypes.c_int]
        lib.sbgen_factor_stats.argtypes = [ctypes.POINTER(SbGenParams)] + [ctypes.POINTER(ctypes.c_int64)] * 3
        lib._sb_typed = True
    return lib


# ----------------------------------------------------------------- scenarios

def preset(config: int, index: int = 0, **overrides) -> SbGenParams:
    """Parameters of one BASELINE-configuration scenario, optionally overridden."""
    p = SbGenParams()
    if gen_lib().sbgen_preset(config, index, ctypes.byref(p)) != 0:
        raise ValueError(f"no preset for config {config} index {index}")
    for k, v in overrides.items():
        if not hasattr(p, k):
            raise KeyError(k)
        setattr(p, k, v)
    return p


def write_scenario(path: str | os.PathLike, params: SbGenParams) -> Path:
    err = ctypes.create_string_buffer(512)
    if gen_lib().sbgen_write(str(path).encode(), ctypes.byref(params), err, 512) != 0:
        raise RuntimeError(f"sbgen_write: {err.value.decode()}")
    return Path(path)


def factor_stats(params: SbGenParams) -> tuple[int, int, int]:
    n, l, u = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    if gen_lib().sbgen_factor_stats(ctypes.byref(params), ctypes.byref(n), ctypes.byref(l), ctypes.byref(u)) != 0:
        raise RuntimeError("sbgen_factor_stats failed")
    return n.value, l.value, u.value


def config_dir(config: int, root: str | os.PathLike | None = None, **overrides) -> Path:
    """Directory of the blobs of a BASELINE configuration (generated once, cached).

    config 1: one scenario; config 2: 30 scenarios named c2_L<layout>__clim<climate>.sbb
    (building-first round robin groups the five climates of a layout); config 3: one scenario.
    """
    root = Path(root or os.environ.get("SB_SCENARIO_CACHE", ROOT / ".sbb_cache"))
    tag = "".join(f"_{k}{v}" for k, v in sorted(overrides.items()))
    d = root / f"config{config}{tag}"
    d.mkdir(parents=True, exist_ok=True)
    count = 30 if config == 2 else 1
    for i in range(count):
        name = f"c2_L{i // 5}__clim{i % 5}.sbb" if config == 2 else f"c{config}__w0.sbb"
        path = d / name
        if not path.exists():
            write_scenario(path, preset(config, i, **overrides))
    return d


# ----------------------------------------------------------------- the env

class SmartBuildingsVec:
    """n envs on one GPU behind the PufferLib GPU-backend ABI.

    obs / actions / rewards / terminals are device tensors owned here and handed
    to the native env exactly as the trainer's buffers would be.
    """

    def __init__(self, n: int, blob: str | None = None, blob_dir: str | None = None, device: str = "cuda:0",
                 **kwargs):
        import torch

        if not torch.cuda.is_available():
            raise RuntimeError("SmartBuildingsVec needs a CUDA device (no CPU fallback)")
        self.torch = torch
        self.lib = env_lib()
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        self.n = n
        self.obs = torch.zeros(n, SB_OBS, dtype=torch.float32, device=self.device)
        self.actions = torch.zeros(n, SB_NUM_ATNS, dtype=torch.float32, device=self.device)
        self.rewards = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.terminals = torch.zeros(n, dtype=torch.float32, device=self.device)
        kw = self.lib.sb_dict_new(16)
        try:
            if blob:
                self.lib.dict_set_str(kw, b"blob", str(blob).encode())
            if blob_dir:
                self.lib.dict_set_str(kw, b"blob_dir", str(blob_dir).encode())
            for k, v in kwargs.items():
                self.lib.dict_set(kw, k.encode(), float(v))
            torch.cuda.synchronize(self.device)
            ptr = self.lib.puf_vec_create(n, kw, self.obs.data_ptr(), self.actions.data_ptr(),
                                          self.rewards.data_ptr(), self.terminals.data_ptr())
        finally:
            self.lib.sb_dict_free(kw)
        if not ptr:
            raise RuntimeError(f"puf_vec_create: {self.lib.sb_last_error().decode()}")
        self._envs_ptr = ptr
        self.records = ctypes.cast(ptr, ctypes.POINTER(EnvRecord * n)).contents
        shp = (ctypes.c_int * 8)()
        self.lib.sb_shape(shp)
        self.shape = list(shp)
        ol = (ctypes.c_int * n)()
        sc = (ctypes.c_int * n)()
        self.lib.sb_env_info(ol, sc)
        self.obs_len = np.array(ol[:], dtype=np.int64)
        self.scenario = np.array(sc[:], dtype=np.int64)
        self.closed = False
        # every launch of the env goes to this stream (puf_bind_stream)
        self.stream = torch.cuda.Stream(device=self.device)
        self.bind_stream(self.stream)

    # -- PufferLib entry points
    def bind_stream(self, stream) -> None:
        self.lib.puf_bind_stream(ctypes.c_void_p(stream.cuda_stream))

    def reset(self) -> None:
        self.lib.puf_reset(self._envs_ptr)
        self._check()

    def step(self, actions=None) -> None:
        """One puf_step on the env stream; `actions` (if given) is copied in first on that stream."""
        if actions is not None:
            self.stream.wait_stream(self.torch.cuda.current_stream(self.device))
            with self.torch.cuda.stream(self.stream):
                self.actions.copy_(actions, non_blocking=True)
        self.lib.puf_step(self._envs_ptr)

    def synchronize(self) -> None:
        self.stream.synchronize()

    def mask(self, width: int = SB_MASK_WIDTH):
        m = self.torch.zeros(self.n, width, dtype=self.torch.uint8, device=self.device)
        self.lib.puf_mask_init(ctypes.c_void_p(m.data_ptr()), width, self.n)
        self._check()
        return m

    def log(self) -> dict:
        """Sum of every env's Log, written through puf_log (the trainer's aggregation)."""
        self.torch.cuda.synchronize(self.device)
        agg = Log()
        for f in LOG_FIELDS:
            setattr(agg, f, float(sum(getattr(r.log, f) for r in self.records)))
        d = self.lib.sb_dict_new(16)
        try:
            self.lib.puf_log(ctypes.byref(agg), d)
            return _dict_to_py(d)
        finally:
            self.lib.sb_dict_free(d)

    def live_log(self) -> dict:
        d = self.lib.sb_dict_new(64)
        try:
            self.lib.puf_live_log(self._envs_ptr, d)
            return _dict_to_py(d)
        finally:
            self.lib.sb_dict_free(d)

    # -- inspection (host copies)
    def temp(self, env: int, n_cvs: int) -> np.ndarray:
        out = np.zeros(n_cvs)
        if self.lib.sb_get_temp(env, out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), n_cvs) != 0:
            raise RuntimeError("sb_get_temp failed")
        return out

    def mass(self, env: int, n_solved: int) -> np.ndarray:
        out = np.zeros(n_solved)
        if self.lib.sb_get_mass(env, out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), n_solved) != 0:
            raise RuntimeError("sb_get_mass failed")
        return out

    def reward_f64(self) -> tuple[np.ndarray, np.ndarray]:
        r = np.zeros(self.n)
        p = np.zeros((self.n, SB_NPARTS))
        if self.lib.sb_get_reward_f64(r.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                                      p.ctypes.data_as(ctypes.POINTER(ctypes.c_double))) != 0:
            raise RuntimeError("sb_get_reward_f64 failed")
        return r, p

    def snapshot(self, env: int, path) -> None:
        """Writes env `env`'s visible state after the last step to an SBS1 file (`read_snapshot`)."""
        if self.lib.sb_snapshot_write(env, str(path).encode()) != 0:
            raise RuntimeError(self.lib.sb_last_error().decode())

    def episode_options(self) -> tuple[np.ndarray, np.ndarray]:
        """Per env: the first episode's length (desync) and the random-start
        stream's state before its first draw."""
        fl = (ctypes.c_int * self.n)()
        sr = (ctypes.c_ulonglong * self.n)()
        if self.lib.sb_episode_options(fl, sr) != 0:
            raise RuntimeError("sb_episode_options failed")
        return np.array(fl[:], dtype=np.int64), np.array(sr[:], dtype=np.uint64)

    def status(self) -> int:
        return int(self.lib.sb_device_status())

    def step_timed(self) -> dict:
        """One step with CUDA events around each kernel (diagnostic; not capturable)."""
        ms = (ctypes.c_float * 7)()
        if self.lib.sb_step_timed(ms) != 0:
            raise RuntimeError("sb_step_timed failed")
        # the next transition's k_conv + k_occ run beside phase 1 and have no time of their own (-1)
        names = ["random_inputs", "k_pre", "k_solve", "k_post", "k_solve_phase0", "k_dense", "k_solve_phase1"]
        return {k: v for k, v in zip(names, list(ms)) if v >= 0.0}

    def solve_bytes(self) -> float:
        b = ctypes.c_double()
        if self.lib.sb_solve_bytes(ctypes.byref(b)) != 0:
            raise RuntimeError("sb_solve_bytes failed")
        return b.value

    def solve_flops(self) -> float:
        f = ctypes.c_double()
        if self.lib.sb_solve_flops(ctypes.byref(f)) != 0:
            raise RuntimeError("sb_solve_flops failed")
        return f.value

    def scenario_stats(self, clear: bool = False) -> np.ndarray:
        """[n_scenarios][6] episode-statistics sums (dist.STAT_KEYS order)."""
        out = np.zeros((self.shape[1], 6))
        if self.lib.sb_scenario_stats(out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), 1 if clear else 0) < 0:
            raise RuntimeError("sb_scenario_stats failed")
        return out

    def _check(self) -> None:
        err = self.lib.sb_last_error().decode()
        if err:
            raise RuntimeError(err)

    def close(self) -> None:
        if not self.closed:
            self.lib.puf_close(self._envs_ptr)
            self.closed = True

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def fp64_peak_tflops() -> float:
    """Measured fp64 issue rate of the current GPU (libsbenv's probe kernel)."""
    t = ctypes.c_double()
    if env_lib().sb_fp64_peak(ctypes.byref(t)) != 0:
        raise RuntimeError(env_lib().sb_last_error().decode())
    return t.value


def _dict_to_py(d) -> dict:
    out = {}
    dd = d.contents
    for i in range(dd.size):
        it = dd.items[i]
        out[it.key.decode()] = it.str.decode() if it.str else it.value
    return out
