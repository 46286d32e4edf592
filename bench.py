#!/usr/bin/env python3
"""Benchmark: fp64 building-steps/s of the batched Smart Buildings env step on B200.

Workload (the metric's configuration): 960 synthetic buildings
per GPU -- six seeded layouts of 41-81 zones with 1-4 AHUs, each paired with five
synthetic climates, 32 envs per scenario -- driven with seeded Beta(a, b) actions,
a, b ~ U(0.5, 12) per env and head (the trainer's 2x-1 Beta contract), run bits on.
One step = one puf_step of every env (decode, HVAC, fp64 thermal solve with the
air side, convection, occupancy, observation, reward, episode log).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    python bench.py --rollout [--gpus N --steps K --warmup W]

--rollout measures BASELINE configuration 5 instead: the end-to-end env+policy
step rate of policy-in-loop rollouts (a random-init shared MLP, hidden 128, tanh,
in PyTorch; Beta heads with floor 1 and concentration cap 12 drawn by the
library's sampler; one env+policy step captured in a CUDA graph and replayed
over 128-step rollout horizons), 960 envs per GPU.

N > 1 is launched with torch.distributed.run: every rank owns a disjoint slice of
960 envs (weak scaling, no per-step collective); episode statistics are summed
over ranks with one NCCL all-reduce after the timed region.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fp64 building-steps/s"
UNIT = "building-steps/s"
ENVS_PER_GPU = 960
WORKLOAD = ("config2: 960 synthetic buildings per GPU = 6 seeded layouts (41-81 zones, 1-4 AHUs, "
            "64x48 grid) x 5 climates x 32 envs; seeded Beta(a,b) actions, a,b~U(0.5,12)")
SMI_Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--envs", type=int, default=ENVS_PER_GPU, help="envs per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rollout", action="store_true", help="configuration 5: env+policy steps in a CUDA graph")
    ap.add_argument("--horizon", type=int, default=128, help="rollout horizon (--rollout)")
    ap.add_argument("--solve", default="exact", choices=["exact", "folded"],
                    help="exact: the reference core's two triangular solves, bit for bit; folded: one L/U "
                         "pair (the reference GPU backend's folded air side, 1e-9 per-step contract)")
    return ap.parse_args()


# ---------------------------------------------------------------- clocks

class ClockSampler:
    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.f = None

    def __enter__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={SMI_Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.f.name):
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU side

def _cpu_worker(args):
    """Steps a slice of envs on the CPU oracle (the reference C core when present)."""
    lib_kind, blobs, n_steps, seconds, seed = args
    sys.path.insert(0, str(ROOT / "tests"))
    from oracle_util import PORT, REF, OracleEnv, actions

    path = REF if lib_kind == "reference" else PORT
    envs = [OracleEnv(b, path=path) for b in blobs]
    for e in envs:
        e.reset()
    rng = np.random.default_rng(seed)
    acts = [actions(rng, 1, e.n_cont, e.n_disc, wild=False)[0] for e in envs]
    steps = 0
    per_step = []
    t0 = time.perf_counter()
    while True:
        ts = time.perf_counter()
        for e, a in zip(envs, acts):
            e.step(a)
        per_step.append(time.perf_counter() - ts)
        steps += 1
        if (n_steps and steps >= n_steps) or (not n_steps and time.perf_counter() - t0 >= seconds):
            break
    return steps * len(envs), time.perf_counter() - t0, per_step


def cpu_kind() -> str:
    return "reference" if (ROOT / "oracle" / "_ref" / "libcsimref.so").exists() else "port"


def blob_list(cache: Path, n_env: int) -> list[Path]:
    from neurips2026_smart_building_challenge_b200 import config_dir

    d = config_dir(2, cache)
    scen = sorted(d.glob("*.sbb"))
    return [scen[i % len(scen)] for i in range(n_env)]


def cpu_baseline(cache: Path, seconds: float = 12.0) -> dict:
    """Bounded sample: every host core steps one env of a different config-2 scenario for ~12 s."""
    cores = os.cpu_count() or 1
    blobs = blob_list(cache, 30)
    work = [(cpu_kind(), [blobs[i % 30]], 0, seconds, i) for i in range(cores)]
    with mp.get_context("spawn").Pool(cores) as pool:
        res = pool.map(_cpu_worker, work)
    steps = sum(r[0] for r in res)
    wall = max(r[1] for r in res)
    return {"value": steps / wall, "unit": UNIT, "cores": cores, "kind": cpu_kind(),
            "sample": f"{cores} processes x 1 env (config-2 scenarios round robin), ~{seconds:.0f} s each, "
                      f"{steps} env-steps"}


def run_reference(args) -> None:
    """Reference arm: the reference's own C core stepping the same 960-env workload on all host cores."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cache = ROOT / ".sbb_cache" / "bench"
    blobs = blob_list(cache, args.envs)
    cores = min(os.cpu_count() or 1, args.envs)
    slices = [blobs[i::cores] for i in range(cores)]
    total = args.warmup + args.steps
    work = [(cpu_kind(), s, total, 0.0, i) for i, s in enumerate(slices)]
    with mp.get_context("spawn").Pool(cores) as pool:
        res = pool.map(_cpu_worker, work)
    # a step ends when the slowest core finishes its slice
    per_step = np.max(np.array([r[2] for r in res]), axis=0)[args.warmup:]
    ms = float(per_step.sum() / len(per_step) * 1e3)
    value = args.envs / (ms / 1e3)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "envs": args.envs},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": cpu_kind(),
                             "sample": f"{args.envs} envs over {cores} processes, {args.steps} timed steps"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU side

def action_pool(n: int, n_batches: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    a = rng.uniform(0.5, 12.0, size=(n, 256))
    b = rng.uniform(0.5, 12.0, size=(n, 256))
    out = np.zeros((n_batches, n, 272), np.float32)
    for i in range(n_batches):
        out[i, :, :256] = 2.0 * rng.beta(a, b) - 1.0
        out[i, :, 256:] = 1.0
    return out


def profile_traffic() -> float | None:
    """DRAM bytes per solve launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "k_solve_config2_960.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class E2EPipe:
    """One env step per call with its host copies: H2D of the step's actions into a
    device staging slot on one copy stream, a device copy into the env's action buffer
    and puf_step on the env stream, a device copy of obs/rewards/terminals into an
    output slot, D2H of that slot on a second copy stream. Two slots of each, so the
    copies of steps i-1 and i+1 overlap step i's kernels."""

    def __init__(self, env, h_act, torch):
        self.env, self.h_act, self.torch = env, h_act, torch
        n, dev = env.n, env.device
        self.cin = torch.cuda.Stream(device=dev)
        self.cout = torch.cuda.Stream(device=dev)
        self.d_act = [torch.empty(n, 272, dtype=torch.float32, device=dev) for _ in range(2)]
        self.d_out = [(torch.empty(n, 1024, dtype=torch.float32, device=dev),
                       torch.empty(n, dtype=torch.float32, device=dev),
                       torch.empty(n, dtype=torch.float32, device=dev)) for _ in range(2)]
        self.h_out = [tuple(t.cpu().pin_memory() for t in o) for o in self.d_out]
        E = torch.cuda.Event
        self.ev_in, self.ev_used, self.ev_out, self.ev_host = ([E() for _ in range(2)] for _ in range(4))
        self.started = [False, False]

    def start_after(self, ev) -> None:
        self.cin.wait_event(ev)

    def step(self, i: int) -> None:
        torch, env, k = self.torch, self.env, i % 2
        s = env.stream
        with torch.cuda.stream(self.cin):
            if self.started[k]:
                self.cin.wait_event(self.ev_used[k])
            self.d_act[k].copy_(self.h_act[k], non_blocking=True)
            self.ev_in[k].record(self.cin)
        s.wait_event(self.ev_in[k])
        with torch.cuda.stream(s):
            env.actions.copy_(self.d_act[k], non_blocking=True)
            self.ev_used[k].record(s)
        env.step()
        with torch.cuda.stream(s):
            if self.started[k]:
                s.wait_event(self.ev_host[k])
            for dst, src in zip(self.d_out[k], (env.obs, env.rewards, env.terminals)):
                dst.copy_(src, non_blocking=True)
            self.ev_out[k].record(s)
        with torch.cuda.stream(self.cout):
            self.cout.wait_event(self.ev_out[k])
            for dst, src in zip(self.h_out[k], self.d_out[k]):
                dst.copy_(src, non_blocking=True)
            self.ev_host[k].record(self.cout)
        self.started[k] = True


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # the CPU baseline's process pool starts before the first GPU call (spawned)
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(ROOT / ".sbb_cache" / "bench")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec, config_dir, env_lib

    cache = ROOT / ".sbb_cache" / f"bench_rank{rank}"
    d = config_dir(2, cache)
    n = args.envs
    env = SmartBuildingsVec(n, blob_dir=str(d), groups=30, device=f"cuda:{local}",
                            solve_exact=1 if args.solve == "exact" else 0)
    env.reset()
    pool = torch.from_numpy(action_pool(n, 8, seed=1234 + rank)).to(env.device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=env.device)   # > 126 MB L2
    s = env.stream

    def one_step(i):
        with torch.cuda.stream(s):
            env.actions.copy_(pool[i % len(pool)], non_blocking=True)
            flush.fill_(i & 0xFF)

    for i in range(args.warmup):
        one_step(i)
        env.step()
    env.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            one_step(i)
            starts[i].record(s)
            env.step()
            ends[i].record(s)
        env.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_local = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    ms_t = torch.tensor([ms_local], dtype=torch.float64, device=env.device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_total = float(ms_t.item())
    ms_per_step = ms_total / args.steps
    value = world * n * args.steps / (ms_total / 1e3)
    status = env.status()

    # per-kernel durations (diagnostic steps after the timed region)
    kt = {}
    for i in range(5):
        one_step(i)
        env.synchronize()
        for k, v in env.step_timed().items():
            kt.setdefault(k, []).append(v)
    k_ms = {k: float(np.mean(v)) for k, v in kt.items()}
    bytes_launch = env.solve_bytes()
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    achieved = bytes_launch / (k_ms["k_solve"] / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": profile_traffic(), "kernel": "k_solve", "peak_source": peak_src,
                "kernel_ms": k_ms["k_solve"], "algorithmic_bytes_per_launch": bytes_launch,
                "per_kernel_ms": k_ms}

    # end to end through the C ABI: pinned host actions in, obs/rewards/terminals out, every
    # step; the copies run on two copy streams (double-buffered device staging) and overlap
    # the neighbouring steps' kernels, as a trainer feeding the env would run them
    h_act = torch.from_numpy(action_pool(n, 2, seed=99 + rank)).pin_memory()
    e_steps = max(3, min(args.steps, 20))
    pipe = E2EPipe(env, h_act, torch)
    for i in range(2):
        pipe.step(i)
    env.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    pipe.start_after(e0)
    for i in range(e_steps):
        pipe.step(i)
    s.wait_stream(pipe.cout)
    e1.record(s)
    env.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=env.device)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = {"value": world * n * e_steps / (float(e_ms.item()) / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": n * 272 * 4, "d2h_bytes_per_step": n * (1024 + 2) * 4,
           "copies": "pinned host buffers, two copy streams overlapping the kernels"}

    # episode statistics gathered over ranks (the path's only collective)
    live = env.live_log()
    stats = torch.tensor([live.get("live/reward", 0.0), live.get("live/comfort_dev_K", 0.0), 1.0],
                         dtype=torch.float64, device=env.device)
    if world > 1:
        dist.all_reduce(stats)
    launches = env_lib().sb_kernels_per_step() * args.steps
    env.close()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": {"workload": WORKLOAD, "envs_per_gpu": n, "total_envs": n * world, "solve": args.solve,
                           "l2": "flushed between timed steps (256 MiB write, untimed)",
                           "parallelism": f"env-sharded x{world}, no per-step collective"},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk.summary(), "device_status": status,
                "episode_stats_allreduce": {"mean_live_reward": float(stats[0] / stats[2])}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


ROLLOUT_METRIC = "env+policy building-steps/s"
ROLLOUT_WORKLOAD = ("config5: policy-in-loop rollouts, 960 envs per GPU over the config-2 scenario mix; "
                    "random-init shared MLP 1024-128-128 tanh (f32, PyTorch) -> Beta heads (floor 1, cap 12) "
                    "+ categorical discrete heads drawn by the library sampler; one env+policy step per CUDA "
                    "graph replay, 128-step horizons")


def run_rollout(args) -> None:
    """Configuration 5: timed env+policy steps (graph replays), horizons of args.horizon steps."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
    from neurips2026_smart_building_challenge_b200 import SmartBuildingsVec, config_dir
    from neurips2026_smart_building_challenge_b200.rollout import Rollout, ZonePolicy

    d = config_dir(2, ROOT / ".sbb_cache" / f"bench_rank{rank}")
    n = args.envs
    env = SmartBuildingsVec(n, blob_dir=str(d), groups=30, device=f"cuda:{local}")
    env.reset()
    ro = Rollout(env, ZonePolicy(env.device, seed=17), seed=1000 + rank, beta_floor=1.0, beta_cap=12.0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=env.device)   # > 126 MB L2
    s = env.stream
    for i in range(args.warmup):
        ro.step()
    env.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            if i % args.horizon == 0:
                env.reset()   # a new rollout: every env restarts its episode (untimed)
            with torch.cuda.stream(s):
                flush.fill_(i & 0xFF)
            starts[i].record(s)
            ro.step()
            ends[i].record(s)
        env.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_t = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, ends))], dtype=torch.float64,
                        device=env.device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_total = float(ms_t.item())
    value = world * n * args.steps / (ms_total / 1e3)

    # end to end through the public API: graph replay + rewards and terminals read back every step
    h_rew = torch.empty(n, dtype=torch.float32).pin_memory()
    h_term = torch.empty(n, dtype=torch.float32).pin_memory()
    e_steps = max(3, min(args.steps, 64))
    env.reset()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(e_steps):
        ro.step()
        with torch.cuda.stream(s):
            h_rew.copy_(env.rewards, non_blocking=True)
            h_term.copy_(env.terminals, non_blocking=True)
    e1.record(s)
    env.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=env.device)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = {"value": world * n * e_steps / (float(e_ms.item()) / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": n * 2 * 4}
    status = env.status()
    k_ms = {}
    for _ in range(3):
        for k, v in env.step_timed().items():
            k_ms.setdefault(k, []).append(v)
    k_ms = {k: float(np.mean(v)) for k, v in k_ms.items()}
    launches = (env.lib.sb_kernels_per_step() + 1) * args.steps   # the env's kernels + the sampler
    env.close()
    if rank == 0:
        line = {"metric": ROLLOUT_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f64 env, f32 policy", "data": "synthetic",
                "config": {"workload": ROLLOUT_WORKLOAD, "envs_per_gpu": n, "total_envs": n * world,
                           "horizon": args.horizon, "l2": "flushed between timed steps (256 MiB write, untimed)",
                           "parallelism": f"env-sharded x{world}, no per-step collective"},
                "env_kernel_ms": k_ms, "e2e": e2e, "gpu_launches": launches, "clocks": clk.summary(),
                "device_status": status}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.rollout:
        run_rollout(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
