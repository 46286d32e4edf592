"""Policy-in-loop rollouts.

A random-init shared MLP policy in PyTorch (observation -> 128 tanh -> 128 tanh
-> two logit blocks of 288 columns) feeds the library's action sampler
(`sb_beta_actions`: Beta heads with alpha, beta = softplus + floor and the
concentration capped, categorical discrete heads, the env's action mask), whose
actions the env steps on (`puf_step`). The logit layout, the Beta map and the
cap follow the reference trainer (patches/pufferlib_core.diff:2490-2580,
config/smart_buildings.ini beta_floor = 1, beta_conc_max = 12 in the run this
configuration names).

One env+policy step (the policy's GEMMs, the sampler, the env's kernels and
the draw counter's increment) is captured in a CUDA graph on the env's bound
stream and replayed over the rollout horizon, as the reference trainer captures
its rollout step.
"""
from __future__ import annotations

from . import SB_MASK_WIDTH, SB_OBS, SmartBuildingsVec


class ZonePolicy:
    """Shared MLP over the observation, random init from a seed (f32).

    `forward(obs, out)` writes the two logit blocks into `out` [2][n][288]."""

    def __init__(self, device, hidden: int = 128, seed: int = 0, obs: int = SB_OBS, width: int = SB_MASK_WIDTH):
        import torch

        g = torch.Generator().manual_seed(seed)

        def lin(i, o):
            bound = 1.0 / i ** 0.5
            w = (torch.rand(o, i, generator=g) * 2 - 1) * bound
            b = (torch.rand(o, generator=g) * 2 - 1) * bound
            return w.to(device), b.to(device)

        self.torch = torch
        self.w1, self.b1 = lin(obs, hidden)
        self.w2, self.b2 = lin(hidden, hidden)
        self.wu, self.bu = lin(hidden, width)
        self.wv, self.bv = lin(hidden, width)

    def forward(self, obs, out) -> None:
        torch = self.torch
        h = torch.tanh(torch.addmm(self.b1, obs, self.w1.t()))
        h = torch.tanh(torch.addmm(self.b2, h, self.w2.t()))
        torch.addmm(self.bu, h, self.wu.t(), out=out[0])
        torch.addmm(self.bv, h, self.wv.t(), out=out[1])


class Rollout:
    """Env + policy steps; `graph=True` captures one step and replays it.

    `call` is the device draw counter the sampler reads; each step advances it,
    so replays draw fresh numbers. Steps run on the env's stream."""

    def __init__(self, env: SmartBuildingsVec, policy: ZonePolicy, seed: int = 0, beta_floor: float = 1.0,
                 beta_cap: float = 12.0, graph: bool = True, masked: bool = True):
        import torch

        self.env, self.policy, self.torch = env, policy, torch
        self.seed, self.floor, self.cap = seed, beta_floor, beta_cap
        self.call = torch.zeros(1, dtype=torch.int64, device=env.device)
        self.raw = torch.zeros(2, env.n, SB_MASK_WIDTH, dtype=torch.float32, device=env.device)
        self.mask = env.mask() if masked else None
        torch.cuda.synchronize(env.device)
        self.graph = None
        if graph:
            # a policy forward first (lazy cuBLAS init; the env does not step), then the capture
            with torch.cuda.stream(env.stream):
                policy.forward(env.obs, self.raw)
            env.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=env.stream):
                self._step_body()
            env.synchronize()

    def _step_body(self) -> None:
        env = self.env
        self.policy.forward(env.obs, self.raw)
        mask = self.mask.data_ptr() if self.mask is not None else None
        if env.lib.sb_beta_actions(self.raw.data_ptr(), mask, env.actions.data_ptr(), env.n, self.floor, self.cap,
                                   self.seed, self.call.data_ptr()) != 0:
            raise RuntimeError(env.lib.sb_last_error().decode())
        env.lib.puf_step(env._envs_ptr)
        self.call.add_(1)

    def step(self) -> None:
        with self.torch.cuda.stream(self.env.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._step_body()

    def run(self, horizon: int) -> None:
        for _ in range(horizon):
            self.step()
