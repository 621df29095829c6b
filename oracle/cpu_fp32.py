"""CPU baseline: the reference's FP32 eager GLAD actor forward on the host
cores (test/benchmark infrastructure only).

Restates ``ActorCriticEncoder.act_inference`` in FP32 eager PyTorch on the
CPU (rsl_rl/modules/actor_critic_encoder.py:342-350), using the package's
GLAD module, which reproduces the reference's parameter names, init order
and float forward: its means, values and top-k indices equal the reference's
own FP32 outputs bit for bit (tests/test_cpu_fp32.py against the goldens the
reference produced). This is the reference's own CPU-capable path for the
GLAD forward; qrt's INT8 path has no CPU implementation (its conv kernels
are Triton GPU kernels).
"""
from __future__ import annotations

import os
import time

import torch


class Fp32Forward:
    """The FP32 eager GLAD actor forward of one ``batch`` of synthetic observations
    on ``threads`` host threads (all of them by default), built once."""

    def __init__(self, batch: int = 256, threads: int | None = None, seed: int = 0):
        from rl_quant_b200.glad_model import build_glad
        from rl_quant_b200.synthetic import glad_obs

        self.batch = batch
        self.threads = threads or os.cpu_count() or 1
        self.model = build_glad(seed=seed, critic_seed=2, dtype=torch.float32, device="cpu").eval()
        self.obs = glad_obs(batch, seed=1234)

    def run(self, n: int) -> float:
        """Seconds that ``n`` forwards take back to back."""
        prev = torch.get_num_threads()
        torch.set_num_threads(self.threads)
        try:
            with torch.inference_mode():
                t0 = time.perf_counter()
                for _ in range(n):
                    self.model.act_inference(self.obs)
                return time.perf_counter() - t0
        finally:
            torch.set_num_threads(prev)

    def forwards_for(self, seconds: float) -> int:
        """How many forwards take about ``seconds`` (measured on a short run)."""
        self.run(2)
        t = self.run(3) / 3
        return max(1, int(round(seconds / max(t, 1e-6))))


def time_fp32_forward(batch: int = 256, budget_s: float = 12.0, threads: int | None = None,
                      seed: int = 0) -> dict:
    """Throughput of ``budget_s`` seconds of back-to-back forwards after a warm-up:
    env-obs/s over the whole timed region and its seconds per forward."""
    f = Fp32Forward(batch, threads, seed)
    f.run(max(1, f.forwards_for(1.0)))                       # about a second of warm-up
    n = f.forwards_for(budget_s)
    dt = f.run(n)
    return {"sec_per_step": dt / n, "obs_per_s": batch * n / dt, "reps": n, "threads": f.threads,
            "batch": batch}
