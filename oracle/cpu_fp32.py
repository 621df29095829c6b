"""CPU baseline: the reference's FP32 eager GLAD actor forward on the host
cores (test/benchmark infrastructure only).

Restates ``ActorCriticEncoder.act_inference`` in FP32 eager PyTorch on the
CPU (rsl_rl/modules/actor_critic_encoder.py:342-350), using the package's
GLAD module, which reproduces the reference's parameter names, init order
and float forward. This is the reference's own CPU-capable path for the
GLAD forward; qrt's INT8 path has no CPU implementation (its conv kernels
are Triton GPU kernels).
"""
from __future__ import annotations

import os
import time

import torch


def time_fp32_forward(batch: int = 256, budget_s: float = 12.0, threads: int | None = None,
                      min_reps: int = 5, max_reps: int | None = None, seed: int = 0) -> dict:
    """Median seconds per forward of ``batch`` envs, and env-obs/s."""
    from rl_quant_b200.glad_model import build_glad
    from rl_quant_b200.synthetic import glad_obs

    threads = threads or os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        model = build_glad(seed=seed, critic_seed=2, dtype=torch.float32, device="cpu").eval()
        obs = glad_obs(batch, seed=1234)
        times = []
        with torch.inference_mode():
            for _ in range(2):
                model.act_inference(obs)
            t_end = time.perf_counter() + budget_s
            while True:
                t0 = time.perf_counter()
                model.act_inference(obs)
                times.append(time.perf_counter() - t0)
                if max_reps and len(times) >= max_reps:
                    break
                if len(times) >= min_reps and time.perf_counter() > t_end:
                    break
    finally:
        torch.set_num_threads(prev)
    times.sort()
    med = times[len(times) // 2]
    return {"sec_per_step": med, "obs_per_s": batch / med, "reps": len(times), "threads": threads,
            "batch": batch}
