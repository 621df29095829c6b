"""Seeded synthetic GLAD observations.

The reference measures on no public dataset: its benches draw random
observations (``qrt/bench/_common.py:88-123``). This module builds the
stand-in workload used by the tests and the benchmark:

* columns ``[0, P)`` are proprioception, ``N(0, 1)``;
* columns ``[P, P + 2079)`` are the height-map scan in the memory order the
  encoder reshapes it with (``rsl_rl/modules/actor_critic_encoder.py:208-209``):
  ``[W=21][L=33][xyz]``.  ``x`` is an evenly spaced grid ``linspace(-1, 1, 33)``
  along ``L``, ``y`` is ``linspace(-1, 1, 21)`` along ``W`` and the height
  ``z`` is ``N(0, 0.3^2)``.

Everything is drawn from a CPU ``torch.Generator`` so the values do not depend
on the device the caller later moves them to.
"""
from __future__ import annotations

import torch

MAP_L, MAP_W, MAP_C = 33, 21, 3
MAP_SIZE = MAP_L * MAP_W * MAP_C          # 2079
ACTOR_PROPRIO = 96
CRITIC_PROPRIO = 99
NUM_ACTIONS = 29


def height_map(batch: int, gen: torch.Generator) -> torch.Tensor:
    """``[batch, 2079]`` fp32 scan in ``[W][L][xyz]`` order."""
    xs = torch.linspace(-1.0, 1.0, MAP_L)
    ys = torch.linspace(-1.0, 1.0, MAP_W)
    yy, xx = torch.meshgrid(ys, xs, indexing="ij")            # [W, L]
    z = torch.randn(batch, MAP_W, MAP_L, generator=gen) * 0.3
    scan = torch.stack([xx.expand(batch, -1, -1), yy.expand(batch, -1, -1), z], dim=-1)
    return scan.reshape(batch, MAP_SIZE).contiguous()


def glad_obs(batch: int, seed: int, proprio_dim: int = ACTOR_PROPRIO) -> torch.Tensor:
    """One observation group ``[batch, proprio_dim + 2079]`` fp32 on the CPU."""
    gen = torch.Generator().manual_seed(int(seed))
    proprio = torch.randn(batch, proprio_dim, generator=gen)
    return torch.cat([proprio, height_map(batch, gen)], dim=1).contiguous()


def glad_obs_pair(batch: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Actor and critic groups that share the same scan.

    The critic group carries three more proprio columns in front of the scan,
    as in ``qrt/bench/_common.py:60``.
    """
    gen = torch.Generator().manual_seed(int(seed))
    proprio = torch.randn(batch, CRITIC_PROPRIO, generator=gen)
    scan = height_map(batch, gen)
    actor = torch.cat([proprio[:, :ACTOR_PROPRIO], scan], dim=1).contiguous()
    critic = torch.cat([proprio, scan], dim=1).contiguous()
    return actor, critic
