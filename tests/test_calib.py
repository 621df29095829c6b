"""Calibration pinned to the reference (CPU).

tests/golden/glad_calib.npz holds what qrt's own ``calib.make_plan``
(qrt/calib.py:93-129 with quant/let.py:140-233) returned when run with torch's
global generator seeded, on an fp16 copy of this package's GLAD module, on two
batches of seeded synthetic observations (make_golden.py, ``calib_golden``).
The package's ``make_plan`` with the same seed on the same model and batches
picks the same rows, so every alpha, beta and s_z must be identical, not close.
"""
import os

import numpy as np
import pytest
import torch

from rl_quant_b200 import calib
from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.synthetic import glad_obs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "glad_calib.npz")
PATHS = ["actor.0", "actor.2", "actor.4", "actor.6", "actor_proprio_embedding", "query_projector"]


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def _batches(g):
    rows, n = int(g["meta.rows"]), int(g["meta.batches"])
    obs = glad_obs(n * rows, seed=int(g["meta.obs_seed"])).half()
    return [{"policy_obs": obs[i * rows:(i + 1) * rows]} for i in range(n)]


def test_make_plan_equals_reference_plan(golden):
    torch.set_num_threads(max(1, min(8, os.cpu_count() or 1)))
    model = build_glad(seed=0, critic_seed=2).half().eval()
    it = iter(_batches(golden))
    plan = calib.make_plan(model, PATHS, obs_fn=lambda: next(it), n_calib=int(golden["meta.batches"]),
                           use_let=True, let_steps=int(golden["meta.steps"]), act_mode="dynamic",
                           verbose=False, seed=int(golden["meta.seed"]))
    assert list(plan) == PATHS
    for p in PATHS:
        assert plan[p]["act_mode"] == "dynamic"
        np.testing.assert_array_equal(plan[p]["alpha"].numpy(), golden[f"{p}.alpha"], err_msg=p)
        np.testing.assert_array_equal(plan[p]["beta"].numpy(), golden[f"{p}.beta"], err_msg=p)
        assert plan[p]["s_z"] == float(golden[f"{p}.s_z"]), p


def test_plan_without_let_and_dynamic_full(golden):
    model = build_glad(seed=0, critic_seed=2).half().eval()
    batches = _batches(golden)
    it = iter(batches)
    plan = calib.make_plan(model, PATHS[:2], obs_fn=lambda: next(it), n_calib=len(batches), use_let=False,
                           verbose=False)
    rows = calib.record_inputs(model, PATHS[:2], iter(batches).__next__, len(batches), torch.Generator())
    for p in PATHS[:2]:
        assert plan[p]["alpha"] is None and plan[p]["beta"] is None
        assert plan[p]["s_z"] == rows[p].abs().amax().item() / 127.0
    full = calib.make_plan(model, PATHS, act_mode="dynamic_full")
    assert all(v == {"s_z": None, "alpha": None, "beta": None, "act_mode": "dynamic_full"} for v in full.values())
