"""The timed CPU baseline computes the reference's FP32 forward exactly (CPU).

oracle/cpu_fp32.py times the package's GLAD module in FP32 eager PyTorch as the
reference's own CPU path (rsl_rl/modules/actor_critic_encoder.py:342-350). The
goldens carry that path's outputs as the reference produced them (fp32.mean,
fp32.value, fp32.topk_idx; tests/golden/make_golden.py): the timed module must
reproduce them bit for bit.
"""
import numpy as np
import pytest
import torch

from oracle.cpu_fp32 import Fp32Forward
from rl_quant_b200.glad_model import build_glad


@pytest.mark.parametrize("B", [1, 3, 16])
def test_fp32_forward_equals_reference_outputs(golden_fwd, B):
    d = golden_fwd[B]
    m = build_glad(seed=0, critic_seed=2, dtype=torch.float32, device="cpu").eval()
    with torch.inference_mode():
        mean, _, idx, _ = m.act_inference({"policy_obs": torch.from_numpy(d["policy_obs"])})
        value = m.evaluate({"critic_obs": torch.from_numpy(d["critic_obs"])})
    assert np.array_equal(mean.numpy(), d["fp32.mean"])
    assert np.array_equal(idx.numpy(), d["fp32.topk_idx"])
    assert np.array_equal(value.numpy(), d["fp32.value"])


def test_timed_forward_runs():
    f = Fp32Forward(batch=4, threads=1)
    assert f.run(1) > 0.0 and f.forwards_for(0.01) >= 1
