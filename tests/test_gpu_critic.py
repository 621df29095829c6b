"""Fused critic forward (glad_critic_forward) vs the reference goldens and the oracle
(qrt/integration.py:133-135: shared encoder, fp16 critic embedding and MLP)."""
import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights, critic_forward

pytestmark = pytest.mark.gpu
MAX_ABS = 1e-2
MIN_COS = 0.99999


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


@pytest.fixture(scope="module")
def dw(golden_weights):
    return DeviceWeights(golden_weights)


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [1, 3, 16])
def test_critic_matches_reference_golden(dw, golden_fwd, mode, B):
    d = golden_fwd[B]
    v, _ = critic_forward(dw, torch.from_numpy(d["critic_obs"]).cuda(), mode)
    ref = d[f"{mode}.value"]
    assert np.abs(v.cpu().numpy() - ref).max() <= MAX_ABS
    if B > 1:
        assert cos(v.cpu().numpy(), ref) >= MIN_COS


@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_critic_vs_oracle(dw, golden_weights, mode):
    B = 300
    obs = glad_obs(B, seed=31, proprio_dim=99)
    v, aux = critic_forward(dw, obs.cuda(), mode)
    oaux = {}
    ref = O.critic_forward(obs.numpy(), O.GladWeights(golden_weights), mode, aux=oaux)
    got = v.cpu().numpy()
    assert np.abs(got - ref).max() <= MAX_ABS
    assert cos(got, ref) >= MIN_COS
    lg = aux["topk_logits"].cpu().numpy()
    idx = aux["topk_idx"].cpu().numpy()
    assert np.array_equal(idx, O.topk_lowest_index(lg, 32))
    enc = aux["encoded"].cpu().numpy()[:, :227].astype(np.float32)
    assert cos(enc, oaux["enc"].astype(np.float32)) > 0.9999
    assert np.array_equal(aux["encoded"].cpu().numpy()[:, 128:227], obs[:, :99].half().numpy())
