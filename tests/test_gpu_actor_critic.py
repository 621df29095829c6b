"""Fused actor + critic (one read of the shared scan) equals the two separate
fused forwards bit for bit: the same kernels compute the same values, the
critic's query-projector absmax lands in its own slot."""
import pytest
import torch

from rl_quant_b200 import QuantLinear
from rl_quant_b200.fused import FusedActor, FusedActorCritic, FusedCritic
from rl_quant_b200.synthetic import glad_obs_pair

from gpu_util import golden_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def infer(golden_weights):
    m, _ = golden_model(golden_weights)
    return m


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [5, 700])
def test_actor_critic_equals_separate_heads(infer, mode, B):
    for mod in infer.modules():
        if isinstance(mod, QuantLinear):
            mod.act_mode = mode
    po, co = glad_obs_pair(B, seed=900 + B)
    po, co = po.cuda(), co.cuda()
    fa, fc, fac = FusedActor(infer), FusedCritic(infer), FusedActorCritic(infer)
    m1 = torch.empty(B, 29, device="cuda")
    v1 = torch.empty(B, 1, device="cuda")
    fa.run(po, m1)
    fc.run(co, v1)
    m2 = torch.empty(B, 29, device="cuda")
    v2 = torch.empty(B, 1, device="cuda")
    fac.run(po, co, m2, v2)
    torch.cuda.synchronize()
    assert torch.isfinite(m2).all() and torch.isfinite(v2).all()
    assert torch.equal(m1, m2)
    assert torch.equal(v1, v2)
