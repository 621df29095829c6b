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


@pytest.mark.parametrize("B", [5, 700])
def test_actor_critic_train_mode(infer, B):
    """Train-mode fused call: the actor's Gumbel term at offset k (the mean equals
    FusedActor's train-mode forward bit for bit), the critic's at k + 1 (the value
    equals FusedCritic fed the oracle's Gumbel term at k + 1), offset advanced by two."""
    import numpy as np
    from oracle import glad_oracle as O

    for mod in infer.modules():
        if isinstance(mod, QuantLinear):
            mod.act_mode = "dynamic"
    po, co = glad_obs_pair(B, seed=950 + B)
    po, co = po.cuda(), co.cuda()
    fa, fc, fac = FusedActor(infer), FusedCritic(infer), FusedActorCritic(infer)
    off = torch.tensor([3], dtype=torch.int64, device="cuda")
    m2 = torch.empty(B, 29, device="cuda")
    v2 = torch.empty(B, 1, device="cuda")
    fac.run(po, co, m2, v2, gumbel=(77, off))
    torch.cuda.synchronize()
    assert int(off.item()) == 5
    off1 = torch.tensor([3], dtype=torch.int64, device="cuda")
    m1 = torch.empty(B, 29, device="cuda")
    fa.run(po, m1, gumbel=(77, off1))
    v1 = torch.empty(B, 1, device="cuda")
    fc.run(co, v1, torch.from_numpy(O.gumbel16(77, 4, B)).cuda())
    torch.cuda.synchronize()
    assert torch.equal(m1, m2)
    a, b = v1.cpu().numpy(), v2.cpu().numpy()
    # the oracle's Gumbel term is computed with numpy's log: equal to the kernel's after
    # the fp16 rounding except in rare last-bit cases
    assert np.mean(a == b) >= 0.99 and np.abs(a - b).max() <= 1e-2
    # eval-mode values differ: the noise is really applied
    v3 = torch.empty(B, 1, device="cuda")
    fac.run(po, co, m1, v3)
    assert not torch.equal(v3, v2)
