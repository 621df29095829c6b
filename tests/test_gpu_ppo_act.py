"""PPO.act in one fused forward: InferenceRunner.ppo_act and the opt-in
accelerate_runner(fused_ppo_act=True) hook against the unfused pieces -- the
action mean equals act(), the value equals evaluate(), the sample equals the
oracle's Philox/Box-Muller draw at the runner's seed and offset, the
log-probability equals torch's Normal.log_prob of the returned actions."""
import types

import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200 import InferenceRunner
from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.integration import accelerate_runner
from rl_quant_b200.synthetic import glad_obs_pair

from gpu_util import golden_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def infer(golden_weights):
    m, _ = golden_model(golden_weights)
    return m


def _check_transition(run, po, co, actions, values, log_prob, mean, sigma, std, offset):
    B = po.shape[0]
    assert torch.equal(mean, run.act(po).float())
    assert torch.equal(values, run.evaluate(co).float())
    ea, _ = O.ppo_epilogue(mean.cpu().numpy(), std.float().cpu().numpy(), run._ppo_seed, offset)
    np.testing.assert_allclose(actions.cpu().numpy(), ea, rtol=2e-6, atol=2e-6)
    ref = torch.distributions.Normal(mean.cpu(), std.float().cpu().expand(B, 29)).log_prob(actions.cpu()).sum(-1)
    np.testing.assert_allclose(log_prob.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=5e-5)
    assert torch.equal(sigma, std.float().expand(B, 29))


@pytest.mark.parametrize("mode", ["eager", "manual-graph"])
def test_runner_ppo_act(infer, mode):
    infer.eval()
    r = InferenceRunner(infer, mode=mode, with_critic=True)
    B = 300
    po, co = glad_obs_pair(B, seed=4242)
    po, co = po.cuda(), co.cuda()
    std = (0.3 + 0.02 * torch.arange(29, dtype=torch.float32)).cuda()
    for k in range(3):
        a, v, lp, m, sg = (t.clone() for t in r.ppo_act(po, co, std=std))
        torch.cuda.synchronize()
        _check_transition(r, po, co, a, v, lp, m, sg, std, offset=k)
    assert r._ppo_rng.cpu().tolist() == [3, 0]


def test_runner_ppo_act_train_mode(infer):
    """Train mode: both heads draw Gumbel terms (offset advances by two per call), the
    action noise stream advances by one."""
    infer.train()
    for mod in infer.modules():
        if isinstance(mod, torch.nn.modules.batchnorm._BatchNorm):
            mod.eval()
    try:
        r = InferenceRunner(infer, mode="manual-graph", with_critic=True)
        po, co = glad_obs_pair(64, seed=77)
        po, co = po.cuda(), co.cuda()
        out1 = [t.clone() for t in r.ppo_act(po, co)]
        out2 = [t.clone() for t in r.ppo_act(po, co)]
        torch.cuda.synchronize()
        assert int(r._gumbel_offset.item()) == 4
        assert r._ppo_rng.cpu().tolist() == [2, 0]
        assert all(torch.isfinite(t).all() for t in out1 + out2)
        assert not torch.equal(out1[0], out2[0])
    finally:
        infer.eval()


class _Transition:
    def clear(self):
        self.__dict__.clear()


class _PPO:
    """The rollout half of rsl_rl's PPO (rsl_rl/algorithms/ppo.py:129-140)."""

    def __init__(self, policy):
        self.policy = policy
        self.transition = _Transition()

    def act(self, obs):
        self.transition.actions = self.policy.act(obs).detach()
        self.transition.values = self.policy.evaluate(obs).detach()
        self.transition.actions_log_prob = self.policy.get_actions_log_prob(self.transition.actions).detach()
        self.transition.action_mean = self.policy.action_mean.detach()
        self.transition.action_sigma = self.policy.action_std.detach()
        self.transition.observations = obs
        return self.transition.actions

    def update(self):
        return {}


def test_accelerate_runner_fused_ppo_act():
    policy = build_glad(seed=0, critic_seed=2, dtype=torch.float32, device="cuda")
    with torch.no_grad():
        policy.std.copy_(0.5 + 0.01 * torch.arange(29, dtype=torch.float32))
    runner = types.SimpleNamespace(alg=_PPO(policy), device="cuda", env=None)
    calib = []
    for i in range(2):
        po, co = glad_obs_pair(64, seed=600 + i)
        calib.append({"policy_obs": po.cuda(), "critic_obs": co.cuda()})
    acc = accelerate_runner(runner, calib_obs=calib, let_steps=10, mode="manual-graph", rollout_training=False,
                            fused_ppo_act=True, verbose=False)
    po, co = glad_obs_pair(128, seed=31)
    obs = {"policy_obs": po.cuda(), "critic_obs": co.cuda()}
    with torch.inference_mode():
        a = runner.alg.act(obs)
    t = runner.alg.transition
    assert a is t.actions and t.observations is obs
    _check_transition(acc._runner, obs["policy_obs"], obs["critic_obs"], t.actions.clone(), t.values.clone(),
                      t.actions_log_prob.clone(), t.action_mean.clone(), t.action_sigma.clone(), policy.std.detach(),
                      offset=0)
    # the unfused drop-in path: the same mean and value, torch's own sample
    acc.detach()
    acc2 = accelerate_runner(runner, calib_obs=calib, let_steps=10, mode="manual-graph",
                             rollout_training=False, verbose=False)
    with torch.inference_mode():
        runner.alg.act(obs)
    t2 = runner.alg.transition
    assert t2.actions.shape == (128, 29) and t2.values.shape == (128, 1)
    acc2.detach()
