"""Observation normaliser in the row load (GladObsNorm): the fused actor and
critic on the raw f32 group with an EmpiricalNormalization equal, bit for bit,
the same kernels on the group normalised by torch on the GPU (rsl_rl's
policy.act path: normalise in fp32, then the fp16 cast); the ABI rejects the
cases it does not cover; ppo_act and the accelerate_runner hook with active
normalisers."""
import types

import numpy as np
import pytest
import torch

from rl_quant_b200 import InferenceRunner, QuantLinear
from rl_quant_b200 import _native as N
from rl_quant_b200.fused import FusedActor, FusedActorCritic, FusedCritic, FusedUnsupported
from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.integration import accelerate_runner
from rl_quant_b200.synthetic import glad_obs_pair

from gpu_util import EmpiricalNorm, golden_model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def infer(golden_weights):
    m, _ = golden_model(golden_weights)
    return m


def _norm(width, seed):
    g = torch.Generator().manual_seed(seed)
    n = EmpiricalNorm(width).cuda()
    for _ in range(3):
        n.update((1.5 * torch.randn(512, width, generator=g) + 0.3).cuda())
    return n


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [7, 900])
def test_fused_heads_normalise_in_load(infer, mode, B):
    for mod in infer.modules():
        if isinstance(mod, QuantLinear):
            mod.act_mode = mode
    infer.eval()
    po, co = glad_obs_pair(B, seed=70 + B)
    po, co = po.cuda(), co.cuda()
    an, cn = _norm(po.shape[1], 1), _norm(co.shape[1], 2)
    fa, fc = FusedActor(infer), FusedCritic(infer)
    m1, m2 = torch.empty(B, 29, device="cuda"), torch.empty(B, 29, device="cuda")
    fa.run(po, m1, obs_norm=an)
    fa.run(an(po), m2)                       # torch's fp32 normalisation on the GPU
    v1, v2 = torch.empty(B, 1, device="cuda"), torch.empty(B, 1, device="cuda")
    fc.run(co, v1, obs_norm=cn)
    fc.run(cn(co), v2)
    torch.cuda.synchronize()
    assert torch.isfinite(m1).all() and torch.isfinite(v1).all()
    assert torch.equal(m1, m2)
    assert torch.equal(v1, v2)
    # the normaliser really acts, and its buffers are read in place on every call
    m3 = torch.empty(B, 29, device="cuda")
    fa.run(po, m3)
    assert not torch.equal(m3, m1)
    an.update((torch.randn(256, po.shape[1]) * 0.5).cuda())
    m4, m5 = torch.empty(B, 29, device="cuda"), torch.empty(B, 29, device="cuda")
    fa.run(po, m4, obs_norm=an)
    fa.run(an(po), m5)
    torch.cuda.synchronize()
    assert torch.equal(m4, m5) and not torch.equal(m4, m1)


def test_obs_norm_argument_checks(infer):
    infer.eval()
    po, co = glad_obs_pair(4, seed=5)
    po, co = po.cuda(), co.cuda()
    an = _norm(po.shape[1], 3)
    fa, fac = FusedActor(infer), FusedActorCritic(infer)
    m = torch.empty(4, 29, device="cuda")
    with pytest.raises(ValueError):             # fp16 rows: the normaliser runs before the cast
        fa.run(po.half(), m, obs_norm=an)
    with pytest.raises(ValueError):             # wrong width
        fa.run(po, m, obs_norm=_norm(100, 4))
    # the shared-scan call takes no normaliser
    w = fac.actor.weights(an)
    ws = torch.zeros(N.load().glad_actor_critic_workspace_size(4), dtype=torch.uint8, device="cuda")
    v = torch.empty(4, 1, device="cuda")
    rc = N.load().glad_actor_critic_forward(w, fac.critic.weights(), po.data_ptr(), co.data_ptr(), N.DTYPE_F32, 4,
                                            po.stride(0), co.stride(0), N.ACT_MODES[fac.actor.act_mode],
                                            m.data_ptr(), v.data_ptr(), ws.data_ptr(), ws.numel(),
                                            N.stream_handle())
    assert rc == -1


def test_ppo_act_with_normalisers(infer):
    infer.eval()
    B = 256
    po, co = glad_obs_pair(B, seed=808)
    po, co = po.cuda(), co.cuda()
    an, cn = _norm(po.shape[1], 11), _norm(co.shape[1], 12)
    r = InferenceRunner(infer, mode="manual-graph", with_critic=True, normalize=False)
    std = torch.full((29,), 0.4, device="cuda")
    a, v, lp, m, sg = (t.clone() for t in r.ppo_act(po, co, std=std, obs_norm=(an, cn)))
    torch.cuda.synchronize()
    assert torch.equal(m, r.act(an(po)).float())
    assert torch.equal(v, r.evaluate(cn(co)).float())
    ref = torch.distributions.Normal(m, std.expand(B, 29)).log_prob(a).sum(-1)
    np.testing.assert_allclose(lp.cpu().numpy(), ref.cpu().numpy(), rtol=1e-6, atol=5e-5)
    with pytest.raises(FusedUnsupported):
        InferenceRunner(build_glad(0).cuda().half(), mode="eager", with_critic=True).ppo_act(po, co)


class _PPO:
    def __init__(self, policy):
        self.policy = policy
        self.transition = types.SimpleNamespace()

    def act(self, obs):  # rsl_rl/algorithms/ppo.py:129-140
        self.transition.actions = self.policy.act(obs).detach()
        self.transition.values = self.policy.evaluate(obs).detach()
        self.transition.actions_log_prob = self.policy.get_actions_log_prob(self.transition.actions).detach()
        self.transition.action_mean = self.policy.action_mean.detach()
        self.transition.action_sigma = self.policy.action_std.detach()
        self.transition.observations = obs
        return self.transition.actions

    def update(self):
        return {}


def test_accelerate_runner_with_normalisers():
    """Active normalisers: the unfused hook normalises once (master's fp32 module, as
    rsl_rl's policy.act does) and the fused PPO.act normalises in the kernels; both give
    the same action means and values."""
    policy = build_glad(seed=0, critic_seed=2, dtype=torch.float32, device="cuda")
    po, co = glad_obs_pair(64, seed=900)
    policy.actor_obs_normalizer = _norm(po.shape[1], 21)
    policy.critic_obs_normalizer = _norm(co.shape[1], 22)
    runner = types.SimpleNamespace(alg=_PPO(policy), device="cuda", env=None)
    calib = [{"policy_obs": po.cuda(), "critic_obs": co.cuda()}]
    acc = accelerate_runner(runner, calib_obs=calib, let_steps=5, mode="manual-graph", rollout_training=False,
                            fused_ppo_act=True, verbose=False)
    po2, co2 = glad_obs_pair(96, seed=901)
    obs = {"policy_obs": po2.cuda(), "critic_obs": co2.cuda()}
    with torch.inference_mode():
        runner.alg.act(obs)
        t = runner.alg.transition
        fused = (t.action_mean.clone(), t.values.clone())
        acc.detach()
        acc2_mean = acc._runner.act(policy.actor_obs_normalizer(obs["policy_obs"])).float()
        acc2_val = acc._runner.evaluate(policy.critic_obs_normalizer(obs["critic_obs"])).float()
    assert torch.equal(fused[0], acc2_mean)
    assert torch.equal(fused[1], acc2_val)
