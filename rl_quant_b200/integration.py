"""accelerate_runner: one-call drop-in for an rsl_rl OnPolicyRunner
(qrt/integration.py:1-296).

    acc = accelerate_runner(runner)     # after the runner exists, before learn()
    runner.learn(...)                   # unchanged training code

What it does (qrt/integration.py:94-247):
  * an fp16 inference copy of ``runner.alg.policy`` (the fp32 master stays as is);
  * LET calibration of the qrt INT8 paths on real observations, swap to
    QuantLinear; QuantCNN for the map CNN; the encoder rewrite;
  * ``policy.update_distribution`` / ``policy.evaluate`` are rerouted to the
    copy whenever inference mode is on (the rollout); gradient-mode calls
    (the PPO update) keep the original float path;
  * ``alg.update`` is wrapped so every PPO iteration first checks the device
    status of the rollout's fused forwards (``InferenceRunner.check_status``,
    raising ``DeviceStatusError`` if a bounded device-side wait ran out) and
    ends with ``sync_weights_from`` (one graphed cast-copy + requantisation).

Training-side options of the reference (``accelerate_update``,
``update_amp``, ``cocalib``) concern the PPO update, which is outside this
package's scope: ``accelerate_update``/``update_amp`` are accepted and leave
the update path untouched; ``cocalib=True`` is rejected.
"""
from __future__ import annotations

import copy
import time
import types

import torch
from torch.distributions import Normal

from . import calib as _calib
from . import swap as _swap
from .encoder_opt import patch_encoder
from .qconv import calib_cnn_scale, swap_cnn
from .runtime import InferenceRunner

INT8_PATHS_DEFAULT = ["actor.0", "actor.2", "actor.4", "actor.6",
                      "actor_proprio_embedding", "query_projector"]


@torch.inference_mode()
def collect_calib_obs(runner, n_steps: int = 8):
    """Roll the current policy ``n_steps`` in the real env and keep the
    observations (qrt/integration.py:46-61)."""
    obs_list = []
    obs = runner.env.get_observations().to(runner.device)
    policy = runner.alg.policy
    was = policy.training
    policy.eval()
    for _ in range(n_steps):
        obs_list.append({k: v.clone() for k, v in obs.items()})
        actions = policy.act(obs)
        obs, _, _, _ = runner.env.step(actions.to(runner.env.device))
        obs = obs.to(runner.device)
    policy.train(was)
    return obs_list


class QRTAccelerator:
    def __init__(self, runner, int8_linear: bool = True, int8_cnn: bool = True,
                 graph_rewrite: bool = True, accelerate_update: bool = True,
                 rollout_training: bool = True, update_amp: str | None = "bf16",
                 act_mode: str = "dynamic", cocalib: bool = False, cocalib_source: str = "eager",
                 int8_paths: list[str] | None = None, calib_obs: list | None = None,
                 let_steps: int = 200, mode: str = "max-autotune", fused_ppo_act: bool = False,
                 verbose: bool = True):
        if cocalib:
            raise NotImplementedError("online co-calibration (training side) is not part of this package")
        if update_amp not in ("bf16", "fp32", None):
            raise ValueError(f"unknown update_amp: {update_amp}")
        t0 = time.perf_counter()
        self.runner = runner
        self.alg = runner.alg
        self.policy = runner.alg.policy
        dev = runner.device
        infer = copy.deepcopy(self.policy).half().to(dev)
        self.infer = infer
        self.rollout_training = rollout_training
        self.set_infer_training(rollout_training)
        self.swapped = {}
        if int8_linear or int8_cnn:
            if calib_obs is None:
                calib_obs = collect_calib_obs(runner)
            calib16 = [{k: v.half() for k, v in o.items()} for o in calib_obs]
            it = iter(calib16 * 64)
            obs_fn = lambda: next(it)  # noqa: E731
        if int8_linear:
            paths = [p for p in (int8_paths or INT8_PATHS_DEFAULT) if self._has_linear(infer, p)]
            plan = _calib.make_plan(infer, paths, obs_fn=obs_fn, n_calib=len(calib_obs), use_let=True,
                                    let_steps=let_steps, act_mode=act_mode, verbose=False)
            self.swapped = _swap.apply(infer, plan)
        if int8_cnn:
            swap_cnn(infer, calib_cnn_scale(infer, obs_fn, n_batches=len(calib_obs)))
        if graph_rewrite:
            patch_encoder(infer)
        self.set_infer_training(rollout_training)
        # observations reach the runner normalised by the fp32 master's normalisers
        # (policy.act / evaluate_qrt), as qrt compiles its heads without them
        self._runner = InferenceRunner(infer, mode=mode, with_critic=True, normalize=False)
        self._sync_runner = self._runner

        policy = self.policy
        self._orig_ud = policy.update_distribution
        self._orig_eval = policy.evaluate
        run = self._runner

        def _make_dist(self_p, mean):
            std = self_p.std.expand_as(mean) if getattr(self_p, "noise_std_type", "scalar") == "scalar" \
                else torch.exp(self_p.log_std).expand_as(mean)
            self_p.distribution = Normal(mean, std)

        acc = self

        def update_distribution_qrt(self_p, actor_obs):
            if torch.is_inference_mode_enabled():
                _make_dist(self_p, run.act(actor_obs).float())
            else:
                acc._orig_ud(actor_obs)

        def evaluate_qrt(self_p, obs, **kwargs):
            if torch.is_inference_mode_enabled():
                co = self_p.critic_obs_normalizer(self_p.get_critic_obs(obs))
                return run.evaluate(co.half()).float()
            return acc._orig_eval(obs, **kwargs)

        policy.update_distribution = types.MethodType(update_distribution_qrt, policy)
        policy.evaluate = types.MethodType(evaluate_qrt, policy)

        # opt-in: PPO.act (ppo.py:129-140) as one fused forward -- actor + critic (from one
        # read of the height scan when no normaliser is active: the policy and critic
        # groups must then carry the same scan), then the Normal sample and its
        # log-probability drawn in the kernel (Philox) instead of by torch.normal.
        self._orig_act = self.alg.act
        if fused_ppo_act:
            alg = self.alg

            def act_fused(obs):
                if policy.is_recurrent:
                    return acc._orig_act(obs)
                # raw groups; the master's normalisers run inside the kernels' row loads
                ao = policy.get_actor_obs(obs)
                co = policy.get_critic_obs(obs)
                kw = {"log_std": policy.log_std} if getattr(policy, "noise_std_type", "scalar") == "log" \
                    else {"std": policy.std}
                a, v, lp, m, sg = run.ppo_act(
                    ao, co, obs_norm=(policy.actor_obs_normalizer, policy.critic_obs_normalizer), **kw)
                t = alg.transition
                t.actions, t.values, t.actions_log_prob = a, v, lp
                t.action_mean, t.action_sigma = m, sg
                t.observations = obs
                return t.actions

            self.alg.act = act_fused

        self._orig_update = self.alg.update

        def update_qrt():
            # the rollout this update consumes ran on the fused kernels: raise before
            # training on it if any of their bounded device-side waits ran out
            acc._runner.check_status()
            out = acc._orig_update()
            acc._runner.sync_weights_from(acc.policy)
            return out

        self.alg.update = update_qrt
        if verbose:
            print(f"[rl_quant_b200] accelerate_runner ready ({time.perf_counter() - t0:.1f}s): "
                  f"int8_linear={int8_linear} int8_cnn={int8_cnn} rewrite={graph_rewrite} "
                  f"quant_modules={len(self._runner._quant_layers)} rollout_training={rollout_training}")

    def set_infer_training(self, flag: bool):
        """Train/eval flag of the copy (Gumbel exploration on/off); BatchNorm
        stays in eval (running statistics)."""
        self.infer.train(flag)
        for m in self.infer.modules():
            if isinstance(m, torch.nn.modules.batchnorm._BatchNorm):
                m.eval()

    @staticmethod
    def _has_linear(model, path):
        try:
            return isinstance(model.get_submodule(path), torch.nn.Linear)
        except AttributeError:
            return False

    @torch.inference_mode()
    def warmup(self, obs=None):
        if obs is None:
            obs = self.runner.env.get_observations().to(self.runner.device)
        p = self.policy
        ao = p.actor_obs_normalizer(p.get_actor_obs(obs))
        co = p.critic_obs_normalizer(p.get_critic_obs(obs))
        t0 = time.perf_counter()
        for _ in range(3):
            self._runner.act(ao.half())
            self._runner.evaluate(co.half())
        torch.cuda.synchronize()
        self._runner.sync_weights_from(self.policy)
        print(f"[rl_quant_b200] warmup done ({time.perf_counter() - t0:.1f}s)")
        return self

    def detach(self):
        """Undo every monkeypatch (training goes back to the original path)."""
        self.policy.update_distribution = self._orig_ud
        self.policy.evaluate = self._orig_eval
        self.alg.update = self._orig_update
        self.alg.act = self._orig_act


def accelerate_runner(runner, **kwargs) -> QRTAccelerator:
    return QRTAccelerator(runner, **kwargs)
