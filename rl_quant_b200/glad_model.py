"""GLAD actor-critic module: a self-contained stand-in for rsl_rl's
``ActorCriticEncoder`` (``rsl_rl/modules/actor_critic_encoder.py:17-377``).

The GPU path of this package never runs this module's float forward for
inference; the module exists so that

* the benchmark and the tests can build the GLAD network without rsl_rl,
* parameter and buffer names match the reference exactly (``map_cnn.0/2/3/5``,
  ``actor_proprio_embedding``, ``critic_proprio_embedding``,
  ``global_pool_selector``, ``query_projector``, ``topk_scorer``, ``mha``,
  ``actor.0/2/4/6``, ``critic.0/2/4/6``, ``std``) so state dicts load in both
  directions, and
* sub-modules are created in the reference's order, so the same
  ``torch.manual_seed`` yields the same default initialisation.

Only the GLAD main configuration is modelled: stride-2 CNN, global context on,
top-K on, no spatial prior (the configuration ``qrt/encoder_opt.py:128-133``
accepts).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.distributions import Normal

from .synthetic import MAP_C, MAP_L, MAP_W


def _mlp(in_dim: int, out_dim: int, hidden: list[int]) -> nn.Sequential:
    """Linear/ELU stack with Linear layers at even indices (``networks/mlp.py:59-83``)."""
    dims = [in_dim] + list(hidden)
    layers: list[nn.Module] = []
    for a, b in zip(dims[:-1], dims[1:]):
        layers += [nn.Linear(a, b), nn.ELU()]
    layers.append(nn.Linear(dims[-1], out_dim))
    return nn.Sequential(*layers)


class GladActorCritic(nn.Module):
    is_recurrent = False

    def __init__(self, actor_proprio_dim: int = 96, critic_proprio_dim: int = 99,
                 num_actions: int = 29, mha_dim: int = 64, num_heads: int = 16,
                 topk: int = 32, actor_hidden_dims=(512, 256, 128),
                 critic_hidden_dims=(512, 256, 128), init_noise_std: float = 1.0,
                 obs_groups: dict | None = None, topk_soft_tau: float = 1.0):
        super().__init__()
        D = mha_dim
        self.L, self.W, self.coord_dim = MAP_L, MAP_W, MAP_C
        self.mha_dim, self.num_heads, self.topk = D, num_heads, topk
        self.topk_soft_tau = topk_soft_tau
        self.use_global_context = True
        self.role_disentangle = False
        self.actor_proprio_dim = actor_proprio_dim
        self.critic_proprio_dim = critic_proprio_dim
        self.obs_groups = obs_groups or {"policy": ["policy_obs"], "critic": ["critic_obs"]}
        # Creation order below fixes the default-init RNG stream
        # (actor_critic_encoder.py:84-114).
        self.map_cnn = nn.Sequential(
            nn.Conv2d(3, 16, kernel_size=5, padding=2, stride=2), nn.ReLU(), nn.BatchNorm2d(16),
            nn.Conv2d(16, D, kernel_size=3, padding=1), nn.ReLU(), nn.BatchNorm2d(D))
        self.actor_proprio_embedding = nn.Linear(actor_proprio_dim, D)
        self.critic_proprio_embedding = nn.Linear(critic_proprio_dim, D)
        self.global_pool_selector = nn.Linear(D, 1)
        self.query_projector = nn.Linear(2 * D, D)
        self.topk_scorer = nn.Linear(2 * D, 1)
        self.mha = nn.MultiheadAttention(embed_dim=D, num_heads=num_heads, batch_first=True)
        self.actor = _mlp(2 * D + actor_proprio_dim, num_actions, list(actor_hidden_dims))
        self.critic = _mlp(2 * D + critic_proprio_dim, 1, list(critic_hidden_dims))
        self.actor_obs_normalizer = nn.Identity()
        self.critic_obs_normalizer = nn.Identity()
        self.noise_std_type = "scalar"
        self.std = nn.Parameter(init_noise_std * torch.ones(num_actions))
        self.distribution = None
        Normal.set_default_validate_args(False)

    # -- float encoder (reference math, actor_critic_encoder.py:195-312) ------
    def _encode_terrain(self, obs):
        n_map = self.L * self.W * self.coord_dim
        scan = obs[:, -n_map:].reshape(-1, self.W, self.L, self.coord_dim)
        feat = self.map_cnn(scan.permute(0, 3, 1, 2))                 # [B, D, 11, 17]
        B_, D_ = feat.shape[0], feat.shape[1]
        local = feat.permute(0, 2, 3, 1).reshape(B_, -1, D_)          # [B, N, D]
        proprio = obs[:, :-n_map]
        if proprio.shape[1] == self.actor_proprio_dim:
            emb = self.actor_proprio_embedding(proprio)
        elif proprio.shape[1] == self.critic_proprio_dim:
            emb = self.critic_proprio_embedding(proprio)
        else:
            raise ValueError(f"proprio width {proprio.shape[1]} matches neither "
                             f"actor({self.actor_proprio_dim}) nor critic({self.critic_proprio_dim})")
        gc_w = F.softmax(self.global_pool_selector(local).squeeze(-1), dim=1).unsqueeze(-1)
        gc = torch.bmm(gc_w.transpose(1, 2), local).squeeze(1)
        query = self.query_projector(torch.cat([gc, emb], dim=-1))
        n_tok = local.shape[1]
        k = min(self.topk, n_tok)
        scorer_in = torch.cat([local, query.unsqueeze(1).expand(-1, n_tok, -1)], dim=-1)
        logits = self.topk_scorer(scorer_in).squeeze(-1)
        if self.training:
            u = torch.rand_like(logits)
            logits = logits - torch.log(-torch.log(u + 1e-10) + 1e-10)
        idx = torch.topk(logits, k, dim=-1).indices
        sparse = torch.gather(local, 1, idx.unsqueeze(-1).expand(-1, -1, D_))
        if self.training:
            soft = torch.gather(F.softmax(logits / max(self.topk_soft_tau, 1e-6), dim=-1), 1, idx)
            soft_feat = sparse * soft.unsqueeze(-1)
            sparse = sparse.detach() + (soft_feat - soft_feat.detach())
        att, att_w = self.mha(query=query.unsqueeze(1), key=sparse, value=sparse)
        encoded = torch.cat([att.squeeze(1), gc, proprio], dim=-1)
        return encoded, att_w, idx, gc_w

    # -- rsl_rl policy interface (actor_critic_encoder.py:315-373) -------------
    def reset(self, dones=None):
        pass

    @property
    def action_mean(self):
        return self.distribution.mean

    @property
    def action_std(self):
        return self.distribution.stddev

    @property
    def entropy(self):
        return self.distribution.entropy().sum(dim=-1)

    def update_distribution(self, obs):
        enc, _, _, _ = self._encode_terrain(obs)
        mean = self.actor(enc)
        self.distribution = Normal(mean, self.std.expand_as(mean))

    def act(self, obs, **kwargs):
        self.update_distribution(self.actor_obs_normalizer(self.get_actor_obs(obs)))
        return self.distribution.sample()

    def act_inference(self, obs):
        enc, att_w, idx, gc_w = self._encode_terrain(
            self.actor_obs_normalizer(self.get_actor_obs(obs)))
        return self.actor(enc), att_w, idx, gc_w

    def evaluate(self, obs, **kwargs):
        enc, _, _, _ = self._encode_terrain(self.critic_obs_normalizer(self.get_critic_obs(obs)))
        return self.critic(enc)

    def get_actor_obs(self, obs):
        if isinstance(obs, torch.Tensor):
            return obs
        return torch.cat([obs[g] for g in self.obs_groups["policy"]], dim=-1)

    def get_critic_obs(self, obs):
        if isinstance(obs, torch.Tensor):
            return obs
        return torch.cat([obs[g] for g in self.obs_groups["critic"]], dim=-1)

    def get_actions_log_prob(self, actions):
        return self.distribution.log_prob(actions).sum(dim=-1)


def build_glad(seed: int = 0, critic_seed: int | None = 2, dtype=torch.float32,
               device="cpu") -> GladActorCritic:
    """GLAD main configuration with default init from ``seed``.

    BatchNorm running statistics keep their defaults (mean 0, var 1). When
    ``critic_seed`` is given, the critic-only modules (critic proprio
    embedding and critic MLP) are re-initialised from that seed, which is how
    the actor+critic workload separates the two heads.
    """
    torch.manual_seed(int(seed))
    m = GladActorCritic()
    if critic_seed is not None:
        torch.manual_seed(int(critic_seed))
        m.critic_proprio_embedding.reset_parameters()
        for layer in m.critic:
            if isinstance(layer, nn.Linear):
                layer.reset_parameters()
    return m.to(device=device, dtype=dtype).eval()
