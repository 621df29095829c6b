"""patch_encoder / unpatch_encoder (qrt/encoder_opt.py:126-146).

The patched ``_encode_terrain`` is the reference's algebraic rewrite
(qrt/encoder_opt.py:41-123):
  * GPS selector and the local half of the top-k scorer share one [D->2]
    product over the local features; the query half is a per-env scalar;
  * the multi-head attention is a single-query attention written out.

Without autograd it runs the fused sm_100a encoder in encoder-only mode
(glad_actor_forward for the actor observation group, glad_critic_forward for
the critic group): conv chain, pooling, query, top-32, attention. With autograd (PPO update) it runs the same rewrite in float torch
ops on the model's own parameters, as the reference does.
"""
from __future__ import annotations

import types
import warnings

import torch
import torch.nn.functional as F

from .fused import FusedActor, FusedCritic


def _encode_terrain_float(self, obs):
    n_map = self.L * self.W * self.coord_dim
    scan = obs[:, -n_map:].reshape(-1, self.W, self.L, self.coord_dim)
    feat = self.map_cnn(scan.permute(0, 3, 1, 2))
    B, D = feat.shape[0], feat.shape[1]
    local = feat.permute(0, 2, 3, 1).reshape(B, -1, D)
    n_tok = local.shape[1]
    prop = obs[:, :-n_map]
    if prop.shape[1] == self.actor_proprio_dim:
        emb = self.actor_proprio_embedding(prop)
    elif prop.shape[1] == self.critic_proprio_dim:
        emb = self.critic_proprio_embedding(prop)
    else:
        raise ValueError(f"proprio dim {prop.shape[1]} matches neither actor({self.actor_proprio_dim}) "
                         f"nor critic({self.critic_proprio_dim})")
    w_s = self.topk_scorer.weight
    both = local @ torch.cat([self.global_pool_selector.weight, w_s[:, :D]], dim=0).t()
    gc_w = F.softmax(both[..., 0] + self.global_pool_selector.bias, dim=1).unsqueeze(-1)
    gc = torch.bmm(gc_w.transpose(1, 2), local).squeeze(1)
    query = self.query_projector(torch.cat([gc, emb], dim=-1))
    logits = both[..., 1] + (query @ w_s[:, D:].t() + self.topk_scorer.bias)
    k = min(self.topk, n_tok)
    if self.training:
        u = torch.rand_like(logits)
        logits = logits - torch.log(-torch.log(u + 1e-10) + 1e-10)
    idx = torch.topk(logits, k, dim=-1).indices
    sparse = torch.gather(local, 1, idx.unsqueeze(-1).expand(-1, -1, D))
    if self.training:
        soft = torch.gather(F.softmax(logits / max(self.topk_soft_tau, 1e-6), dim=-1), 1, idx)
        sf = sparse * soft.unsqueeze(-1)
        sparse = sparse.detach() + (sf - sf.detach())
    W_in, b_in = self.mha.in_proj_weight, self.mha.in_proj_bias
    H = self.num_heads
    hd = D // H
    q = (query @ W_in[:D].t() + b_in[:D]).view(B, H, 1, hd)
    kk = (sparse @ W_in[D:2 * D].t() + b_in[D:2 * D]).view(B, k, H, hd).transpose(1, 2)
    v = (sparse @ W_in[2 * D:].t() + b_in[2 * D:]).view(B, k, H, hd).transpose(1, 2)
    attn = F.softmax((q @ kk.transpose(-1, -2)) * (1.0 / hd ** 0.5), dim=-1)
    foot = (attn @ v).reshape(B, D) @ self.mha.out_proj.weight.t() + self.mha.out_proj.bias
    enc = torch.cat([foot, gc, prop], dim=-1)
    return enc, attn.squeeze(2).mean(dim=1, keepdim=True), idx, gc_w


def _gumbel_noise(logit_shape, device, dtype=torch.float16):
    u = torch.rand(logit_shape, device=device, dtype=dtype)
    return (-torch.log(-torch.log(u + 1e-10) + 1e-10)).float()


def _encode_terrain_opt(self, obs):
    if torch.is_grad_enabled():
        return _encode_terrain_float(self, obs)
    n_map = self.L * self.W * self.coord_dim
    P = obs.shape[1] - n_map
    # the group picks its embedding by its proprio width (qrt/encoder_opt.py:57-66;
    # the actor's when both widths agree, rsl_rl actor_critic_encoder.py:226-229)
    if P == self.actor_proprio_dim:
        key, make = "_glad_fused", lambda: FusedActor(self, need_mlp=False)
    elif P == self.critic_proprio_dim:
        key, make = "_glad_fused_critic", lambda: FusedCritic(self, need_mlp=False)
    else:
        raise ValueError(f"proprio dim {P} matches neither actor({self.actor_proprio_dim}) "
                         f"nor critic({self.critic_proprio_dim})")
    fused = self.__dict__.get(key)
    if fused is None:
        fused = make()
        self.__dict__[key] = fused
    noise = _gumbel_noise((obs.shape[0], 187), obs.device) if self.training else None
    return fused.encode(obs, noise)


def patch_encoder(model):
    """Replace ``model._encode_terrain`` by the rewrite (instance level)."""
    if not (getattr(model, "use_global_context", True) and getattr(model, "topk", None) is not None):
        warnings.warn("[rl_quant_b200] patch_encoder supports the GLAD main config (gc + topk) only; not patched")
        return model
    if getattr(model, "role_disentangle", False):
        warnings.warn("[rl_quant_b200] role_disentangle=True is not supported; not patched")
        return model
    if getattr(model, "_encode_terrain_orig", None) is None:
        model._encode_terrain_orig = model._encode_terrain
    model._encode_terrain = types.MethodType(_encode_terrain_opt, model)
    return model


def unpatch_encoder(model):
    orig = getattr(model, "_encode_terrain_orig", None)
    if orig is not None:
        model._encode_terrain = orig
        model._encode_terrain_orig = None
    return model
