"""Driver of the fused GLAD forward (``glad_actor_forward``).

``FusedActor`` reads the quantised model in place: the C weight struct holds
pointers to the modules' own buffers and parameters (QuantCNN, QuantLinear,
fp16 GPS selector / scorer / MHA), so ``requantize_`` / ``sync_weights_from``
updates are seen by the next call and by captured CUDA graphs.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _native as N
from .qconv import QuantCNN
from .qlinear import QuantLinear

MLP_PATHS = ("actor.0", "actor.2", "actor.4", "actor.6")


class FusedUnsupported(NotImplementedError):
    pass


class DeviceStatusError(RuntimeError):
    """A bounded device-side wait (a tensor-core completion or a grid barrier) ran out in
    one of the launches since the last status check: their outputs are not valid."""


def check_workspaces(workspaces, who: str) -> None:
    """Read and clear the device status word of every workspace (one host sync). Raises
    DeviceStatusError naming the status bits when one was set."""
    lib = N.load()
    bad = []
    for key, ws in workspaces.items():
        st = N.c_uint32(0)
        rc = lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle(ws.device))
        if rc == N.GLAD_ERR_DEVICE:
            bad.append((key, st.value))
        else:
            N.check(rc, f"{who} status")
    if bad:
        raise DeviceStatusError(f"{who}: a bounded device-side wait ran out (status " +
                                ", ".join(f"B={k[0]}: 0x{v:x}" for k, v in bad) +
                                "); the results since the previous check are not valid")


def _fp16(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
        raise FusedUnsupported(f"{name} must be a contiguous fp16 CUDA tensor (the inference copy is .half())")
    return t


def obs_norm_struct(norm, width: int) -> N.GladObsNorm:
    """GladObsNorm of an rsl_rl EmpiricalNormalization (rsl_rl/networks/normalization.py:
    44-47): its fp32 ``_mean`` / ``_var`` buffers, read in place on every call, and its
    eps. None or nn.Identity: no normaliser."""
    if norm is None or isinstance(norm, nn.Identity):
        return N.GladObsNorm()
    mean, var = getattr(norm, "_mean", None), getattr(norm, "_var", None)
    if mean is None or var is None or not hasattr(norm, "eps"):
        raise FusedUnsupported(f"{type(norm).__name__} is not an EmpiricalNormalization (_mean, _var, eps)")
    for t, nm in ((mean, "_mean"), (var, "_var")):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous() or t.numel() != width:
            raise ValueError(f"normaliser {nm} must be a contiguous fp32 CUDA tensor of {width} values")
    return N.GladObsNorm(mean.data_ptr(), var.data_ptr(), float(norm.eps), width)


def model_act_mode(model: nn.Module) -> str:
    modes = {m.act_mode for m in model.modules() if isinstance(m, QuantLinear)}
    if len(modes) != 1 or not modes <= {"static", "dynamic"}:
        raise FusedUnsupported(f"fused path needs one act_mode in {{static, dynamic}}, model has {sorted(modes)}")
    return modes.pop()


class FusedActor:
    """The fused encoder (+ INT8 actor MLP) of one GLAD inference copy."""

    def __init__(self, model: nn.Module, need_mlp: bool = True):
        self.model = model
        self.check(model, need_mlp)
        self.act_mode = model_act_mode(model)
        self._ws: dict[tuple, torch.Tensor] = {}

    @staticmethod
    def check(model: nn.Module, need_mlp: bool = True) -> None:
        if not isinstance(model.map_cnn, QuantCNN):
            raise FusedUnsupported("map_cnn is not a QuantCNN (swap_cnn first)")
        for p in ("actor_proprio_embedding", "query_projector") + (MLP_PATHS if need_mlp else ()):
            if not isinstance(model.get_submodule(p), QuantLinear):
                raise FusedUnsupported(f"{p} is not a QuantLinear (swap.apply the qrt INT8 paths)")
        if model.actor_proprio_embedding.in_features != 96:
            raise FusedUnsupported("the fused encoder is built for a 96-wide actor proprio")
        if getattr(model, "num_heads", 16) != 16 or getattr(model, "mha_dim", 64) != 64:
            raise FusedUnsupported("the fused encoder is built for D=64, 16 heads")

    def weights(self, obs_norm=None) -> N.GladActorWeights:
        m = self.model
        w = N.GladActorWeights()
        w.obs_norm = obs_norm_struct(obs_norm, 96 + 2079)
        w.conv = m.map_cnn.conv_struct()
        w.proprio_emb = N.qlinear_struct(m.actor_proprio_embedding)
        w.query_proj = N.qlinear_struct(m.query_projector)
        w.gps_w = _fp16(m.global_pool_selector.weight, "global_pool_selector.weight").data_ptr()
        w.gps_b = _fp16(m.global_pool_selector.bias, "global_pool_selector.bias").data_ptr()
        w.scorer_w = _fp16(m.topk_scorer.weight, "topk_scorer.weight").data_ptr()
        w.scorer_b = _fp16(m.topk_scorer.bias, "topk_scorer.bias").data_ptr()
        w.mha_in_w = _fp16(m.mha.in_proj_weight, "mha.in_proj_weight").data_ptr()
        w.mha_in_b = _fp16(m.mha.in_proj_bias, "mha.in_proj_bias").data_ptr()
        w.mha_out_w = _fp16(m.mha.out_proj.weight, "mha.out_proj.weight").data_ptr()
        w.mha_out_b = _fp16(m.mha.out_proj.bias, "mha.out_proj.bias").data_ptr()
        for i, p in enumerate(MLP_PATHS):
            layer = m.get_submodule(p)
            if isinstance(layer, QuantLinear):
                w.mlp[i] = N.qlinear_struct(layer)
        return w

    def workspace(self, B: int, device) -> torch.Tensor:
        key = (B, str(device))
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.zeros(N.load().glad_actor_workspace_size(B), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def check_status(self) -> None:
        """Raise DeviceStatusError if a launch since the previous check reported a
        device-side timeout (reads and clears each workspace's status word; one sync)."""
        check_workspaces(self._ws, "fused actor")

    def run(self, obs: torch.Tensor, mean: torch.Tensor | None, aux: N.GladActorAux | None = None,
            noise: torch.Tensor | None = None, gumbel: tuple | None = None, obs_norm=None) -> None:
        """Launch the fused forward on the current stream (no host sync).

        ``noise``: f32 [B,187] added to the top-k logits. ``gumbel = (seed, offset)``
        instead draws the train-mode Gumbel term inside the kernel; ``offset`` is an
        int64 device tensor of one element that every call advances by one.
        ``obs_norm``: an EmpiricalNormalization applied to the f32 rows as they load
        (the observations are then the raw group)."""
        N.require_cuda(obs)
        if obs.dim() != 2 or obs.stride(1) != 1:
            raise ValueError("obs must be a row-major [B, 96+2079] tensor")
        if obs.dtype not in (torch.float32, torch.float16):
            raise TypeError("obs must be float32 or float16")
        if noise is not None and gumbel is not None:
            raise ValueError("pass either noise or gumbel")
        B = obs.shape[0]
        ws = self.workspace(B, obs.device)
        dt = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
        if gumbel is not None:
            seed, offset = gumbel
            N.require_cuda(offset)
            if offset.dtype != torch.int64 or offset.numel() != 1:
                raise ValueError("gumbel offset must be a one-element int64 CUDA tensor")
            rc = N.load().glad_actor_forward_train(
                self.weights(obs_norm), obs.data_ptr(), dt, B, obs.stride(0), N.ACT_MODES[self.act_mode],
                int(seed) & 0xFFFFFFFFFFFFFFFF, offset.data_ptr(), N.ptr(mean), aux, ws.data_ptr(), ws.numel(),
                N.stream_handle(obs.device))
            N.check(rc, "glad_actor_forward_train")
            return
        rc = N.load().glad_actor_forward(
            self.weights(obs_norm), obs.data_ptr(), dt, B, obs.stride(0), N.ACT_MODES[self.act_mode], N.ptr(noise),
            N.ptr(mean), aux, ws.data_ptr(), ws.numel(), N.stream_handle(obs.device))
        N.check(rc, "glad_actor_forward")

    def act(self, obs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        B = obs.shape[0]
        mean = out if out is not None else torch.empty(B, 29, dtype=torch.float32, device=obs.device)
        self.run(obs, mean)
        return mean

    def encode(self, obs: torch.Tensor, noise: torch.Tensor | None = None):
        """``_encode_terrain`` outputs: (encoded [B,224] fp16, attn_weights [B,1,32],
        topk_indices [B,32] int64, gc_weights [B,187,1])."""
        B, dev = obs.shape[0], obs.device
        enc = torch.empty(B, 224, dtype=torch.float16, device=dev)
        attn = torch.empty(B, 1, 32, dtype=torch.float16, device=dev)
        idx = torch.empty(B, 32, dtype=torch.int64, device=dev)
        gcw = torch.empty(B, 187, 1, dtype=torch.float16, device=dev)
        aux = N.GladActorAux()
        aux.encoded, aux.attn_weights, aux.topk_idx, aux.gc_weights = (
            enc.data_ptr(), attn.data_ptr(), idx.data_ptr(), gcw.data_ptr())
        self.run(obs, None, aux, noise)
        return enc, attn, idx, gcw


class FusedCritic:
    """The fused critic forward (``glad_critic_forward``) of one GLAD inference
    copy: shared encoder, critic proprio embedding, fp16 critic MLP."""

    def __init__(self, model: nn.Module, need_mlp: bool = True):
        self.model = model
        self.need_mlp = need_mlp
        if not isinstance(model.map_cnn, QuantCNN):
            raise FusedUnsupported("map_cnn is not a QuantCNN (swap_cnn first)")
        if not isinstance(model.query_projector, QuantLinear):
            raise FusedUnsupported("query_projector is not a QuantLinear")
        for p in ("critic.0", "critic.2", "critic.4", "critic.6") if need_mlp else ():
            layer = model.get_submodule(p)
            if type(layer) is not nn.Linear:
                raise FusedUnsupported(f"{p} must be an fp16 nn.Linear (the critic MLP is not quantised)")
        self.P = int(model.critic_proprio_dim)
        if self.P > 104:
            raise FusedUnsupported("critic proprio width above 104")
        # the reference picks the actor's embedding when both widths agree
        # (rsl_rl actor_critic_encoder.py:226-229)
        self.use_actor_emb = self.P == int(model.actor_proprio_dim)
        if self.use_actor_emb and not isinstance(model.actor_proprio_embedding, QuantLinear):
            raise FusedUnsupported("actor_proprio_embedding must be a QuantLinear")
        self.act_mode = model_act_mode(model)
        self._ws: dict[tuple, torch.Tensor] = {}

    def weights(self, obs_norm=None) -> N.GladCriticWeights:
        m = self.model
        w = N.GladCriticWeights()
        w.obs_norm = obs_norm_struct(obs_norm, self.P + 2079)
        w.conv = m.map_cnn.conv_struct()
        if self.use_actor_emb:
            w.proprio_emb_q = N.qlinear_struct(m.actor_proprio_embedding)
        else:
            e = m.critic_proprio_embedding
            w.proprio_emb = N.GladLinear16(_fp16(e.weight, "critic_proprio_embedding.weight").data_ptr(),
                                           N.ptr(e.bias), e.in_features, e.out_features)
        w.query_proj = N.qlinear_struct(m.query_projector)
        w.gps_w = _fp16(m.global_pool_selector.weight, "global_pool_selector.weight").data_ptr()
        w.gps_b = _fp16(m.global_pool_selector.bias, "global_pool_selector.bias").data_ptr()
        w.scorer_w = _fp16(m.topk_scorer.weight, "topk_scorer.weight").data_ptr()
        w.scorer_b = _fp16(m.topk_scorer.bias, "topk_scorer.bias").data_ptr()
        w.mha_in_w = _fp16(m.mha.in_proj_weight, "mha.in_proj_weight").data_ptr()
        w.mha_in_b = _fp16(m.mha.in_proj_bias, "mha.in_proj_bias").data_ptr()
        w.mha_out_w = _fp16(m.mha.out_proj.weight, "mha.out_proj.weight").data_ptr()
        w.mha_out_b = _fp16(m.mha.out_proj.bias, "mha.out_proj.bias").data_ptr()
        for i, p in enumerate(("critic.0", "critic.2", "critic.4", "critic.6")):
            L = m.get_submodule(p)
            if not isinstance(L, nn.Linear):
                if self.need_mlp:
                    raise FusedUnsupported(f"{p} must be an fp16 nn.Linear")
                continue
            w.mlp[i] = N.GladLinear16(_fp16(L.weight, f"{p}.weight").data_ptr(),
                                      N.ptr(_fp16(L.bias, f"{p}.bias")) if L.bias is not None else None,
                                      L.in_features, L.out_features)
        return w

    def check_status(self) -> None:
        """As FusedActor.check_status, for the critic's workspaces."""
        check_workspaces(self._ws, "fused critic")

    def run(self, obs: torch.Tensor, value: torch.Tensor | None, noise: torch.Tensor | None = None,
            obs_norm=None, gumbel: tuple | None = None, aux: N.GladActorAux | None = None) -> None:
        """Launch the fused critic forward on the current stream (no host sync).

        ``noise``: f32 [B,187] added to the top-k logits; ``gumbel = (seed, offset)`` instead
        draws the train-mode Gumbel term inside the kernel (``offset``: one-element int64
        device tensor, advanced by one per call). ``obs_norm``: an EmpiricalNormalization
        applied to the f32 rows as they load. ``value`` None runs the encoder only (``aux``
        must then receive ``encoded``)."""
        N.require_cuda(obs)
        if obs.dim() != 2 or obs.stride(1) != 1:
            raise ValueError("obs must be a row-major [B, P+2079] tensor")
        if noise is not None and gumbel is not None:
            raise ValueError("pass either noise or gumbel")
        B = obs.shape[0]
        key = (B, str(obs.device))
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.zeros(N.load().glad_critic_workspace_size(B), dtype=torch.uint8, device=obs.device)
            self._ws[key] = ws
        dt = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
        if gumbel is not None:
            seed, offset = gumbel
            N.require_cuda(offset)
            if offset.dtype != torch.int64 or offset.numel() != 1:
                raise ValueError("gumbel offset must be a one-element int64 CUDA tensor")
            rc = N.load().glad_critic_forward_train(
                self.weights(obs_norm), obs.data_ptr(), dt, B, obs.stride(0), N.ACT_MODES[self.act_mode],
                int(seed) & 0xFFFFFFFFFFFFFFFF, offset.data_ptr(), N.ptr(value), aux, ws.data_ptr(), ws.numel(),
                N.stream_handle(obs.device))
            N.check(rc, "glad_critic_forward_train")
            return
        rc = N.load().glad_critic_forward(
            self.weights(obs_norm), obs.data_ptr(), dt, B, obs.stride(0), N.ACT_MODES[self.act_mode], N.ptr(noise),
            N.ptr(value), aux, ws.data_ptr(), ws.numel(), N.stream_handle(obs.device))
        N.check(rc, "glad_critic_forward")

    def encode(self, obs: torch.Tensor, noise: torch.Tensor | None = None):
        """``_encode_terrain`` outputs for critic-width observations: (encoded [B,128+P]
        fp16, attn_weights [B,1,32], topk_indices [B,32] int64, gc_weights [B,187,1])."""
        B, dev = obs.shape[0], obs.device
        enc = torch.empty(B, 232, dtype=torch.float16, device=dev)
        attn = torch.empty(B, 1, 32, dtype=torch.float16, device=dev)
        idx = torch.empty(B, 32, dtype=torch.int64, device=dev)
        gcw = torch.empty(B, 187, 1, dtype=torch.float16, device=dev)
        aux = N.GladActorAux()
        aux.encoded, aux.attn_weights, aux.topk_idx, aux.gc_weights = (
            enc.data_ptr(), attn.data_ptr(), idx.data_ptr(), gcw.data_ptr())
        self.run(obs, None, noise, aux=aux)
        return enc[:, :128 + self.P].contiguous(), attn, idx, gcw


class FusedActorCritic:
    """Actor and critic of one rollout step from ONE read of the shared height
    scan (``glad_actor_critic_forward``, eval mode). The critic group must carry
    the same scan as the policy group (as in the reference's benchmarks); its
    proprio columns come first. Results equal FusedActor.run + FusedCritic.run."""

    def __init__(self, model: nn.Module):
        self.actor = FusedActor(model)
        self.critic = FusedCritic(model)
        if self.critic.use_actor_emb:
            raise FusedUnsupported("critic and actor proprio widths agree: the critic reuses the actor "
                                   "embedding, run the two heads separately")
        self._ws: dict[tuple, torch.Tensor] = {}

    def check_status(self) -> None:
        """As FusedActor.check_status, for this call's workspaces and both heads'."""
        check_workspaces(self._ws, "fused actor + critic")
        self.actor.check_status()
        self.critic.check_status()

    def run(self, policy_obs: torch.Tensor, critic_obs: torch.Tensor, mean: torch.Tensor,
            value: torch.Tensor, gumbel: tuple | None = None) -> None:
        """``gumbel=(seed, offset)`` (offset: int64 device tensor of one element) runs the
        train-mode rollout forward: each head adds its own in-kernel Gumbel term, the actor
        at offset[0], the critic at offset[0] + 1; the call adds two to offset[0]."""
        N.require_cuda(policy_obs)
        N.require_cuda(critic_obs)
        if policy_obs.dtype != critic_obs.dtype or policy_obs.shape[0] != critic_obs.shape[0]:
            raise ValueError("policy and critic groups must share dtype and batch")
        if policy_obs.stride(1) != 1 or critic_obs.stride(1) != 1:
            raise ValueError("observation rows must be contiguous")
        B = policy_obs.shape[0]
        key = (B, str(policy_obs.device))
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.zeros(N.load().glad_actor_critic_workspace_size(B), dtype=torch.uint8,
                             device=policy_obs.device)
            self._ws[key] = ws
        dt = N.DTYPE_F32 if policy_obs.dtype == torch.float32 else N.DTYPE_F16
        if gumbel is None:
            rc = N.load().glad_actor_critic_forward(
                self.actor.weights(), self.critic.weights(), policy_obs.data_ptr(), critic_obs.data_ptr(), dt,
                B, policy_obs.stride(0), critic_obs.stride(0), N.ACT_MODES[self.actor.act_mode],
                mean.data_ptr(), value.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(policy_obs.device))
            N.check(rc, "glad_actor_critic_forward")
            return
        seed, offset = gumbel
        if offset.dtype != torch.int64 or offset.device != policy_obs.device or offset.numel() < 1:
            raise ValueError("gumbel offset must be an int64 tensor on the observations' device")
        rc = N.load().glad_actor_critic_forward_train(
            self.actor.weights(), self.critic.weights(), policy_obs.data_ptr(), critic_obs.data_ptr(), dt,
            B, policy_obs.stride(0), critic_obs.stride(0), N.ACT_MODES[self.actor.act_mode],
            int(seed) & (2 ** 64 - 1), offset.data_ptr(), mean.data_ptr(), value.data_ptr(), ws.data_ptr(),
            ws.numel(), N.stream_handle(policy_obs.device))
        N.check(rc, "glad_actor_critic_forward_train")


def ppo_epilogue(mean: torch.Tensor, std: torch.Tensor, seed: int, rng_state: torch.Tensor,
                 actions: torch.Tensor, log_prob: torch.Tensor, sigma: torch.Tensor | None = None) -> None:
    """PPO.act epilogue (``glad_ppo_epilogue``, rsl_rl/algorithms/ppo.py:129-140): actions
    sampled from Normal(mean, std) and their summed log-probability. ``rng_state`` is an
    int64 device tensor of two elements {offset, scratch} (zero-initialised once); each
    call uses offset rng_state[0] and adds one to it on the device."""
    N.require_cuda(mean)
    B, n = mean.shape
    for t, nm in ((mean, "mean"), (std, "std"), (actions, "actions"), (log_prob, "log_prob")):
        if t.dtype != torch.float32 or t.device != mean.device:
            raise ValueError(f"{nm} must be float32 on the device of mean")
    if mean.stride(1) != 1 or actions.stride(1) != 1 or not std.is_contiguous() or std.numel() != n:
        raise ValueError("mean/actions rows must be contiguous and std must hold one value per action")
    if actions.shape != mean.shape or log_prob.numel() != B:
        raise ValueError("actions must match mean and log_prob must hold one value per row")
    if rng_state.dtype != torch.int64 or rng_state.numel() < 2 or rng_state.device != mean.device:
        raise ValueError("rng_state must be an int64 device tensor of two elements")
    if sigma is not None and (sigma.dtype != torch.float32 or not sigma.is_contiguous() or sigma.shape != mean.shape):
        raise ValueError("sigma must be a contiguous float32 tensor shaped like mean")
    rc = N.load().glad_ppo_epilogue(mean.data_ptr(), B, mean.stride(0), std.data_ptr(), n,
                                    int(seed) & (2 ** 64 - 1), rng_state.data_ptr(), actions.data_ptr(),
                                    actions.stride(0), log_prob.data_ptr(),
                                    sigma.data_ptr() if sigma is not None else None,
                                    N.stream_handle(mean.device))
    N.check(rc, "glad_ppo_epilogue")
