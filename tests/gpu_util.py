"""Helpers of the GPU tests: golden/oracle weights -> CUDA tensors -> C-ABI structs."""
from __future__ import annotations

import numpy as np
import torch

from rl_quant_b200 import _native as N

QL_NAMES = ("actor_proprio_embedding", "query_projector", "actor.0", "actor.2", "actor.4", "actor.6")


def fp16_ulp_close(a, b, max_ulp=1, min_exact=0.999):
    """fp16 arrays equal except for rare one-ulp differences (the conv2
    epilogue runs with fused multiply-adds; qrt's eager order rounds twice)."""
    a = np.asarray(a, np.float16).astype(np.float32)
    b = np.asarray(b, np.float16).astype(np.float32)
    ulp = np.maximum(np.spacing(np.maximum(np.abs(a), np.abs(b)).astype(np.float16)).astype(np.float32),
                     np.float32(2.0 ** -24))
    d = np.abs(a - b) / ulp
    assert d.max() <= max_ulp + 1e-6, float(d.max())
    assert (d == 0).mean() >= min_exact, float((d == 0).mean())


class DeviceWeights:
    """Every tensor of the golden state dict on the GPU (kept alive here)."""

    def __init__(self, sd: dict, device="cuda"):
        self.t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in sd.items()
                  if isinstance(v, np.ndarray) and v.dtype != np.int64}
        self.keep = []

    def __getitem__(self, k):
        return self.t[k]

    def conv(self) -> N.GladConvWeights:
        g = lambda k: self.t[f"map_cnn.{k}"]  # noqa: E731
        return N.conv_weights(g("w1p"), g("b1f"), g("qa"), g("qc"), g("w8"), g("dq"), g("b2f"), g("a2"), g("c2"))

    def ql(self, name: str) -> N.GladQLinear:
        t = self.t
        w = t[f"{name}.weight"]
        alpha = t.get(f"{name}.alpha")
        beta = t.get(f"{name}.beta")
        return N.GladQLinear(N.ptr(t[f"{name}.w8"]), N.ptr(t[f"{name}.dq_scale"]), N.ptr(t[f"{name}.s_w"]),
                             N.ptr(t[f"{name}.b_prime"]), N.ptr(alpha), N.ptr(beta), N.ptr(t[f"{name}.s_z"]),
                             N.ptr(t[f"{name}.inv_sz"]), int(w.shape[1]), int(w.shape[0]))

    def actor(self) -> N.GladActorWeights:
        t = self.t
        w = N.GladActorWeights()
        w.conv = self.conv()
        w.proprio_emb = self.ql("actor_proprio_embedding")
        w.query_proj = self.ql("query_projector")
        w.gps_w, w.gps_b = N.ptr(t["global_pool_selector.weight"]), N.ptr(t["global_pool_selector.bias"])
        w.scorer_w, w.scorer_b = N.ptr(t["topk_scorer.weight"]), N.ptr(t["topk_scorer.bias"])
        w.mha_in_w, w.mha_in_b = N.ptr(t["mha.in_proj_weight"]), N.ptr(t["mha.in_proj_bias"])
        w.mha_out_w, w.mha_out_b = N.ptr(t["mha.out_proj.weight"]), N.ptr(t["mha.out_proj.bias"])
        for i, n in enumerate(("actor.0", "actor.2", "actor.4", "actor.6")):
            w.mlp[i] = self.ql(n)
        return w


def critic_weights(dw: DeviceWeights) -> N.GladCriticWeights:
    t = dw.t
    w = N.GladCriticWeights()
    w.conv = dw.conv()
    e = t["critic_proprio_embedding.weight"]
    w.proprio_emb = N.GladLinear16(e.data_ptr(), t["critic_proprio_embedding.bias"].data_ptr(),
                                   int(e.shape[1]), int(e.shape[0]))
    w.query_proj = dw.ql("query_projector")
    w.gps_w, w.gps_b = N.ptr(t["global_pool_selector.weight"]), N.ptr(t["global_pool_selector.bias"])
    w.scorer_w, w.scorer_b = N.ptr(t["topk_scorer.weight"]), N.ptr(t["topk_scorer.bias"])
    w.mha_in_w, w.mha_in_b = N.ptr(t["mha.in_proj_weight"]), N.ptr(t["mha.in_proj_bias"])
    w.mha_out_w, w.mha_out_b = N.ptr(t["mha.out_proj.weight"]), N.ptr(t["mha.out_proj.bias"])
    for i, n in enumerate(("critic.0", "critic.2", "critic.4", "critic.6")):
        W = t[f"{n}.weight"]
        w.mlp[i] = N.GladLinear16(W.data_ptr(), t[f"{n}.bias"].data_ptr(), int(W.shape[1]), int(W.shape[0]))
    return w


def critic_forward(dw: DeviceWeights, obs: torch.Tensor, act_mode: str, with_aux=True):
    B, dev = obs.shape[0], obs.device
    value = torch.empty(B, 1, dtype=torch.float32, device=dev)
    aux = N.GladActorAux()
    aux_t = {}
    if with_aux:
        aux_t = {"topk_logits": torch.empty(B, 187, dtype=torch.float16, device=dev),
                 "topk_idx": torch.empty(B, 32, dtype=torch.int64, device=dev),
                 "encoded": torch.empty(B, 232, dtype=torch.float16, device=dev),
                 "local": torch.empty(B, 187, 64, dtype=torch.float16, device=dev),
                 "attn_weights": torch.empty(B, 32, dtype=torch.float16, device=dev),
                 "proprio_emb": torch.empty(B, 64, dtype=torch.float16, device=dev),
                 "query": torch.empty(B, 64, dtype=torch.float16, device=dev)}
        for k, v in aux_t.items():
            setattr(aux, k, v.data_ptr())
    lib = N.load()
    nbytes = lib.glad_critic_workspace_size(B)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    dtype = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
    N.check(lib.glad_critic_forward(critic_weights(dw), obs.data_ptr(), dtype, B, obs.stride(0),
                                    N.ACT_MODES[act_mode], None, value.data_ptr(), aux, ws.data_ptr(), nbytes,
                                    N.stream_handle()), "glad_critic_forward")
    st = N.c_uint32(0)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "device status")
    torch.cuda.synchronize()
    return value, aux_t


def actor_critic_forward(dw: DeviceWeights, policy_obs: torch.Tensor, critic_obs: torch.Tensor, act_mode: str):
    """glad_actor_critic_forward (one read of the shared scan); returns (mean, value)."""
    B, dev = policy_obs.shape[0], policy_obs.device
    mean = torch.empty(B, 29, dtype=torch.float32, device=dev)
    value = torch.empty(B, 1, dtype=torch.float32, device=dev)
    lib = N.load()
    nbytes = lib.glad_actor_critic_workspace_size(B)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    dtype = N.DTYPE_F32 if policy_obs.dtype == torch.float32 else N.DTYPE_F16
    N.check(lib.glad_actor_critic_forward(dw.actor(), critic_weights(dw), policy_obs.data_ptr(), critic_obs.data_ptr(),
                                          dtype, B, policy_obs.stride(0), critic_obs.stride(0),
                                          N.ACT_MODES[act_mode], mean.data_ptr(), value.data_ptr(), ws.data_ptr(),
                                          nbytes, N.stream_handle()), "glad_actor_critic_forward")
    st = N.c_uint32(0)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "device status")
    torch.cuda.synchronize()
    return mean, value


def actor_forward(dw: DeviceWeights, obs: torch.Tensor, act_mode: str, noise=None, with_aux=True):
    """Run glad_actor_forward; returns (mean, aux dict of tensors)."""
    B = obs.shape[0]
    dev = obs.device
    mean = torch.empty(B, 29, dtype=torch.float32, device=dev)
    aux_t = {}
    aux = N.GladActorAux()
    if with_aux:
        aux_t = {
            "z8": torch.empty(B * 187, 16, dtype=torch.int8, device=dev),
            "local": torch.empty(B, 187, 64, dtype=torch.float16, device=dev),
            "gc_weights": torch.empty(B, 187, dtype=torch.float16, device=dev),
            "score_local": torch.empty(B, 187, dtype=torch.float16, device=dev),
            "topk_logits": torch.empty(B, 187, dtype=torch.float16, device=dev),
            "topk_idx": torch.empty(B, 32, dtype=torch.int64, device=dev),
            "attn_weights": torch.empty(B, 32, dtype=torch.float16, device=dev),
            "encoded": torch.empty(B, 224, dtype=torch.float16, device=dev),
            "act_scales": torch.empty(6, dtype=torch.float32, device=dev),
            "proprio_emb": torch.empty(B, 64, dtype=torch.float16, device=dev),
            "query": torch.empty(B, 64, dtype=torch.float16, device=dev),
        }
        for k, v in aux_t.items():
            setattr(aux, k, v.data_ptr())
    lib = N.load()
    ws_bytes = lib.glad_actor_workspace_size(B)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    w = dw.actor()
    dtype = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
    rc = lib.glad_actor_forward(w, obs.data_ptr(), dtype, B, obs.stride(0), N.ACT_MODES[act_mode],
                                N.ptr(noise), mean.data_ptr(), aux, ws.data_ptr(), ws_bytes,
                                N.stream_handle())
    N.check(rc, "glad_actor_forward")
    st = N.c_uint32(0)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "device status")
    torch.cuda.synchronize()
    return mean, aux_t


def actor_forward_train(dw: DeviceWeights, obs: torch.Tensor, act_mode: str, seed: int, offset: torch.Tensor):
    """glad_actor_forward_train (in-kernel Gumbel); returns (mean, aux)."""
    B, dev = obs.shape[0], obs.device
    mean = torch.empty(B, 29, dtype=torch.float32, device=dev)
    aux_t = {"topk_logits": torch.empty(B, 187, dtype=torch.float16, device=dev),
             "topk_idx": torch.empty(B, 32, dtype=torch.int64, device=dev)}
    aux = N.GladActorAux()
    for k, v in aux_t.items():
        setattr(aux, k, v.data_ptr())
    lib = N.load()
    nbytes = lib.glad_actor_workspace_size(B)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    dtype = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
    N.check(lib.glad_actor_forward_train(dw.actor(), obs.data_ptr(), dtype, B, obs.stride(0),
                                         N.ACT_MODES[act_mode], seed, offset.data_ptr(), mean.data_ptr(), aux,
                                         ws.data_ptr(), nbytes, N.stream_handle()), "glad_actor_forward_train")
    st = N.c_uint32(0)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "device status")
    torch.cuda.synchronize()
    return mean, aux_t


def golden_model(w):
    """fp16 GLAD copy with the golden state dict and the reference's LET plan,
    swapped/patched through the package API exactly as qrt's integration does."""
    from oracle import glad_oracle as O
    from rl_quant_b200 import patch_encoder, swap, swap_cnn
    from rl_quant_b200.glad_model import build_glad
    QL = O.GladWeights.QL
    m = build_glad(seed=0, critic_seed=2).cuda()
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()
          if not k.startswith(("plan.", "meta.")) and k in m.state_dict()}
    m.load_state_dict(sd, strict=False)
    m = m.half().eval()
    plan = {p: {"s_z": float(w[f"plan.{p}.s_z"]), "alpha": torch.from_numpy(w[f"{p}.alpha"]).cuda(),
                "beta": torch.from_numpy(w[f"{p}.beta"]).cuda(), "act_mode": "dynamic"} for p in QL}
    # load the plain weights first (the golden file has the inference copy's params)
    for p in QL:
        lin = m.get_submodule(p)
        lin.weight.data.copy_(torch.from_numpy(w[f"{p}.weight"]))
        lin.bias.data.copy_(torch.from_numpy(w[f"{p}.bias"]))
    swapped = swap.apply(m, plan)
    swap_cnn(m, float(w["meta.s_cnn"]))
    patch_encoder(m)
    return m.eval(), swapped


class EmpiricalNorm(torch.nn.Module):
    """rsl_rl's EmpiricalNormalization restated for the tests (rsl_rl/networks/
    normalization.py:14-80): running mean/var buffers updated in place, _std
    recomputed as sqrt(_var), forward (x - mean) / (std + eps)."""

    def __init__(self, n, eps=1e-2):
        super().__init__()
        self.eps = eps
        self.register_buffer("_mean", torch.zeros(n).unsqueeze(0))
        self.register_buffer("_var", torch.ones(n).unsqueeze(0))
        self.register_buffer("_std", torch.ones(n).unsqueeze(0))
        self.register_buffer("count", torch.tensor(0, dtype=torch.long))

    def forward(self, x):
        return (x - self._mean) / (self._std + self.eps)

    @torch.no_grad()
    def update(self, x):
        count_x = x.shape[0]
        self.count += count_x
        rate = count_x / self.count
        var_x = torch.var(x, dim=0, unbiased=False, keepdim=True)
        mean_x = torch.mean(x, dim=0, keepdim=True)
        delta_mean = mean_x - self._mean
        self._mean += rate * delta_mean
        self._var += rate * (var_x - self._var + delta_mean * (mean_x - self._mean))
        self._std = torch.sqrt(self._var)
