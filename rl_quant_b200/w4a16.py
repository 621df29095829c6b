"""W4A16 actor MLP: int4 weights, fp16 activations.

The reference names INT4 only as future work (README.md:259), so the format is
this package's own (the C ABI documents it in ``include/glad_b200.h``):
symmetric int4 q in [-8, 7] per weight, one fp16 scale per 64 consecutive
inputs of a row (s = absmax / 7, round half to even), two weights per byte
along K (even k in the low nibble). A layer computes
``fp16(x @ fp16(q * s)^T + b)`` with fp32 accumulation and ELU between layers.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _native as N

GROUP = 64


@torch.no_grad()
def quantize_w4(weight: torch.Tensor, group: int = GROUP):
    """weight [N, K] -> (packed uint8 [N, K/2], scales fp16 [N, ceil(K/group)])."""
    W = weight.detach().float()
    Nn, K = W.shape
    if K % 2:
        raise ValueError("K must be even")
    G = (K + group - 1) // group
    Wp = torch.zeros(Nn, G * group, dtype=torch.float32, device=W.device)
    Wp[:, :K] = W
    s = (Wp.view(Nn, G, group).abs().amax(dim=-1) / 7.0).half()
    sf = s.float()
    sf = torch.where(sf > 0, sf, torch.ones_like(sf))
    q = torch.round(Wp.view(Nn, G, group) / sf[..., None]).clamp_(-8, 7).to(torch.int16).view(Nn, G * group)[:, :K]
    q = (q & 0xF).to(torch.uint8)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).contiguous()
    return packed, s.contiguous()


class W4A16MLP(nn.Module):
    """The actor MLP 224->512->256->128->29 of an rsl_rl actor (``actor.0/2/4/6``) in
    W4A16 form. ``forward(encoded)`` and ``actor_forward`` run the fused kernel."""

    def __init__(self, linears):
        super().__init__()
        if len(linears) != 4:
            raise ValueError("four Linear layers expected")
        shapes = [(l.out_features, l.in_features) for l in linears]
        if shapes != [(512, 224), (256, 512), (128, 256), (29, 128)]:
            raise ValueError(f"unexpected actor MLP shapes {shapes}")
        self.src = list(linears)
        dev = linears[0].weight.device
        for i, l in enumerate(linears):
            packed, scales = quantize_w4(l.weight)
            self.register_buffer(f"packed{i}", packed.to(dev))
            self.register_buffer(f"scales{i}", scales.to(dev))
            self.register_buffer(f"bias{i}", (l.bias.detach().half() if l.bias is not None
                                             else torch.zeros(l.out_features, dtype=torch.float16)).to(dev))

    @classmethod
    def from_actor(cls, actor: nn.Module):
        return cls([actor[i] for i in (0, 2, 4, 6)])

    @torch.no_grad()
    def requantize_(self):
        """Re-pack from the source Linear weights in place (fixed buffer addresses)."""
        for i, l in enumerate(self.src):
            packed, scales = quantize_w4(l.weight)
            getattr(self, f"packed{i}").copy_(packed)
            getattr(self, f"scales{i}").copy_(scales)
            if l.bias is not None:
                getattr(self, f"bias{i}").copy_(l.bias.detach().half())
        return self

    def layers(self):
        arr = (N.GladW4Linear * 4)()
        for i, (k, n) in enumerate(((224, 512), (512, 256), (256, 128), (128, 29))):
            arr[i] = N.GladW4Linear(getattr(self, f"packed{i}").data_ptr(), getattr(self, f"scales{i}").data_ptr(),
                                    getattr(self, f"bias{i}").data_ptr(), k, n)
        return arr

    @torch.no_grad()
    def forward(self, encoded: torch.Tensor) -> torch.Tensor:
        N.require_cuda(encoded)
        if encoded.dtype != torch.float16 or encoded.dim() != 2 or encoded.shape[1] < 224:
            raise ValueError("encoded must be fp16 [M, >=224]")
        mean = torch.empty(encoded.shape[0], 29, dtype=torch.float32, device=encoded.device)
        N.check(N.load().glad_w4a16_mlp_forward(self.layers(), encoded.data_ptr(), encoded.shape[0],
                                                encoded.stride(0), mean.data_ptr(),
                                                N.stream_handle(encoded.device)), "glad_w4a16_mlp_forward")
        return mean

    @torch.no_grad()
    def actor_forward(self, fused_actor, obs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The whole actor with the INT8 encoder of ``fused_actor`` (a FusedActor) and this MLP."""
        N.require_cuda(obs)
        B = obs.shape[0]
        mean = out if out is not None else torch.empty(B, 29, dtype=torch.float32, device=obs.device)
        ws = fused_actor.workspace(B, obs.device)
        dt = N.DTYPE_F32 if obs.dtype == torch.float32 else N.DTYPE_F16
        N.check(N.load().glad_actor_forward_w4a16(
            fused_actor.weights(), self.layers(), obs.data_ptr(), dt, B, obs.stride(0),
            N.ACT_MODES[fused_actor.act_mode], mean.data_ptr(), ws.data_ptr(), ws.numel(),
            N.stream_handle(obs.device)), "glad_actor_forward_w4a16")
        return mean
