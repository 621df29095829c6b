"""LET: learnable equivalent transformation of a Linear's input (OmniQuant,
Shao et al. 2023, section 3), as used by qrt's calibration
(quant/let.py:59-233 of the reference).

For a Linear ``y = W x + b`` the per-input-channel transform
``z = alpha * x + beta`` is folded into the weights as ``W' = W / alpha`` and
``b' = b - W' beta`` so that ``W' z + b' == W x + b`` exactly. Calibration
fits ``alpha, beta`` by minimising the reconstruction error of the quantised
block ``Qw(W') Qa(z) + b'`` against the float output, with straight-through
rounding; activations are per-tensor symmetric int8, weights per output
channel.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

QMAX, QMIN = 127, -128


def _ste_round(x: torch.Tensor) -> torch.Tensor:
    return x + (x.round() - x).detach()


def fake_quant_act(z: torch.Tensor) -> torch.Tensor:
    """Per-tensor absmax int8 fake-quantisation with STE (quant/let.py:108-114)."""
    scale = z.detach().abs().amax().clamp_min(1e-8) / QMAX
    return _ste_round((z / scale).clamp(QMIN, QMAX)) * scale


def fake_quant_weight(w: torch.Tensor) -> torch.Tensor:
    """Per-output-channel absmax int8 fake-quantisation with STE (quant/let.py:116-126)."""
    scale = w.detach().abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / QMAX
    return _ste_round((w / scale).clamp(QMIN, QMAX)) * scale


class LETQuantizer(nn.Module):
    """Learnable ``alpha`` (scale) and ``beta`` (shift) of one Linear's input."""

    def __init__(self, n_channels: int):
        super().__init__()
        self.n_channels = n_channels
        self.alpha = nn.Parameter(torch.ones(n_channels))
        self.beta = nn.Parameter(torch.zeros(n_channels))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Fake-quantised ``x`` seen through the transform (quant/let.py:130-138)."""
        z = self.alpha * x + self.beta
        return (fake_quant_act(z) - self.beta) / self.alpha.clamp_min(1e-8)

    def folded(self, linear: nn.Linear) -> tuple[torch.Tensor, torch.Tensor]:
        """``(W', b')`` with ``W' = W/alpha``, ``b' = b - W' beta``."""
        w = linear.weight.detach() / self.alpha.unsqueeze(0)
        b = linear.bias.detach() if linear.bias is not None else torch.zeros_like(w[:, 0])
        return w, b - (w * self.beta.unsqueeze(0)).sum(dim=1)

    def block_reconstruction_loss(self, x: torch.Tensor, linear: nn.Linear):
        """MSE(Qw(W') Qa(z) + b', W x + b) (quant/let.py:140-189).

        The bias correction uses the exact ``W'`` while the product uses the
        quantised one, so ``beta`` receives the weight-quantisation error as
        its gradient."""
        with torch.no_grad():
            target = F.linear(x, linear.weight, linear.bias)
        zq = fake_quant_act(self.alpha * x + self.beta)
        w, b = self.folded(linear)
        y = F.linear(zq, fake_quant_weight(w), b)
        return y, F.mse_loss(y, target)

    @torch.no_grad()
    def initialize_from_activation(self, x: torch.Tensor) -> None:
        """alpha = 1/std, beta = -mean/std per channel (quant/let.py:193-207)."""
        flat = x.detach().reshape(-1, self.n_channels)
        sigma = flat.std(dim=0).clamp_min(1e-8)
        self.alpha.copy_(1.0 / sigma)
        self.beta.copy_(-flat.mean(dim=0) / sigma)

    @torch.no_grad()
    def calibrate_scale(self, x: torch.Tensor) -> float:
        """Static activation scale absmax(alpha x + beta)/127 (quant/let.py:217-233)."""
        z = self.alpha * x + self.beta
        return max(z.abs().amax().item() / QMAX, 1e-8)
