"""LET calibration of qrt's INT8 linears -> the plan ``swap.apply`` consumes.

The reference builds this plan in qrt/calib.py:62-129 with quant/let.py:140-233.
Here it is three small pieces:

  * ``record_inputs``  runs the model on calibration batches and keeps, for each
    quantised Linear, the rows of its input (at most ``max_rows // n_batches``
    per batch, picked at random);
  * ``fit_layer``      fits OmniQuant's learnable equivalent transformation
    (``LETQuantizer``) of one Linear's input with Adam on the block
    reconstruction loss, then measures the static activation scale;
  * ``make_plan``      returns ``{path: {"s_z", "alpha", "beta", "act_mode"}}``.

Random row picks come from one ``torch.Generator`` seeded by ``seed``. They are
drawn in the order the reference draws them from torch's global generator: one
pick per recorded input per batch (layers in forward order), then one pick per
fitting step, layer after layer. A reference run seeded with
``torch.manual_seed(seed)`` on the CPU therefore picks the same rows and ends
with the same alpha, beta and s_z (tests/test_calib.py).
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .let import LETQuantizer


def _pick(gen: torch.Generator, n: int, k: int, device) -> torch.Tensor:
    """k row indices in [0, n), drawn with replacement on the generator's device."""
    return torch.randint(0, n, (k,), generator=gen, device=gen.device).to(device)


@torch.no_grad()
def record_inputs(model: nn.Module, paths: list[str], obs_fn, n_batches: int, gen: torch.Generator,
                  max_rows: int = 16384) -> dict[str, torch.Tensor]:
    """The fp32 input rows each module in ``paths`` sees over ``n_batches`` calls of
    ``model.act_inference(obs_fn())`` in eval mode, ``{path: [rows, in_features]}``."""
    budget = max_rows // n_batches
    seen: dict[str, list[torch.Tensor]] = {p: [] for p in paths}

    def recorder(path):
        def record(module, args, output):
            rows = args[0].detach().flatten(0, -2)
            if rows.shape[0] > budget:
                rows = rows[_pick(gen, rows.shape[0], budget, rows.device)]
            seen[path].append(rows.float())
        return record

    handles = [model.get_submodule(p).register_forward_hook(recorder(p)) for p in paths]
    training = model.training
    model.eval()
    try:
        with torch.inference_mode():
            for _ in range(n_batches):
                model.act_inference(obs_fn())
    finally:
        for h in handles:
            h.remove()
        model.train(training)
    return {p: torch.cat(rows, dim=0) for p, rows in seen.items()}


@dataclass
class LetFit:
    """Result of ``fit_layer``: the transform, the activation scale over all the
    recorded rows, and the reconstruction loss of every step (when kept)."""
    alpha: torch.Tensor
    beta: torch.Tensor
    s_z: float
    losses: list[float] = field(default_factory=list)


def fit_layer(rows: torch.Tensor, linear: nn.Linear, gen: torch.Generator, steps: int = 200, lr: float = 5e-3,
              batch_rows: int = 4096, keep_losses: bool = False) -> LetFit:
    """Fit ``z = alpha * x + beta`` for one Linear on an fp32 copy of it.

    Start from the per-channel statistics of ``rows`` (alpha = 1/std, beta =
    -mean/std), then ``steps`` Adam steps on MSE(Qw(W') Qa(z) + b', W x + b), each
    on ``batch_rows`` rows drawn with replacement. ``s_z = absmax(alpha x + beta) / 127``
    over every row."""
    target = copy.deepcopy(linear).float().requires_grad_(False)
    x = rows.float()
    let = LETQuantizer(target.in_features).to(x.device)
    let.initialize_from_activation(x)
    opt = torch.optim.Adam(let.parameters(), lr=lr)
    take = min(batch_rows, x.shape[0])
    losses = []
    for _ in range(steps):
        sample = x[_pick(gen, x.shape[0], take, x.device)]
        with torch.enable_grad():
            loss = let.block_reconstruction_loss(sample, target)[1]
            opt.zero_grad()
            loss.backward()
        opt.step()
        if keep_losses:
            losses.append(float(loss))
    return LetFit(let.alpha.detach().clone(), let.beta.detach().clone(), let.calibrate_scale(x), losses)


def make_plan(model: nn.Module, paths: list[str], obs_fn=None, use_let: bool = True, n_calib: int = 8,
              let_steps: int = 200, act_mode: str = "static", verbose: bool = True,
              seed: int = 0) -> dict[str, dict]:
    """The ``swap.apply`` plan for the Linears at ``paths`` (qrt/calib.py:93-129 interface).

    ``use_let=True``: LET per layer (alpha, beta, the calibrated s_z); ``use_let=False``:
    plain absmax PTQ (s_z = absmax(x) / 127, no transform); ``act_mode="dynamic_full"``
    needs no calibration data (every scale is computed at run time). ``seed`` seeds the
    row picks (an extension of the reference signature, whose picks are unseeded)."""
    if act_mode == "dynamic_full":
        return {p: {"s_z": None, "alpha": None, "beta": None, "act_mode": act_mode} for p in paths}
    gen = torch.Generator().manual_seed(int(seed))
    recorded = record_inputs(model, paths, obs_fn, n_calib, gen)
    plan: dict[str, dict] = {}
    for path in paths:
        rows = recorded[path]
        if not use_let:
            s_z = rows.abs().amax().item() / 127.0
            plan[path] = {"s_z": s_z, "alpha": None, "beta": None, "act_mode": act_mode}
            if verbose:
                print(f"[rl_quant_b200] absmax scale of {path}: {s_z:.4g}")
            continue
        fit = fit_layer(rows, model.get_submodule(path), gen, steps=let_steps, keep_losses=verbose)
        plan[path] = {"s_z": fit.s_z, "alpha": fit.alpha, "beta": fit.beta, "act_mode": act_mode}
        if verbose:
            first, last = (fit.losses[0], fit.losses[-1]) if fit.losses else (float("nan"),) * 2
            print(f"[rl_quant_b200] LET of {path}: {rows.shape[0]} rows x {rows.shape[1]}, "
                  f"loss {first:.3e} -> {last:.3e}, s_z {fit.s_z:.4g}")
    return plan
