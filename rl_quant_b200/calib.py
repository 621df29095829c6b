"""Calibration pipeline: activation capture -> LET fit -> swap plan
(qrt/calib.py:25-129).

Difference from the reference: row sampling draws from an explicit
``torch.Generator`` (seeded by ``seed``) instead of the global RNG, so a plan
is reproducible.
"""
from __future__ import annotations

import copy

import torch
import torch.nn as nn

from .let import LETQuantizer


@torch.no_grad()
def collect_inputs(model: nn.Module, paths: list[str], obs_fn, n_batches: int = 8,
                   max_rows: int = 16384, generator: torch.Generator | None = None) -> dict[str, torch.Tensor]:
    """Inputs of each layer in ``paths`` over ``n_batches`` of ``obs_fn()``
    (rows subsampled to ``max_rows``), as ``{path: [S, K] fp32}``."""
    feats: dict[str, list[torch.Tensor]] = {p: [] for p in paths}
    per = max(1, max_rows // n_batches)

    def hook(p):
        def fn(mod, inp, out):
            x = inp[0].detach().reshape(-1, inp[0].shape[-1])
            if x.shape[0] > per:
                idx = torch.randint(0, x.shape[0], (per,), generator=generator,
                                    device="cpu" if generator is not None else x.device).to(x.device)
                x = x[idx]
            feats[p].append(x.float())
        return fn

    hooks = [model.get_submodule(p).register_forward_hook(hook(p)) for p in paths]
    was = model.training
    model.eval()
    try:
        with torch.inference_mode():
            for _ in range(n_batches):
                model.act_inference(obs_fn())
    finally:
        model.train(was)
        for h in hooks:
            h.remove()
    return {p: torch.cat(v, dim=0) for p, v in feats.items()}


def fit_let(x: torch.Tensor, linear: nn.Linear, n_steps: int = 200, lr: float = 5e-3,
            batch_rows: int = 4096, generator: torch.Generator | None = None,
            verbose: bool = False) -> tuple[torch.Tensor, torch.Tensor, float]:
    """Fit LET (alpha, beta) for one layer on an fp32 copy; returns (alpha, beta, s_z)."""
    lin32 = copy.deepcopy(linear).float()
    for p in lin32.parameters():
        p.requires_grad_(False)
    x = x.float()
    let = LETQuantizer(lin32.in_features).to(x.device)
    let.initialize_from_activation(x)
    opt = torch.optim.Adam(let.parameters(), lr=lr)
    rows = min(batch_rows, x.shape[0])
    for i in range(n_steps):
        idx = torch.randint(0, x.shape[0], (rows,), generator=generator,
                            device="cpu" if generator is not None else x.device).to(x.device)
        with torch.enable_grad():
            _, loss = let.block_reconstruction_loss(x[idx], lin32)
            opt.zero_grad()
            loss.backward()
        opt.step()
        if verbose and (i + 1) % 50 == 0:
            print(f"      step {i + 1:4d}  recon_loss={loss.item():.3e}")
    return let.alpha.detach().clone(), let.beta.detach().clone(), let.calibrate_scale(x)


def make_plan(model: nn.Module, paths: list[str], obs_fn=None, use_let: bool = True,
              n_calib: int = 8, let_steps: int = 200, act_mode: str = "static",
              verbose: bool = True, seed: int = 0) -> dict[str, dict]:
    """Capture -> (LET) -> scale -> ``swap.apply`` plan (qrt/calib.py:93-129).

    ``use_let=False`` gives the naive PTQ plan (no alpha/beta, s_z = absmax/127);
    ``act_mode="dynamic_full"`` needs no calibration data at all."""
    if act_mode == "dynamic_full":
        return {p: {"s_z": None, "alpha": None, "beta": None, "act_mode": act_mode} for p in paths}
    gen = torch.Generator().manual_seed(int(seed))
    acts = collect_inputs(model, paths, obs_fn, n_batches=n_calib, generator=gen)
    plan: dict[str, dict] = {}
    for p in paths:
        lin = model.get_submodule(p)
        x = acts[p]
        if use_let:
            if verbose:
                print(f"  [calib/LET] {p}  (K={lin.in_features}, samples={x.shape[0]})")
            alpha, beta, s_z = fit_let(x, lin, n_steps=let_steps, generator=gen, verbose=verbose)
            plan[p] = {"s_z": s_z, "alpha": alpha, "beta": beta, "act_mode": act_mode}
        else:
            s_z = x.abs().amax().item() / 127.0
            if verbose:
                print(f"  [calib/naive] {p}  s_z={s_z:.4g}")
            plan[p] = {"s_z": s_z, "alpha": None, "beta": None, "act_mode": act_mode}
    return plan
