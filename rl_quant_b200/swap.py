"""Module surgery: nn.Linear <-> QuantLinear (qrt/swap.py:39-74).

The swap moves the source layer's Parameter objects into the QuantLinear
(no copies), so optimisers created before or after stay valid, and both
directions carry over the train/eval flag.
"""
from __future__ import annotations

import torch.nn as nn

from .qlinear import QuantLinear


def get_module(model: nn.Module, path: str) -> nn.Module:
    return model.get_submodule(path)


def set_module(model: nn.Module, path: str, mod: nn.Module) -> None:
    parent_path, _, name = path.rpartition(".")
    parent = model.get_submodule(parent_path) if parent_path else model
    if name.isdigit() and isinstance(parent, (nn.Sequential, nn.ModuleList)):
        parent[int(name)] = mod
    else:
        setattr(parent, name, mod)


def apply(model: nn.Module, plan: dict[str, dict]) -> dict[str, QuantLinear]:
    """Swap every ``plan`` path to a QuantLinear.
    ``plan = {path: {"s_z": float|None, "alpha": Tensor|None, "beta": Tensor|None, "act_mode": str}}``."""
    swapped: dict[str, QuantLinear] = {}
    for path, cfg in plan.items():
        lin = get_module(model, path)
        assert isinstance(lin, nn.Linear), f"{path} is not an nn.Linear: {type(lin)}"
        q = QuantLinear(lin, s_z=cfg.get("s_z"), alpha=cfg.get("alpha"), beta=cfg.get("beta"),
                        act_mode=cfg.get("act_mode", "static"))
        q.train(lin.training)
        set_module(model, path, q)
        swapped[path] = q
    return swapped


def restore(model: nn.Module, swapped: dict[str, QuantLinear]) -> None:
    """Put plain nn.Linear shells (holding the same Parameters) back."""
    for path, q in swapped.items():
        lin = nn.Linear(q.in_features, q.out_features, bias=q.bias is not None,
                        device=q.weight.device, dtype=q.weight.dtype)
        lin.weight = q.weight
        if q.bias is not None:
            lin.bias = q.bias
        lin.train(q.training)
        set_module(model, path, lin)


def refresh(swapped: dict[str, QuantLinear]) -> None:
    """Requantise every swapped layer after a weight update."""
    for q in swapped.values():
        q.requantize_()
