"""rl_quant_b200 -- the GLAD rollout forward of RL_Quant's qrt path, built for
B200 (sm_100a) with hand-written tcgen05 kernels behind a C ABI.

The public API mirrors qrt (qrt/__init__.py:18-34):
    QuantCNN, swap_cnn, calib_cnn_scale   int8 map CNN      (qrt/qconv.py)
    QuantLinear                           W8A8 + LET linear (qrt/qlinear.py)
    patch_encoder, unpatch_encoder        encoder rewrite   (qrt/encoder_opt.py)
    InferenceRunner                       rollout runner    (qrt/runtime.py)
    accelerate_runner                     rsl_rl drop-in    (qrt/integration.py)
    swap, calib                           module surgery / calibration

Names are resolved lazily, so importing a light submodule (``synthetic``,
``glad_model``) neither loads the CUDA library nor registers the qrt
operators.
"""
from __future__ import annotations

import importlib

_EXPORTS = {
    "QuantCNN": "qconv", "swap_cnn": "qconv", "calib_cnn_scale": "qconv",
    "QuantLinear": "qlinear",
    "patch_encoder": "encoder_opt", "unpatch_encoder": "encoder_opt",
    "InferenceRunner": "runtime",
    "accelerate_runner": "integration", "QRTAccelerator": "integration",
    "INT8_PATHS_DEFAULT": "integration",
    "LETQuantizer": "let",
    "FusedActor": "fused", "DeviceStatusError": "fused",
    "GladActorCritic": "glad_model", "build_glad": "glad_model",
}
_SUBMODULES = ("swap", "calib", "_native", "synthetic", "glad_model", "qconv", "qlinear", "encoder_opt",
               "runtime", "integration", "let", "fused", "build")

__all__ = sorted(_EXPORTS) + ["swap", "calib"]


def __getattr__(name):
    if name in _EXPORTS:
        return getattr(importlib.import_module(f".{_EXPORTS[name]}", __name__), name)
    if name in _SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
