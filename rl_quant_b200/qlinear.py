"""QuantLinear: W8A8 Linear with LET pre-scaling (qrt/qlinear.py:34-173).

Inference (no autograd): ``z = alpha*x + beta``, per-tensor int8 activations
with a static (calibrated) or dynamic (``absmax(z)/127`` of the call's whole
input) scale, per-output-channel int8 weights, int32 accumulation on the
tcgen05 tensor cores, fp32 dequantisation ``acc*s_w*s_z + b'``, cast back to
the input dtype. Training (autograd on): plain ``F.linear`` on the same
Parameter objects, so optimisers and state dicts keep working.

Buffers and their names/shapes are qrt's (``w8 [Np,K] int8``, ``dq_scale``,
``s_w``, ``b_prime`` ``[Np]``, ``s_z``/``inv_sz`` 0-d, ``alpha``/``beta``
``[K]``), kept at fixed device addresses: ``requantize_`` rewrites them in
place, so captured CUDA graphs stay valid.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N

ACT_MODES = ("static", "dynamic", "dynamic_full")


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return N.DTYPE_F16
    if t.dtype == torch.float32:
        return N.DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}; expected float16 or float32")


class QuantLinear(nn.Module):

    def __init__(self, linear: nn.Linear, s_z: float | None = None,
                 alpha: torch.Tensor | None = None, beta: torch.Tensor | None = None,
                 act_mode: str = "static"):
        super().__init__()
        if act_mode not in ACT_MODES:
            raise ValueError(f"unknown act_mode: {act_mode}")
        N_out, K = linear.out_features, linear.in_features
        if K % 8 != 0:
            raise ValueError(f"in_features={K} is not a multiple of 8")
        dev = linear.weight.device
        self.in_features, self.out_features = K, N_out
        self.n_pad = (-N_out) % 8
        self.act_mode = act_mode
        # the source layer's Parameters, transferred (optimiser references stay valid)
        self.weight = linear.weight
        self.bias = linear.bias
        self.has_let = alpha is not None and act_mode != "dynamic_full"
        if self.has_let:
            self.register_buffer("alpha", alpha.detach().float().clamp_min(1e-8).to(dev))
            self.register_buffer("beta", beta.detach().float().to(dev) if beta is not None
                                 else torch.zeros(K, device=dev))
        s = float(max(1.0 if s_z is None else s_z, 1e-8))
        self.register_buffer("s_z", torch.tensor(s, device=dev))
        self.register_buffer("inv_sz", torch.tensor(1.0 / s, device=dev))
        Np = N_out + self.n_pad
        self.register_buffer("w8", torch.zeros(Np, K, dtype=torch.int8, device=dev))
        self.register_buffer("dq_scale", torch.ones(Np, dtype=torch.float32, device=dev))
        self.register_buffer("s_w", torch.ones(Np, dtype=torch.float32, device=dev))
        self.register_buffer("b_prime", torch.zeros(Np, dtype=torch.float32, device=dev))
        self.register_buffer("_ws", torch.zeros(N.load().glad_qlinear_workspace_size(),
                                                dtype=torch.uint8, device=dev), persistent=False)
        self.requantize_()

    # -- weight quantisation (qrt/qlinear.py:84-102) ---------------------------
    def requant_src(self, alpha=None, beta=None, w8=None, dq=None, s_w=None, b_prime=None) -> N.GladQLinearSrc:
        a = self.alpha if self.has_let else alpha
        b = self.beta if self.has_let else beta
        return N.GladQLinearSrc(
            N.ptr(self.weight), N.ptr(self.bias), _dtype_code(self.weight), self.out_features,
            self.in_features, self.out_features + self.n_pad, N.ptr(a), N.ptr(b), N.ptr(self.s_z),
            N.ptr(self.w8 if w8 is None else w8), N.ptr(self.dq_scale if dq is None else dq),
            N.ptr(self.s_w if s_w is None else s_w), N.ptr(self.b_prime if b_prime is None else b_prime))

    @torch.no_grad()
    def requantize_(self):
        """Refresh the int8 buffers from the current weight/bias, in place."""
        if self.act_mode == "dynamic_full":
            return
        N.require_cuda(self.weight)
        src = self.requant_src()
        N.check(N.load().glad_requant_qlinear(src, 1, N.stream_handle(self.weight.device)),
                "QuantLinear.requantize_")

    @torch.no_grad()
    def set_act_scale_(self, s_z: float):
        """Set the static activation scale (call requantize_ afterwards)."""
        self.s_z.fill_(float(max(s_z, 1e-8)))
        self.inv_sz.fill_(1.0 / float(max(s_z, 1e-8)))

    # -- forward ----------------------------------------------------------------
    def forward(self, x):
        if torch.is_grad_enabled():
            return F.linear(x, self.weight, self.bias)
        N.require_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        if self.act_mode == "dynamic_full":
            y = self._forward_dynamic_full(x2)
        else:
            y = torch.empty(x2.shape[0], self.out_features, dtype=x.dtype, device=x.device)
            self._run(x2, y, self.act_mode, N.qlinear_struct(self))
        return y.reshape(*shape[:-1], self.out_features)

    def _run(self, x2, y, mode, L):
        lib = N.load()
        rc = lib.glad_qlinear_forward(L, N.ACT_MODES[mode], x2.data_ptr(), _dtype_code(x2), x2.shape[0],
                                      x2.stride(0), y.data_ptr(), y.stride(0), None, self._ws.data_ptr(),
                                      self._ws.numel(), N.stream_handle(x2.device))
        N.check(rc, "QuantLinear.forward")

    def _forward_dynamic_full(self, x2):
        """alpha = 1/std, beta = -mean/std from the call's batch, weights folded
        and quantised per call (qrt/qlinear.py:140-169)."""
        xf = x2.float()
        sigma = xf.std(dim=0).clamp_min(1e-5)
        alpha = (1.0 / sigma).contiguous()
        beta = (-xf.mean(dim=0) / sigma).contiguous()
        Np = self.out_features + self.n_pad
        dev = x2.device
        w8 = torch.zeros(Np, self.in_features, dtype=torch.int8, device=dev)
        dq = torch.ones(Np, dtype=torch.float32, device=dev)
        s_w = torch.ones(Np, dtype=torch.float32, device=dev)
        bp = torch.zeros(Np, dtype=torch.float32, device=dev)
        src = self.requant_src(alpha, beta, w8, dq, s_w, bp)
        N.check(N.load().glad_requant_qlinear(src, 1, N.stream_handle(dev)), "dynamic_full requant")
        L = N.GladQLinear(N.ptr(w8), N.ptr(dq), N.ptr(s_w), N.ptr(bp), N.ptr(alpha), N.ptr(beta),
                          N.ptr(self.s_z), N.ptr(self.inv_sz), self.in_features, self.out_features)
        y = torch.empty(x2.shape[0], self.out_features, dtype=x2.dtype, device=dev)
        self._run(x2, y, "dynamic", L)
        return y

    def extra_repr(self):
        return (f"in={self.in_features}, out={self.out_features}, let={self.has_let}, "
                f"act_mode={self.act_mode}, pad={self.n_pad}")
