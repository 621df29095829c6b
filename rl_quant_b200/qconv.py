"""QuantCNN: the GLAD map CNN as two int8 implicit-GEMM convolutions on the
tcgen05 tensor cores (qrt/qconv.py:1-333).

    conv1  5x5/s2/p2 fp16 -> +bias, ReLU, BN1, quantise to int8 (z8)
    conv2  3x3/p1 int8 x int8 -> int32 -> dequant, +bias, ReLU, BN2 -> fp16

Operators ``torch.ops.qrt.conv1_fused_q`` and ``torch.ops.qrt.conv2_int8_fused``
keep qrt's names, argument order and fake (meta) implementations, so code that
calls them -- and torch.compile / CUDA-graph capture around them -- works
unchanged. ``QuantCNN.forward`` runs both in one kernel (``glad_conv_chain``):
z8 stays on chip.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _native as N

H1, W1, C1 = 21, 33, 3
H2, W2, C2 = 11, 17, 16
P = H2 * W2
N2 = 64
K1 = 128
K2S = 64


def _conv_struct(w1p=None, b1f=None, qa=None, qc=None, w8=None, dq=None, b2=None, a2=None, c2=None):
    return N.conv_weights(w1p, b1f, qa, qc, w8, dq, b2, a2, c2)


@torch.library.custom_op("qrt::conv1_fused_q", mutates_args=(), device_types="cuda")
def conv1_fused_q(x_nhwc: torch.Tensor, w1p: torch.Tensor, b1: torch.Tensor,
                  qa: torch.Tensor, qc: torch.Tensor) -> torch.Tensor:
    """[B,21,33,3] fp16 -> z8 [B*187,16] int8 (qrt/qconv.py:170-178)."""
    x = x_nhwc.contiguous()
    if x.dtype != torch.float16:
        x = x.half()
    out = torch.empty(x.shape[0] * P, C2, dtype=torch.int8, device=x.device)
    rc = N.load().glad_conv1_fused_q(x.data_ptr(), x.shape[0], _conv_struct(w1p, b1, qa, qc),
                                     out.data_ptr(), N.stream_handle(x.device))
    N.check(rc, "qrt::conv1_fused_q")
    return out


@conv1_fused_q.register_fake
def _(x_nhwc, w1p, b1, qa, qc):
    return x_nhwc.new_empty((x_nhwc.shape[0] * P, C2), dtype=torch.int8)


@torch.library.custom_op("qrt::conv2_int8_fused", mutates_args=(), device_types="cuda")
def conv2_int8_fused(z8: torch.Tensor, w8: torch.Tensor, dq: torch.Tensor, b2: torch.Tensor,
                     a2: torch.Tensor, c2: torch.Tensor) -> torch.Tensor:
    """z8 [B*187,16] int8 -> [B*187,64] fp16 (qrt/qconv.py:186-193)."""
    z = z8.contiguous()
    out = torch.empty(z.shape[0], N2, dtype=torch.float16, device=z.device)
    rc = N.load().glad_conv2_int8_fused(z.data_ptr(), z.shape[0] // P,
                                        _conv_struct(w8=w8, dq=dq, b2=b2, a2=a2, c2=c2),
                                        out.data_ptr(), None, N.stream_handle(z.device))
    N.check(rc, "qrt::conv2_int8_fused")
    return out


@conv2_int8_fused.register_fake
def _(z8, w8, dq, b2, a2, c2):
    return z8.new_empty((z8.shape[0], N2), dtype=torch.float16)


def conv2_int8_acc(z8: torch.Tensor, w8: torch.Tensor) -> torch.Tensor:
    """int32 accumulators of conv2 (a diagnostic view of conv2_int8_fused)."""
    z = z8.contiguous()
    dev = z.device
    one = torch.ones(N2, device=dev)
    zero = torch.zeros(N2, device=dev)
    feat = torch.empty(z.shape[0], N2, dtype=torch.float16, device=dev)
    acc = torch.empty(z.shape[0], N2, dtype=torch.int32, device=dev)
    rc = N.load().glad_conv2_int8_fused(z.data_ptr(), z.shape[0] // P,
                                        _conv_struct(w8=w8, dq=one, b2=zero, a2=one, c2=zero),
                                        feat.data_ptr(), acc.data_ptr(), N.stream_handle(dev))
    N.check(rc, "conv2 accumulators")
    return acc


class QuantCNN(nn.Module):
    """Quantised stand-in for ``map_cnn`` (qrt/qconv.py:205-306).

    Children keep the Sequential's indices ("0" conv1, "2" BN1, "3" conv2,
    "5" BN2), so parameter paths are unchanged. Without autograd the forward
    runs the int8 kernels and returns a zero-copy ``[B,64,11,17]`` view of the
    token-major ``[B*187,64]`` output; with autograd it runs the float layers.
    """

    def __init__(self, map_cnn: nn.Sequential, s_z: float,
                 alpha: torch.Tensor | None = None, beta: torch.Tensor | None = None):
        super().__init__()
        self.add_module("0", map_cnn[0])
        self.add_module("2", map_cnn[2])
        self.add_module("3", map_cnn[3])
        self.add_module("5", map_cnn[5])
        dev = map_cnn[0].weight.device
        self.has_let = alpha is not None
        if self.has_let:
            self.register_buffer("alpha", alpha.detach().float().clamp_min(1e-8).to(dev))
            self.register_buffer("beta", beta.detach().float().to(dev) if beta is not None
                                 else torch.zeros(C2, device=dev))
        self.register_buffer("s_z", torch.tensor(float(max(s_z, 1e-8)), device=dev))
        self.register_buffer("w1p", torch.zeros(K1, C2, dtype=torch.float16, device=dev))
        self.register_buffer("b1f", torch.zeros(C2, dtype=torch.float32, device=dev))
        self.register_buffer("qa", torch.zeros(C2, dtype=torch.float32, device=dev))
        self.register_buffer("qc", torch.zeros(C2, dtype=torch.float32, device=dev))
        self.register_buffer("w8", torch.zeros(3, K2S, N2, dtype=torch.int8, device=dev))
        self.register_buffer("dq", torch.zeros(N2, dtype=torch.float32, device=dev))
        self.register_buffer("b2f", torch.zeros(N2, dtype=torch.float32, device=dev))
        self.register_buffer("a2", torch.zeros(N2, dtype=torch.float32, device=dev))
        self.register_buffer("c2", torch.zeros(N2, dtype=torch.float32, device=dev))
        self.requantize_()

    def conv_struct(self) -> N.GladConvWeights:
        return _conv_struct(self.w1p, self.b1f, self.qa, self.qc, self.w8, self.dq, self.b2f, self.a2, self.c2)

    def requant_src(self) -> N.GladQCNNSrc:
        m = self._modules
        c1, bn1, c2, bn2 = m["0"], m["2"], m["3"], m["5"]
        dt = c1.weight.dtype
        for t in (bn1.weight, bn1.running_mean, c2.weight, bn2.weight, bn2.running_var):
            if t.dtype != dt:
                raise TypeError("QuantCNN parameters must share one dtype (fp16 or fp32)")
        return N.GladQCNNSrc(
            N.ptr(c1.weight), N.ptr(c1.bias), N.ptr(bn1.weight), N.ptr(bn1.bias),
            N.ptr(bn1.running_mean), N.ptr(bn1.running_var), N.ptr(c2.weight), N.ptr(c2.bias),
            N.ptr(bn2.weight), N.ptr(bn2.bias), N.ptr(bn2.running_mean), N.ptr(bn2.running_var),
            N.ptr(self.s_z), float(bn1.eps), float(bn2.eps),
            N.ptr(self.w1p), N.ptr(self.b1f), N.ptr(self.qa), N.ptr(self.qc), N.ptr(self.w8),
            N.ptr(self.dq), N.ptr(self.b2f), N.ptr(self.a2), N.ptr(self.c2),
            N.DTYPE_F16 if dt == torch.float16 else N.DTYPE_F32,
            N.ptr(self.alpha) if self.has_let else None, N.ptr(self.beta) if self.has_let else None)

    @torch.no_grad()
    def requantize_(self):
        """Recompute every packed buffer from the current conv/BN parameters,
        in place (qrt/qconv.py:247-284)."""
        N.require_cuda(self.w1p)
        for t in (self._modules["0"].weight, self._modules["3"].weight):
            if not t.is_contiguous():
                raise ValueError("conv weights must be contiguous")
        N.check(N.load().glad_requant_qcnn(self.requant_src(), N.stream_handle(self.w1p.device)),
                "QuantCNN.requantize_")

    @torch.no_grad()
    def set_act_scale_(self, s_z: float):
        self.s_z.fill_(float(max(s_z, 1e-8)))

    def forward(self, x):                       # x: [B,3,21,33]
        if torch.is_grad_enabled():
            m = self._modules
            h = m["2"](torch.relu(m["0"](x)))
            return m["5"](torch.relu(m["3"](h)))
        N.require_cuda(x)
        B = x.shape[0]
        x_nhwc = x.permute(0, 2, 3, 1)
        if x_nhwc.dtype != torch.float16:
            x_nhwc = x_nhwc.half()
        x_nhwc = x_nhwc.contiguous()
        feat = torch.empty(B * P, N2, dtype=torch.float16, device=x.device)
        rc = N.load().glad_conv_chain(x_nhwc.data_ptr(), B, self.conv_struct(), feat.data_ptr(), None,
                                      N.stream_handle(x.device))
        N.check(rc, "QuantCNN.forward")
        return feat.view(B, H2, W2, N2).permute(0, 3, 1, 2)

    def extra_repr(self):
        return f"GLAD CNN (tcgen05 int8), let={self.has_let}, s_z={self.s_z.item():.4g}"


def swap_cnn(model, s_z: float, alpha=None, beta=None) -> QuantCNN:
    """Replace ``model.map_cnn`` by a QuantCNN with the same train/eval state."""
    q = QuantCNN(model.map_cnn, s_z, alpha=alpha, beta=beta)
    q.train(model.map_cnn.training)
    model.map_cnn = q
    return q


@torch.no_grad()
def calib_cnn_scale(model, obs_fn, n_batches: int = 8) -> float:
    """Per-tensor scale of conv2's input, absmax(BN1 output)/127, measured on
    the float ``map_cnn`` before the swap (qrt/qconv.py:317-333)."""
    amax = [0.0]
    h = model.map_cnn[2].register_forward_hook(
        lambda m, i, o: amax.__setitem__(0, max(amax[0], o.detach().abs().amax().item())))
    was = model.training
    model.eval()
    try:
        with torch.inference_mode():
            for _ in range(n_batches):
                model.act_inference(obs_fn())
    finally:
        model.train(was)
        h.remove()
    return max(amax[0], 1e-6) / 127.0
