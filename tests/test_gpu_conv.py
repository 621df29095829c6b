"""conv operators (qrt::conv1_fused_q / conv2_int8_fused / chain) vs the oracle."""
import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200 import _native as N
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights, fp16_ulp_close

pytestmark = pytest.mark.gpu


def _x_nhwc(B, seed):
    return glad_obs(B, seed)[:, 96:].half().reshape(B, 21, 33, 3).contiguous()


def _conv1(dw, x):
    z8 = torch.empty(x.shape[0] * 187, 16, dtype=torch.int8, device="cuda")
    N.check(N.load().glad_conv1_fused_q(x.data_ptr(), x.shape[0], dw.conv(), z8.data_ptr(), N.stream_handle()))
    torch.cuda.synchronize()
    return z8


def _conv2(dw, z8):
    B = z8.shape[0] // 187
    feat = torch.empty(B * 187, 64, dtype=torch.float16, device="cuda")
    acc = torch.empty(B * 187, 64, dtype=torch.int32, device="cuda")
    N.check(N.load().glad_conv2_int8_fused(z8.data_ptr(), B, dw.conv(), feat.data_ptr(), acc.data_ptr(),
                                           N.stream_handle()))
    torch.cuda.synchronize()
    return feat, acc


@pytest.fixture(scope="module")
def dw(golden_weights):
    return DeviceWeights(golden_weights)


@pytest.mark.parametrize("B", [1, 3, 4, 37, 600])
def test_conv2_int32_accumulators_bit_exact(dw, golden_weights, B):
    rng = np.random.default_rng(B)
    z8 = rng.integers(-128, 128, size=(B * 187, 16), dtype=np.int8)
    feat, acc = _conv2(dw, torch.from_numpy(z8).cuda())
    w = golden_weights
    ref_acc = O.conv2_acc(z8, w["map_cnn.w8"])
    assert np.array_equal(acc.cpu().numpy(), ref_acc)
    ref_feat = O.conv2_epilogue(ref_acc, w["map_cnn.dq"], w["map_cnn.b2f"], w["map_cnn.a2"], w["map_cnn.c2"])
    fp16_ulp_close(feat.cpu().numpy(), ref_feat)


def test_conv1_matches_reference_kernel(dw, golden_conv):
    x = torch.from_numpy(golden_conv["x_nhwc"]).cuda()
    z8 = _conv1(dw, x).cpu().numpy().astype(np.int16)
    ref = golden_conv["z8"].astype(np.int16)
    diff = np.abs(z8 - ref)
    assert diff.max() <= 1
    assert (diff > 0).mean() < 1e-3


@pytest.mark.parametrize("B", [1, 5, 300])
def test_conv1_vs_oracle(dw, golden_weights, B):
    x = _x_nhwc(B, 100 + B)
    z8 = _conv1(dw, x.cuda()).cpu().numpy().astype(np.int16)
    w = golden_weights
    ref = O.conv1_fused_q(x.numpy(), w["map_cnn.w1p"], w["map_cnn.b1f"], w["map_cnn.qa"], w["map_cnn.qc"])
    diff = np.abs(z8 - ref.astype(np.int16))
    assert diff.max() <= 1          # only rounding ties may flip, by one step
    assert (diff > 0).mean() < 1e-3


@pytest.mark.parametrize("B", [2, 129])
def test_conv_chain_equals_two_ops(dw, golden_weights, B):
    x = _x_nhwc(B, 7 + B).cuda()
    feat = torch.empty(B * 187, 64, dtype=torch.float16, device="cuda")
    z8 = torch.empty(B * 187, 16, dtype=torch.int8, device="cuda")
    N.check(N.load().glad_conv_chain(x.data_ptr(), B, dw.conv(), feat.data_ptr(), z8.data_ptr(),
                                     N.stream_handle()))
    torch.cuda.synchronize()
    z8_op = _conv1(dw, x)
    assert torch.equal(z8, z8_op)
    feat_op, _ = _conv2(dw, z8_op)
    assert torch.equal(feat, feat_op)
    w = golden_weights
    ref = O.conv2_int8_fused(z8.cpu().numpy(), w["map_cnn.w8"], w["map_cnn.dq"], w["map_cnn.b2f"],
                             w["map_cnn.a2"], w["map_cnn.c2"])
    fp16_ulp_close(feat.cpu().numpy(), ref)


def test_conv_rejects_bad_arguments(dw):
    lib = N.load()
    with pytest.raises(ValueError):
        N.check(lib.glad_conv1_fused_q(None, 4, dw.conv(), None, N.stream_handle()))
    assert lib.glad_conv1_fused_q(None, 0, dw.conv(), None, N.stream_handle()) == 0


def test_conv_chain_large_batch(dw, golden_weights):
    """B=16384 (the largest conv-only batch): sampled environments equal the oracle
    (z8 within one step at ties, fp16 features within one ulp given the kernel's z8)
    and equal the same environments run as a small batch."""
    B = 16384
    x = _x_nhwc(B, 2024).cuda()
    feat = torch.empty(B * 187, 64, dtype=torch.float16, device="cuda")
    z8 = torch.empty(B * 187, 16, dtype=torch.int8, device="cuda")
    N.check(N.load().glad_conv_chain(x.data_ptr(), B, dw.conv(), feat.data_ptr(), z8.data_ptr(),
                                     N.stream_handle()))
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    envs = np.sort(rng.choice(B, size=24, replace=False))
    xs = x[torch.from_numpy(envs).cuda()].contiguous()
    w = golden_weights
    ref_z8 = O.conv1_fused_q(xs.cpu().numpy(), w["map_cnn.w1p"], w["map_cnn.b1f"], w["map_cnn.qa"],
                             w["map_cnn.qc"])
    got_z8 = z8.view(B, 187, 16)[torch.from_numpy(envs).cuda()].reshape(-1, 16).cpu().numpy()
    d = np.abs(got_z8.astype(np.int16) - ref_z8.astype(np.int16))
    assert d.max() <= 1 and (d > 0).mean() < 1e-3
    ref_feat = O.conv2_int8_fused(got_z8, w["map_cnn.w8"], w["map_cnn.dq"], w["map_cnn.b2f"],
                                  w["map_cnn.a2"], w["map_cnn.c2"])
    got_feat = feat.view(B, 187, 64)[torch.from_numpy(envs).cuda()].reshape(-1, 64).cpu().numpy()
    fp16_ulp_close(got_feat, ref_feat)
    f2 = torch.empty(len(envs) * 187, 64, dtype=torch.float16, device="cuda")
    z2 = torch.empty(len(envs) * 187, 16, dtype=torch.int8, device="cuda")
    N.check(N.load().glad_conv_chain(xs.data_ptr(), len(envs), dw.conv(), f2.data_ptr(), z2.data_ptr(),
                                     N.stream_handle()))
    torch.cuda.synchronize()
    assert np.array_equal(z2.cpu().numpy(), got_z8)
    assert np.array_equal(f2.cpu().numpy(), got_feat)


def test_conv1_rounding_ties_exact(golden_weights):
    """One unit tap per output channel makes every accumulator exact, and half-integer
    inputs put z exactly on rounding ties of both signs and beyond both clamp bounds:
    the kernel's round-half-away-from-zero and clamp equal the oracle's bit for bit
    (qrt/qconv.py:96-101)."""
    w = dict(golden_weights)
    w1p = np.zeros((128, 16), np.float16)
    for n in range(16):
        w1p[2 * 16 + 2 * 3 + n % 3, n] = 1.0        # centre tap (kh = kw = 2) of input channel n % 3
    w["map_cnn.w1p"] = w1p
    w["map_cnn.b1f"] = np.zeros(16, np.float32)
    w["map_cnn.qa"] = np.ones(16, np.float32)
    w["map_cnn.qc"] = np.arange(16, dtype=np.float32) * 16.0 - 140.0   # z from below -128 to above 127
    dev = DeviceWeights(w)
    rng = np.random.default_rng(7)
    x = (rng.integers(-300, 400, size=(64, 21, 33, 3)) * 0.5).astype(np.float16)
    z8 = _conv1(dev, torch.from_numpy(x).cuda()).cpu().numpy()
    q, z = O.conv1_fused_q(x, w1p, w["map_cnn.b1f"], w["map_cnn.qa"], w["map_cnn.qc"], return_z=True)
    assert (np.abs(z - np.trunc(z)) == 0.5).mean() > 0.2           # many exact ties
    assert (z < -128.5).any() and (z > 127.5).any()
    assert np.array_equal(z8, q)
