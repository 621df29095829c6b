"""W4A16 actor MLP (int4 weights, group 64, fp16 activations) vs the oracle's
restatement of the same format; the whole actor with the INT8 encoder.

The format has no reference implementation (README.md:259 names INT4 as future
work): parity is against this repository's CPU restatement. Tolerance: the
kernel accumulates in fp32 where the oracle uses float64, so fp16 roundings may
flip; outputs agree within max-abs 5e-3 and cosine >= 0.99999."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import glad_oracle as O
from rl_quant_b200 import _native as N
from rl_quant_b200.synthetic import glad_obs
from rl_quant_b200.w4a16 import W4A16MLP

from gpu_util import DeviceWeights, actor_forward

pytestmark = pytest.mark.gpu


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


def _np_layers(mlp):
    return [(getattr(mlp, f"packed{i}").cpu().numpy(), getattr(mlp, f"scales{i}").cpu().numpy(),
             getattr(mlp, f"bias{i}").cpu().numpy(), k) for i, k in enumerate((224, 512, 256, 128))]


@pytest.fixture(scope="module")
def mlp():
    torch.manual_seed(3)
    actor = nn.Sequential(nn.Linear(224, 512), nn.ELU(), nn.Linear(512, 256), nn.ELU(), nn.Linear(256, 128),
                          nn.ELU(), nn.Linear(128, 29))
    return W4A16MLP.from_actor(actor.cuda())


@pytest.fixture(scope="module")
def dw(golden_weights):
    return DeviceWeights(golden_weights)


@pytest.mark.parametrize("M", [1, 130, 1000])
def test_w4a16_mlp_vs_oracle(mlp, M):
    g = torch.Generator().manual_seed(M)
    x = (torch.randn(M, 224, generator=g) * 0.8).half()
    got = mlp(x.cuda()).cpu().numpy()
    ref = O.w4a16_mlp(x.numpy(), _np_layers(mlp))
    assert np.abs(got - ref).max() <= 5e-3
    assert cos(got, ref) >= 0.99999
    assert np.array_equal(got, got.astype(np.float16).astype(np.float32))   # float of fp16 values


def test_w4a16_requantize_in_place(mlp):
    ptr = mlp.packed1.data_ptr()
    before = mlp.packed1.clone()
    with torch.no_grad():
        mlp.src[1].weight.mul_(-1.0)
    mlp.requantize_()
    assert mlp.packed1.data_ptr() == ptr
    assert not torch.equal(before, mlp.packed1)
    with torch.no_grad():
        mlp.src[1].weight.mul_(-1.0)
    mlp.requantize_()
    assert torch.equal(before, mlp.packed1)


def _actor_w4(dw, mlp, obs, mode):
    B = obs.shape[0]
    mean = torch.empty(B, 29, dtype=torch.float32, device="cuda")
    lib = N.load()
    nbytes = lib.glad_actor_workspace_size(B)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    N.check(lib.glad_actor_forward_w4a16(dw.actor(), mlp.layers(), obs.data_ptr(), N.DTYPE_F32, B, obs.stride(0),
                                         N.ACT_MODES[mode], mean.data_ptr(), ws.data_ptr(), nbytes,
                                         N.stream_handle()), "glad_actor_forward_w4a16")
    st = N.c_uint32(0)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "device status")
    torch.cuda.synchronize()
    return mean


@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_actor_w4a16_equals_int8_encoder_plus_w4_mlp(dw, mlp, mode):
    B = 200
    obs = glad_obs(B, seed=303).cuda()
    mean = _actor_w4(dw, mlp, obs, mode).cpu().numpy()
    _, aux = actor_forward(dw, obs, mode)                 # same INT8 encoder -> encoded
    ref = O.w4a16_mlp(aux["encoded"].cpu().numpy(), _np_layers(mlp))
    assert np.abs(mean - ref).max() <= 5e-3
    assert cos(mean, ref) >= 0.99999


def test_actor_w4a16_large_batch_rows_independent(dw, mlp):
    """B = 65536 (the largest W4A16 batch), static s_z: sampled rows equal a small batch
    of the same observations."""
    B = 65536
    obs = glad_obs(B, seed=404).cuda()
    big = _actor_w4(dw, mlp, obs, "static")
    rows = torch.tensor([0, 1, 127, 128, 4095, 4096, 30000, 65535], device="cuda")
    small = _actor_w4(dw, mlp, obs[rows].contiguous(), "static")
    assert torch.equal(big[rows], small)
    assert torch.isfinite(big).all()
