"""Device-side failures reach the caller.

Every wait inside the fused kernels is bounded: when one runs out the kernel
sets a bit in the workspace's status word and finishes, so the GPU stays
usable. These tests make the fused actor MLP's grid barrier wait for one CTA
more than the grid holds, with a 1 ms limit (glad_debug_mlp_barrier; nothing
faults, traps or hangs), and check that the failure is reported: the C ABI
returns GLAD_ERR_DEVICE with the barrier bit, InferenceRunner.check_status
raises DeviceStatusError, and the next normal call on the same workspace is
clean again and equal to a fresh run.
"""
import pytest
import torch

from rl_quant_b200 import _native as N
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights, golden_model

pytestmark = pytest.mark.gpu

GLAD_DEVERR_BARRIER_TIMEOUT = 8


@pytest.fixture
def barrier_fault():
    lib = N.load()
    N.check(lib.glad_debug_mlp_barrier(1, 1_000_000), "glad_debug_mlp_barrier")
    try:
        yield
    finally:
        N.check(lib.glad_debug_mlp_barrier(0, 0), "glad_debug_mlp_barrier reset")


def _forward(lib, w, obs, ws, mean):
    N.check(lib.glad_actor_forward(w, obs.data_ptr(), N.DTYPE_F32, obs.shape[0], obs.stride(0), N.ACT_DYNAMIC,
                                   None, mean.data_ptr(), None, ws.data_ptr(), ws.numel(), N.stream_handle()),
            "glad_actor_forward")


def test_barrier_timeout_reported_through_the_abi(golden_weights):
    lib = N.load()
    B = 1024
    assert lib.glad_actor_mlp_fused(B, N.ACT_DYNAMIC) == 1
    dw = DeviceWeights(golden_weights)
    w = dw.actor()
    obs = glad_obs(B, seed=404).cuda()
    ws = torch.zeros(lib.glad_actor_workspace_size(B), dtype=torch.uint8, device="cuda")
    mean = torch.empty(B, 29, device="cuda")
    N.check(lib.glad_debug_mlp_barrier(1, 1_000_000), "glad_debug_mlp_barrier")
    try:
        _forward(lib, w, obs, ws, mean)
        st = N.c_uint32(0)
        rc = lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle())
    finally:
        N.check(lib.glad_debug_mlp_barrier(0, 0), "glad_debug_mlp_barrier reset")
    assert rc == N.GLAD_ERR_DEVICE
    assert st.value & GLAD_DEVERR_BARRIER_TIMEOUT
    assert "bounded device-side wait" in lib.glad_last_error().decode()
    # the read cleared the word; the device is still usable and the next call is clean
    _forward(lib, w, obs, ws, mean)
    st = N.c_uint32(1)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "status after recovery")
    assert st.value == 0
    ws2 = torch.zeros_like(ws)
    mean2 = torch.empty_like(mean)
    _forward(lib, w, obs, ws2, mean2)
    torch.cuda.synchronize()
    assert torch.equal(mean, mean2)


def test_status_word_is_sticky_until_read(golden_weights, barrier_fault):
    """A failed call followed by a good one still reports the failure at the next read."""
    lib = N.load()
    B = 512
    w = DeviceWeights(golden_weights).actor()
    obs = glad_obs(B, seed=405).cuda()
    ws = torch.zeros(lib.glad_actor_workspace_size(B), dtype=torch.uint8, device="cuda")
    mean = torch.empty(B, 29, device="cuda")
    _forward(lib, w, obs, ws, mean)                  # barrier runs out
    N.check(lib.glad_debug_mlp_barrier(0, 0), "reset")
    _forward(lib, w, obs, ws, mean)                  # a normal call does not clear the word
    st = N.c_uint32(0)
    assert lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()) == N.GLAD_ERR_DEVICE
    assert st.value & GLAD_DEVERR_BARRIER_TIMEOUT


def test_runner_check_status_raises(golden_weights):
    from rl_quant_b200 import DeviceStatusError, InferenceRunner

    m, _ = golden_model(golden_weights)
    runner = InferenceRunner(m, mode="eager")
    obs = glad_obs(256, seed=406).cuda()
    runner.act(obs)
    runner.check_status()                            # clean
    lib = N.load()
    N.check(lib.glad_debug_mlp_barrier(1, 1_000_000), "glad_debug_mlp_barrier")
    try:
        runner.act(obs)
    finally:
        N.check(lib.glad_debug_mlp_barrier(0, 0), "reset")
    with pytest.raises(DeviceStatusError):
        runner.check_status()
    good = runner.act(obs).clone()
    runner.check_status()                            # clean again
    torch.cuda.synchronize()
    assert torch.isfinite(good).all()
