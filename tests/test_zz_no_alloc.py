"""glad_actor_forward_noalloc: the allocation-free entry point for callers
whose host runtime owns all device memory and forbids this library to
allocate (its scratch is a static device array inside the library, sized for
at most GLAD_NOALLOC_MAX_B environments).

Checks, through the C ABI: two calls in a row agree with the workspace entry
point (glad_actor_forward) within the parity tolerance of the other GPU tests,
and a batch above the limit is rejected with a clear error. This file is
collected last on purpose; it also passes when run alone.
"""
import numpy as np
import pytest
import torch

from rl_quant_b200 import _native as N
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-2
MIN_COS = 0.99999


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / torch.sqrt((a @ a) * (b @ b)))


def _with_workspace(lib, w, obs, mode):
    B = obs.shape[0]
    mean = torch.empty(B, 29, dtype=torch.float32, device="cuda")
    nbytes = lib.glad_actor_workspace_size(B)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    N.check(lib.glad_actor_forward(w, obs.data_ptr(), N.DTYPE_F32, B, obs.stride(0), N.ACT_MODES[mode], None,
                                   mean.data_ptr(), None, ws.data_ptr(), nbytes, N.stream_handle()),
            "glad_actor_forward")
    return mean


def _no_alloc(lib, w, obs, mode):
    B = obs.shape[0]
    mean = torch.empty(B, 29, dtype=torch.float32, device="cuda")
    N.check(lib.glad_actor_forward_noalloc(w, obs.data_ptr(), N.DTYPE_F32, B, obs.stride(0), N.ACT_MODES[mode],
                                           None, mean.data_ptr(), None, N.stream_handle()),
            "glad_actor_forward_noalloc")
    return mean


@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_no_alloc_matches_workspace_entry_two_calls(golden_weights, mode):
    lib = N.load()
    dw = DeviceWeights(golden_weights)
    w = dw.actor()
    # two calls in a row: a full-size batch, then a smaller one over the same
    # scratch (it still holds the first call's contents)
    for B, seed in ((N.NOALLOC_MAX_B, 11), (37, 12)):
        obs = glad_obs(B, seed=seed).cuda()
        ref = _with_workspace(lib, w, obs, mode)
        got = _no_alloc(lib, w, obs, mode)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - ref).abs().max().item() <= MAX_ABS
        assert _cos(got, ref) >= MIN_COS


def test_no_alloc_rejects_batches_over_the_limit(golden_weights):
    lib = N.load()
    dw = DeviceWeights(golden_weights)
    obs = torch.zeros(1, 2175, device="cuda")
    rc = lib.glad_actor_forward_noalloc(dw.actor(), obs.data_ptr(), N.DTYPE_F32, N.NOALLOC_MAX_B + 1, 2175,
                                        N.ACT_DYNAMIC, None, obs.data_ptr(), None, N.stream_handle())
    assert rc == N.GLAD_ERR_INVALID_ARG
    assert "GLAD_NOALLOC_MAX_B" in lib.glad_last_error().decode()
