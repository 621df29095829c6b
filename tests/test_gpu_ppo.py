"""PPO.act epilogue (glad_ppo_epilogue): Normal(mean, std) sample and summed
log-probability against the oracle's Philox/Box-Muller restatement, the device
offset advance, the distribution of the draws, and the argument checks."""
import numpy as np
import pytest
import scipy.stats as st
import torch

from oracle import glad_oracle as O
from rl_quant_b200 import _native as N
from rl_quant_b200.fused import ppo_epilogue

pytestmark = pytest.mark.gpu


def _case(B, n, seed):
    g = torch.Generator().manual_seed(seed)
    mean = torch.randn(B, n, generator=g).half().float()          # fp16-valued means, as the actor returns
    std = (0.2 + torch.rand(n, generator=g)).float()
    return mean, std


def _run(mean, std, seed, rng, sigma=False):
    B, n = mean.shape
    m, s = mean.cuda(), std.cuda()
    a = torch.empty(B, n, device="cuda")
    lp = torch.empty(B, device="cuda")
    sg = torch.empty(B, n, device="cuda") if sigma else None
    ppo_epilogue(m, s, seed, rng, a, lp, sg)
    torch.cuda.synchronize()
    return a.cpu().numpy(), lp.cpu().numpy(), (sg.cpu().numpy() if sigma else None)


@pytest.mark.parametrize("B,n", [(1, 1), (1000, 29), (333, 64), (77, 33)])
def test_ppo_epilogue_matches_oracle(B, n):
    mean, std = _case(B, n, seed=B + n)
    rng = torch.zeros(2, dtype=torch.int64, device="cuda")
    rng[0] = 11
    a, lp, sg = _run(mean, std, 1234, rng, sigma=True)
    ea, elp = O.ppo_epilogue(mean.numpy(), std.numpy(), 1234, 11)
    # Box-Muller: CUDA logf / sincospif against numpy's log and float64 sin/cos (few ulp)
    np.testing.assert_allclose(a, ea, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(lp, elp, rtol=1e-6, atol=3e-5)
    # the log-probability of the kernel's own actions: the oracle's fp32 terms and sum order
    terms = O.ppo_log_prob_terms(mean.numpy(), np.broadcast_to(std.numpy()[None], (B, n)), a)
    np.testing.assert_allclose(lp, O.butterfly_sum32(terms), rtol=0, atol=2e-5)
    # and torch's own Normal.log_prob of those actions (its sum order differs)
    ref = torch.distributions.Normal(mean, std.expand(B, n)).log_prob(torch.from_numpy(a)).sum(-1).numpy()
    np.testing.assert_allclose(lp, ref, rtol=1e-6, atol=5e-5)
    assert np.array_equal(sg, np.broadcast_to(std.numpy()[None], (B, n)))
    assert rng.cpu().tolist() == [12, 0]


def test_ppo_epilogue_offset_advances():
    mean, std = _case(256, 29, seed=5)
    rng = torch.zeros(2, dtype=torch.int64, device="cuda")
    a0, _, _ = _run(mean, std, 9, rng)
    a1, _, _ = _run(mean, std, 9, rng)
    assert rng.cpu().tolist() == [2, 0]
    assert not np.array_equal(a0, a1)
    np.testing.assert_allclose(a1, O.ppo_epilogue(mean.numpy(), std.numpy(), 9, 1)[0], rtol=2e-6, atol=2e-6)


def test_ppo_epilogue_distribution():
    B, n = 4096, 29
    mean, std = _case(B, n, seed=8)
    rng = torch.zeros(2, dtype=torch.int64, device="cuda")
    a, _, _ = _run(mean, std, 31337, rng)
    z = ((a - mean.numpy()) / std.numpy()[None]).ravel()
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert st.kstest(z, "norm").pvalue > 1e-3
    # per-action columns are independent of one another
    c = np.corrcoef(z.reshape(B, n).T)
    assert np.abs(c - np.eye(n)).max() < 0.08


def test_ppo_epilogue_argument_checks():
    lib = N.load()
    m = torch.zeros(4, 29, device="cuda")
    s = torch.ones(29, device="cuda")
    rng = torch.zeros(2, dtype=torch.int64, device="cuda")
    a = torch.empty(4, 29, device="cuda")
    lp = torch.empty(4, device="cuda")
    st_ = N.stream_handle()
    assert lib.glad_ppo_epilogue(m.data_ptr(), 4, 29, s.data_ptr(), 65, 0, rng.data_ptr(), a.data_ptr(), 29,
                                 lp.data_ptr(), None, st_) != 0
    assert lib.glad_ppo_epilogue(m.data_ptr(), 4, 20, s.data_ptr(), 29, 0, rng.data_ptr(), a.data_ptr(), 29,
                                 lp.data_ptr(), None, st_) != 0
    assert lib.glad_ppo_epilogue(m.data_ptr(), 4, 29, s.data_ptr(), 29, 0, None, a.data_ptr(), 29,
                                 lp.data_ptr(), None, st_) != 0
    assert lib.glad_ppo_epilogue(m.data_ptr(), 0, 29, s.data_ptr(), 29, 0, None, None, 29, None, None, st_) == 0
    with pytest.raises(ValueError):
        ppo_epilogue(m, s, 0, rng[:1], a, lp)
