"""Pin the numpy oracle to the reference (golden vectors made by running qrt)."""
import numpy as np
import pytest

from oracle import glad_oracle as O

QL = O.GladWeights.QL


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


@pytest.mark.parametrize("name", QL)
def test_requant_qlinear_matches_reference(golden_weights, name):
    w = golden_weights
    w8, dq, sw, bp = O.requant_qlinear(w[f"{name}.weight"], w[f"{name}.bias"],
                                       w[f"{name}.alpha"], w[f"{name}.beta"], w[f"{name}.s_z"])
    assert np.array_equal(w8, w[f"{name}.w8"])
    assert np.array_equal(dq, w[f"{name}.dq_scale"])
    assert np.array_equal(sw, w[f"{name}.s_w"])
    np.testing.assert_allclose(bp, w[f"{name}.b_prime"], rtol=0, atol=1e-6)


def test_requant_qcnn_matches_reference(golden_weights):
    c = O.requant_qcnn(golden_weights, golden_weights["map_cnn.s_z"])
    for k, v in c.items():
        assert np.array_equal(v, golden_weights[f"map_cnn.{k}"]), k


def test_conv_chain_matches_reference_kernels(golden_weights, golden_conv):
    w, g = golden_weights, golden_conv
    z8 = O.conv1_fused_q(g["x_nhwc"], w["map_cnn.w1p"], w["map_cnn.b1f"], w["map_cnn.qa"], w["map_cnn.qc"])
    assert np.array_equal(z8, g["z8"])
    feat, acc = O.conv2_int8_fused(g["z8"], w["map_cnn.w8"], w["map_cnn.dq"], w["map_cnn.b2f"],
                                   w["map_cnn.a2"], w["map_cnn.c2"], return_acc=True)
    assert np.array_equal(feat, g["feat"])
    assert np.abs(acc).max() < 2 ** 24


def test_conv1_quant_error_bound(golden_weights, golden_conv):
    """The reference's own kernel-1 bound (qrt/bench/_test_qconv.py:57-67)."""
    s_z = float(golden_weights["map_cnn.s_z"])
    z8 = O.conv1_fused_q(golden_conv["x_nhwc"], *(golden_weights[f"map_cnn.{k}"] for k in ("w1p", "b1f", "qa", "qc")))
    z = z8.astype(np.float32).reshape(4, 11, 17, 16).transpose(0, 3, 1, 2) * s_z
    ref = golden_conv["ref_bn1_fp32"]
    inr = np.abs(ref) < 126.0 * s_z
    assert np.abs(z - ref)[inr].max() < 2.0 * s_z + 1e-3


def test_conv_chain_cosine_vs_fp32(golden_conv):
    feat = golden_conv["feat"].astype(np.float32).reshape(4, 11, 17, 64).transpose(0, 3, 1, 2)
    assert cos(feat, golden_conv["ref_chain_fp32"]) > 0.9995


@pytest.mark.parametrize("B", [1, 3, 16])
@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_actor_forward_matches_reference(golden_weights, golden_fwd, B, mode):
    d = golden_fwd[B]
    aux = {}
    mean = O.actor_forward(d["policy_obs"], O.GladWeights(golden_weights), mode, aux=aux)
    ref = d[f"{mode}.mean"]
    assert np.abs(mean - ref).max() <= 1e-3
    assert cos(mean, ref) >= 0.99999
    for a, b in zip(aux["topk_idx"], d[f"{mode}.topk_idx"]):
        assert set(a.tolist()) == set(b.tolist())
    assert np.array_equal(aux["emb"], d[f"{mode}.actor_proprio_embedding.out"])
    # INT8 path stays close to the fp32 eager model (random init, README.md:240 style)
    assert cos(mean, d["fp32.mean"]) > 0.999


@pytest.mark.parametrize("B", [3, 16])
def test_critic_forward_matches_reference(golden_weights, golden_fwd, B):
    d = golden_fwd[B]
    v = O.critic_forward(d["critic_obs"], O.GladWeights(golden_weights), "dynamic")
    assert np.abs(v - d["dynamic.value"]).max() <= 1e-3


def test_topk_tie_rule():
    lg = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float16)
    assert O.topk_lowest_index(lg, 3).tolist() == [[1, 2, 4]]
    assert O.topk_lowest_index(lg, 2).tolist() == [[1, 2]]


def test_philox4x32_10_known_answer():
    """Philox4x32-10 with a zero counter and key (the Random123 known-answer vector)."""
    out = O.philox4x32_10([np.zeros(1, np.uint32)] * 4, (0, 0))
    assert [int(x[0]) for x in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_gumbel16_distribution():
    """The in-kernel Gumbel term: fp16 values with the Gumbel(0, 1) mean and spread."""
    g = O.gumbel16(seed=1234, offset=0, B=2048)
    fin = g[np.isfinite(g)]
    assert np.isinf(g).mean() < 1e-3            # U == 0 (1/2048) gives -inf, never selected
    assert abs(fin.mean() - 0.5772) < 0.02       # Euler-Mascheroni constant
    assert abs(fin.std() - np.pi / np.sqrt(6.0)) < 0.03
    assert np.array_equal(fin, fin.astype(np.float16).astype(np.float32))
    assert not np.array_equal(g, O.gumbel16(seed=1234, offset=1, B=2048))


def test_w4_quantize_host_matches_oracle():
    """The package's W4A16 quantiser (torch) equals the oracle's restatement; the
    dequantised weights stay within half a scale step of the source."""
    import torch
    from rl_quant_b200.w4a16 import quantize_w4
    rng = np.random.default_rng(3)
    W = (rng.standard_normal((29, 224)) * 0.05).astype(np.float32)
    W[3, 64:128] = 0.0                                   # an all-zero group
    p_ref, s_ref = O.w4_quantize(W)
    p, s = quantize_w4(torch.from_numpy(W))
    assert np.array_equal(p.numpy(), p_ref)
    assert np.array_equal(s.numpy(), s_ref)
    Wd = O.w4_dequant(p_ref, s_ref, 224).astype(np.float32)
    step = s_ref.astype(np.float32)[:, np.arange(224) // 64]
    assert np.all(np.abs(Wd - W) <= step * 0.5 + 1e-3 * step + 1e-8)
    assert np.all(Wd[3, 64:128] == 0.0)


def test_ppo_log_prob_terms_match_torch_normal():
    """The oracle's per-action log-density terms are torch.distributions.Normal.log_prob's
    fp32 arithmetic (rsl_rl/modules/actor_critic_encoder.py:366-367)."""
    import torch
    g = torch.Generator().manual_seed(3)
    mean = torch.randn(64, 29, generator=g)
    std = 0.1 + torch.rand(29, generator=g)
    a = mean + std * torch.randn(64, 29, generator=g)
    ref = torch.distributions.Normal(mean, std.expand(64, 29)).log_prob(a).numpy()
    got = O.ppo_log_prob_terms(mean.numpy(), np.broadcast_to(std.numpy()[None], (64, 29)), a.numpy())
    np.testing.assert_allclose(got, ref, rtol=2e-7, atol=1e-6)
    s = O.butterfly_sum32(got)
    np.testing.assert_allclose(s, ref.astype(np.float64).sum(-1), rtol=1e-6, atol=2e-5)


def test_ppo_normal_distribution_and_pairs():
    """Box-Muller draws: N(0,1) marginals, the cosine and sine halves of a pair share
    their radius, distinct offsets and seeds give distinct draws."""
    import scipy.stats as st
    z = O.ppo_normal(7, 0, 2048, 29)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert st.kstest(z.ravel(), "norm").pvalue > 1e-3
    r2 = z[:, 0] ** 2 + z[:, 1] ** 2
    assert np.all(r2 > 0)
    assert not np.array_equal(z, O.ppo_normal(7, 1, 2048, 29))
    assert not np.array_equal(z, O.ppo_normal(8, 0, 2048, 29))
    a, lp = O.ppo_epilogue(np.zeros((3, 29), np.float32), np.ones(29, np.float32), 7, 0)
    assert np.array_equal(a, z[:3])


def test_obs_normalize_matches_empirical_normalization():
    """The oracle's normaliser is the module's forward bit for bit once _std = sqrt(_var)
    (rsl_rl/networks/normalization.py:44-47,67-68)."""
    import torch
    from gpu_util import EmpiricalNorm
    g = torch.Generator().manual_seed(4)
    norm = EmpiricalNorm(2175)
    for _ in range(3):
        norm.update(3.0 * torch.randn(256, 2175, generator=g) + 1.5)
    # on the GPU, where rsl_rl keeps the module, torch.sqrt is IEEE-rounded; torch's CPU
    # sqrt is not always, so take _std as the rounded square root here
    norm._std = torch.from_numpy(np.sqrt(norm._var.numpy()))
    x = 2.0 * torch.randn(64, 2175, generator=g)
    ref = norm(x).numpy()
    got = O.obs_normalize(x.numpy(), norm._mean.numpy(), norm._var.numpy(), norm.eps)
    assert np.array_equal(got, ref)
