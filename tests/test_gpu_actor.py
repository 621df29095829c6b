"""Fused actor forward (glad_actor_forward) vs the oracle and the reference goldens.

Tolerances of this path's accuracy target: action means within max-abs 1e-2 and
cosine >= 0.99999 of qrt's INT8 path; integer results bit-exact; top-32 index
sets exact on the logits the kernel selected from (value desc, lower index
first on ties).
"""
import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights, actor_forward, actor_forward_train, fp16_ulp_close

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-2
MIN_COS = 0.99999


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


@pytest.fixture(scope="module")
def dw(golden_weights):
    return DeviceWeights(golden_weights)


@pytest.fixture(scope="module")
def Wt(golden_weights):
    return O.GladWeights(golden_weights)


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [1, 3, 16])
def test_actor_matches_reference_golden(dw, golden_fwd, mode, B):
    d = golden_fwd[B]
    mean, _ = actor_forward(dw, torch.from_numpy(d["policy_obs"]).cuda(), mode)
    m = mean.cpu().numpy()
    ref = d[f"{mode}.mean"]
    assert np.abs(m - ref).max() <= MAX_ABS
    assert cos(m, ref) >= MIN_COS


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B,dtype", [(257, torch.float32), (64, torch.float16)])
def test_actor_vs_oracle_with_aux(dw, Wt, golden_weights, mode, B, dtype):
    obs = glad_obs(B, seed=4242 + B)
    mean, aux = actor_forward(dw, obs.to(dtype).cuda(), mode)
    oaux = {}
    ref = O.actor_forward(obs.to(dtype).numpy(), Wt, mode, aux=oaux)
    m = mean.cpu().numpy()
    assert np.abs(m - ref).max() <= MAX_ABS
    assert cos(m, ref) >= MIN_COS
    # z8: equal except rounding ties (one step)
    z8 = aux["z8"].cpu().numpy()
    dz = np.abs(z8.astype(np.int16) - oaux["z8"].astype(np.int16))
    assert dz.max() <= 1 and (dz > 0).mean() < 1e-3
    # local features given the kernel's own z8: integer part exact, epilogue within one fp16 ulp
    w = golden_weights
    loc = O.conv2_int8_fused(z8, w["map_cnn.w8"], w["map_cnn.dq"], w["map_cnn.b2f"], w["map_cnn.a2"],
                             w["map_cnn.c2"]).reshape(B, 187, 64)
    fp16_ulp_close(aux["local"].cpu().numpy(), loc)
    # top-32: exact on the logits the kernel selected from
    lg = aux["topk_logits"].cpu().numpy()
    idx = aux["topk_idx"].cpu().numpy()
    assert np.array_equal(idx, O.topk_lowest_index(lg, 32))
    # and the same sets as the oracle's own path except where the logits differ
    same = [set(a) == set(b) for a, b in zip(idx, oaux["topk_idx"])]
    assert np.mean(same) >= 0.98
    # intermediate fp16 tensors stay within a few fp16 ulps of the oracle
    np.testing.assert_allclose(aux["gc_weights"].cpu().numpy().astype(np.float32),
                               oaux["gc_w"].astype(np.float32), atol=2e-3, rtol=2e-2)
    enc = aux["encoded"].cpu().numpy().astype(np.float32)
    assert cos(enc, oaux["enc"].astype(np.float32)) > 0.9999
    # proprio block of `encoded` is the fp16 cast of the obs, exactly
    assert np.array_equal(aux["encoded"].cpu().numpy()[:, 128:], obs[:, :96].half().numpy())
    scales = aux["act_scales"].cpu().numpy()
    if mode == "dynamic":
        np.testing.assert_allclose(scales[0], oaux["s_pe"], rtol=0, atol=0)
    else:
        np.testing.assert_array_equal(scales, [w[f"{n}.s_z"] for n in
                                               ("actor_proprio_embedding", "query_projector", "actor.0",
                                                "actor.2", "actor.4", "actor.6")])


def test_actor_topk_noise_is_applied(dw, Wt):
    B = 8
    obs = glad_obs(B, seed=9)
    g = torch.Generator().manual_seed(3)
    u = torch.rand(B, 187, generator=g)
    noise = (-torch.log(-torch.log(u + 1e-10) + 1e-10)).half().float()
    _, aux = actor_forward(dw, obs.cuda(), "dynamic", noise=noise.cuda())
    lg = aux["topk_logits"].cpu().numpy()
    assert np.array_equal(aux["topk_idx"].cpu().numpy(), O.topk_lowest_index(lg, 32))
    oaux = {}
    O.actor_forward(obs.numpy(), Wt, "dynamic", noise=noise.numpy(), aux=oaux)
    same = [set(a) == set(b) for a, b in zip(aux["topk_idx"].cpu().numpy(), oaux["topk_idx"])]
    assert np.mean(same) >= 0.9


def test_actor_batch_independence(dw):
    """Static mode: an env's output does not depend on the rest of the batch."""
    obs = glad_obs(40, seed=77).cuda()
    full, _ = actor_forward(dw, obs, "static", with_aux=False)
    part, _ = actor_forward(dw, obs[5:17].contiguous(), "static", with_aux=False)
    assert torch.equal(full[5:17], part)


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [5, 300, 4096])
def test_fused_mlp_equals_per_layer_kernels(dw, mode, B, monkeypatch):
    """The one-kernel actor MLP (clusters + grid barrier) and the one-GEMM-per-layer
    path compute the same integers and the same roundings: means are identical."""
    from rl_quant_b200 import _native as N
    assert N.load().glad_actor_mlp_fused(B, N.ACT_MODES[mode]) == 1
    obs = glad_obs(B, seed=31 + B).cuda()
    fused, _ = actor_forward(dw, obs, mode, with_aux=False)
    monkeypatch.setenv("GLAD_MLP_FUSED", "0")
    assert N.load().glad_actor_mlp_fused(B, N.ACT_MODES[mode]) == 0
    layered, _ = actor_forward(dw, obs, mode, with_aux=False)
    assert torch.isfinite(fused).all()
    assert torch.equal(fused, layered)


@pytest.mark.parametrize("B", [7, 300])
def test_actor_train_mode_gumbel_in_kernel(dw, B):
    """glad_actor_forward_train: perturbed logits = fp16(clean + Philox4x32-10 Gumbel of
    the oracle), the device offset advances by one per call, top-32 on the perturbed
    logits, a new offset draws new noise."""
    obs = glad_obs(B, seed=21 + B).cuda()
    _, clean = actor_forward(dw, obs, "dynamic")
    offset = torch.tensor([5], dtype=torch.int64, device="cuda")
    mean, pert = actor_forward_train(dw, obs, "dynamic", seed=99, offset=offset)
    assert int(offset.item()) == 6
    assert torch.isfinite(mean).all()
    expect = (clean["topk_logits"].cpu().numpy().astype(np.float32) + O.gumbel16(99, 5, B)).astype(np.float16)
    got = pert["topk_logits"].cpu().numpy()
    fin = np.isfinite(expect)
    assert np.array_equal(np.isfinite(got), fin)
    fp16_ulp_close(got[fin], expect[fin])
    lg = got.astype(np.float32)
    assert np.array_equal(pert["topk_idx"].cpu().numpy(), O.topk_lowest_index(lg, 32))
    _, pert2 = actor_forward_train(dw, obs, "dynamic", seed=99, offset=offset)
    assert int(offset.item()) == 7
    assert not torch.equal(pert2["topk_logits"], pert["topk_logits"])


@pytest.mark.parametrize("mode", ["dynamic", "static"])
@pytest.mark.parametrize("B", [1, 150, 4096])
def test_both_fronts_identical(dw, mode, B, monkeypatch):
    """The warp-specialised front (one CTA per SM, default for the actor) and the
    pipelined front (GLAD_FRONT_WS=0) compute the same integers with the same
    summation orders: every output is identical."""
    obs = glad_obs(B, seed=808 + B).cuda()
    monkeypatch.setenv("GLAD_FRONT_WS", "1")
    m1, a1 = actor_forward(dw, obs, mode)
    monkeypatch.setenv("GLAD_FRONT_WS", "0")
    m0, a0 = actor_forward(dw, obs, mode)
    assert torch.isfinite(m1).all()
    assert torch.equal(m1, m0)
    for k in ("z8", "local", "gc_weights", "score_local", "topk_logits", "topk_idx", "attn_weights", "encoded",
              "act_scales", "proprio_emb", "query"):
        assert torch.equal(a1[k], a0[k]), k
