"""Parity of the fused forwards against the oracle at the benchmarked batch.

At B = 4096 every front CTA runs ~14 environments through its software
pipeline (conv1 of environment e+1 under conv2 of e, the next environment's
epilogue under the logits GEMM), the tail runs two groups of 7 environments per
CTA, the dynamic scales are batch-wide absmax reductions over all 4096 rows,
and the actor MLP runs as one cluster kernel behind grid barriers. B = 3001 is
a second batch in that regime that is not a multiple of the tail's 7-environment
groups. Every comparison is against the oracle (the reference's INT8 path
restated on the CPU, qrt/encoder_opt.py:41-123, qrt/qlinear.py:111-138,
qrt/qconv.py:54-163), computed over the whole batch.

Tiers (the accuracy target: int32 accumulators and top-32 indices bit-exact, means and
values within max-abs 1e-2 and cosine >= 0.99999):
- z8 equal except rounding ties (one step, the oracle's pre-rounding value
  within 1e-3 of a half-integer);
- conv2 features, given the kernel's own z8: integer part exact, epilogue within
  one fp16 ulp;
- proprio embedding (int8 GEMM over the exact fp16 proprio): bit-exact, and its
  dynamic scale exactly the oracle's;
- query projector, given the kernel's own gc and proprio embedding: bit-exact
  output and, in dynamic mode, exactly the oracle's scale over the whole batch;
- top-32: exact (value desc, index asc) on the kernel's own logits; the same SET
  as the oracle's own top-32 for every environment except those whose oracle
  32nd and 33rd logits lie within one fp16 ulp (the count is reported) or
  within twice that environment's measured logit difference;
- attention and foothold, given the kernel's query, selection and features:
  fp16 tolerance;
- actor MLP, given the kernel's own `encoded`: means bit-exact and, in dynamic
  mode, all four layer scales exactly the oracle's;
- means / values end to end: max-abs 1e-2, cosine >= 0.99999.
"""
import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200.synthetic import glad_obs, glad_obs_pair

from gpu_util import DeviceWeights, actor_critic_forward, actor_forward, critic_forward, fp16_ulp_close

pytestmark = pytest.mark.gpu

MAX_ABS = 1e-2
MIN_COS = 0.99999
QL = ("actor_proprio_embedding", "query_projector", "actor.0", "actor.2", "actor.4", "actor.6")


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


def topk_sets(kernel_idx, kernel_logits, oracle_logits):
    """Per environment: equal top-32 sets, the oracle's 32nd-33rd gap within one
    fp16 ulp, and the gap within twice the environment's largest logit difference."""
    lo = np.asarray(oracle_logits, np.float16).astype(np.float32)
    lk = np.asarray(kernel_logits, np.float16).astype(np.float32)
    oidx = O.topk_lowest_index(lo, 32)
    same = np.array([set(a) == set(b) for a, b in zip(kernel_idx, oidx)])
    srt = -np.sort(-lo, axis=1)
    l32, l33 = srt[:, 31], srt[:, 32]
    sp = np.maximum(np.spacing(np.abs(l32).astype(np.float16)), np.spacing(np.abs(l33).astype(np.float16)))
    gap = l32 - l33
    near_ulp = gap <= sp.astype(np.float32)
    d = np.abs(lk - lo).max(axis=1)
    near_diff = gap <= 2 * d
    return same, near_ulp, near_diff


@pytest.fixture(scope="module")
def dw(golden_weights):
    return DeviceWeights(golden_weights)


@pytest.fixture(scope="module")
def Wt(golden_weights):
    return O.GladWeights(golden_weights)


@pytest.mark.parametrize("B,mode", [(4096, "dynamic"), (4096, "static"), (3001, "dynamic"), (3001, "static")])
def test_actor_full_batch_vs_oracle(dw, Wt, golden_weights, B, mode):
    w = golden_weights
    obs = glad_obs(B, seed=5150 + B)
    mean, aux = actor_forward(dw, obs.cuda(), mode)
    oaux = {}
    ref = O.actor_forward(obs.numpy(), Wt, mode, aux=oaux)
    a = {k: v.cpu().numpy() for k, v in aux.items()}
    m = mean.cpu().numpy()

    # end to end
    assert np.isfinite(m).all()
    assert np.abs(m - ref).max() <= MAX_ABS, float(np.abs(m - ref).max())
    assert cos(m, ref) >= MIN_COS

    # z8: one step at most, and only where the oracle's value sits on a rounding tie
    x_nhwc = obs[:, 96:].half().numpy().reshape(B, 21, 33, 3)
    c = Wt.cnn()
    z8o, zo = O.conv1_fused_q(x_nhwc, c["w1p"], c["b1f"], c["qa"], c["qc"], return_z=True)
    assert np.array_equal(z8o, oaux["z8"])
    dz = np.abs(a["z8"].astype(np.int16) - z8o.astype(np.int16))
    assert dz.max() <= 1
    flip = dz > 0
    if flip.any():
        zf = np.abs(zo[flip])
        assert np.all(np.abs(zf - np.floor(zf) - 0.5) < 1e-3), "z8 differs away from a rounding tie"
    # conv2 features given the kernel's z8: integer part exact, epilogue within one fp16 ulp
    loc = O.conv2_int8_fused(a["z8"], w["map_cnn.w8"], w["map_cnn.dq"], w["map_cnn.b2f"], w["map_cnn.a2"],
                             w["map_cnn.c2"]).reshape(B, 187, 64)
    fp16_ulp_close(a["local"], loc)

    # proprio embedding: bit-exact, scale exact
    assert np.array_equal(a["proprio_emb"], oaux["emb"])
    scales = a["act_scales"]
    if mode == "dynamic":
        assert scales[0] == oaux["s_pe"]
    else:
        np.testing.assert_array_equal(scales, [w[f"{n}.s_z"] for n in QL])

    # query projector given the kernel's gc and proprio embedding: bit-exact
    enc = a["encoded"]
    qin = np.concatenate([enc[:, 64:128], a["proprio_emb"]], axis=1)
    qa = {}
    L = Wt.ql("query_projector")
    q_ref = O.qlinear_forward(qin, L, mode, L["out_features"], qa)
    assert np.array_equal(a["query"], q_ref)
    if mode == "dynamic":
        assert scales[1] == qa["s_z"]
    # gc and pooling weights against the oracle's own
    np.testing.assert_allclose(a["gc_weights"].astype(np.float32), oaux["gc_w"].astype(np.float32),
                               atol=2e-3, rtol=2e-2)
    assert cos(enc[:, 64:128], oaux["gc"]) > 0.99999
    assert np.array_equal(enc[:, 128:], obs[:, :96].half().numpy())

    # top-32: exact on the kernel's logits; the oracle's set except at near ties
    idx = a["topk_idx"]
    assert np.array_equal(idx, O.topk_lowest_index(a["topk_logits"], 32))
    same, near_ulp, near_diff = topk_sets(idx, a["topk_logits"], oaux["topk_logits"])
    miss = ~same
    msg = (f"top-32 sets differ in {int(miss.sum())} of {B} environments; oracle 32nd/33rd logits within one "
           f"fp16 ulp in {int(near_ulp.sum())} environments ({int((miss & near_ulp).sum())} of the differing ones), "
           f"within twice the logit difference in {int((miss & near_diff & ~near_ulp).sum())} more")
    print(msg)
    assert np.all(same | near_ulp | near_diff), msg
    assert (miss & ~near_ulp).sum() <= max(2, B // 1000), msg

    # attention and foothold given the kernel's query, selection and features
    sparse = np.take_along_axis(a["local"], idx[..., None], axis=1)
    foot, attn_w = O.mha(a["query"], sparse, Wt)
    np.testing.assert_allclose(a["attn_weights"].astype(np.float32), attn_w[:, 0, :].astype(np.float32),
                               atol=1e-3, rtol=1e-2)
    # foothold = out_proj(attention) + bias sums with cancellation: near zero a small absolute
    # difference spans many ulps, so the bound is absolute plus relative
    fk, fo = enc[:, :64].astype(np.float32), foot.astype(np.float32)
    np.testing.assert_allclose(fk, fo, atol=2e-3, rtol=1e-2)
    assert (fk == fo).mean() >= 0.99, float((fk == fo).mean())
    assert cos(enc[:, :64], oaux["foothold"]) > 0.9999

    # actor MLP given the kernel's encoded rows: bit-exact means and scales
    ma = {}
    m_ref = O.actor_mlp(enc, Wt, mode, ma)
    assert np.array_equal(m, m_ref)
    if mode == "dynamic":
        for i, n in enumerate(("actor.0", "actor.2", "actor.4", "actor.6")):
            assert scales[2 + i] == ma[f"{n}.s_z"], n


@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_critic_full_batch_vs_oracle(dw, Wt, mode):
    B = 4096
    obs = glad_obs(B, seed=6160, proprio_dim=99)
    v, aux = critic_forward(dw, obs.cuda(), mode)
    oaux = {}
    ref = O.critic_forward(obs.numpy(), Wt, mode, aux=oaux)
    a = {k: t.cpu().numpy() for k, t in aux.items()}
    got = v.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= MAX_ABS, float(np.abs(got - ref).max())
    assert cos(got, ref) >= MIN_COS
    enc = a["encoded"][:, :227]
    assert np.array_equal(enc[:, 128:], obs[:, :99].half().numpy())
    # fp16 critic embedding: one rounding of an fp32 sum of 99 products in another order; sums
    # that cancel to near zero differ by more ulps than the absolute difference suggests
    pk, po_ = a["proprio_emb"].astype(np.float32), oaux["emb"].astype(np.float32)
    np.testing.assert_allclose(pk, po_, atol=1e-3, rtol=2e-3)
    assert (pk == po_).mean() >= 0.99, float((pk == po_).mean())
    # query projector given the kernel's gc and embedding: bit-exact
    qin = np.concatenate([enc[:, 64:128], a["proprio_emb"]], axis=1)
    L = Wt.ql("query_projector")
    assert np.array_equal(a["query"], O.qlinear_forward(qin, L, mode, L["out_features"]))
    idx = a["topk_idx"]
    assert np.array_equal(idx, O.topk_lowest_index(a["topk_logits"], 32))
    same, near_ulp, near_diff = topk_sets(idx, a["topk_logits"], oaux["topk_logits"])
    msg = (f"critic top-32 sets differ in {int((~same).sum())} of {B}; near ties (one ulp) "
           f"{int(near_ulp.sum())}")
    print(msg)
    assert np.all(same | near_ulp | near_diff), msg
    sparse = np.take_along_axis(a["local"], idx[..., None], axis=1)
    foot, attn_w = O.mha(a["query"], sparse, Wt)
    np.testing.assert_allclose(a["attn_weights"].astype(np.float32), attn_w[:, 0, :].astype(np.float32),
                               atol=1e-3, rtol=1e-2)
    assert cos(enc, oaux["enc"]) > 0.9999
    # fp16 critic MLP given the kernel's encoded rows: fp32 accumulation in another order
    v_ref = O.critic_mlp(enc, Wt)
    assert np.abs(got - v_ref).max() <= 2e-3
    assert cos(got, v_ref) >= 0.999999


@pytest.mark.parametrize("mode", ["dynamic", "static"])
def test_actor_critic_full_batch_vs_oracle(dw, Wt, mode):
    B = 4096
    po, co = glad_obs_pair(B, seed=7170)
    mean, value = actor_critic_forward(dw, po.cuda(), co.cuda(), mode)
    m_ref = O.actor_forward(po.numpy(), Wt, mode)
    v_ref = O.critic_forward(co.numpy(), Wt, mode)
    m, v = mean.cpu().numpy(), value.cpu().numpy()
    assert np.isfinite(m).all() and np.isfinite(v).all()
    assert np.abs(m - m_ref).max() <= MAX_ABS and cos(m, m_ref) >= MIN_COS
    assert np.abs(v - v_ref).max() <= MAX_ABS and cos(v, v_ref) >= MIN_COS
    # and exactly what the two separate heads return
    m1, _ = actor_forward(dw, po.cuda(), mode, with_aux=False)
    v1, _ = critic_forward(dw, co.cuda(), mode, with_aux=False)
    assert torch.equal(mean, m1)
    assert torch.equal(value, v1)
