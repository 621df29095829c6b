"""The qrt-compatible Python API on the GPU: QuantLinear, QuantCNN, the ops,
requantisation, patch_encoder, InferenceRunner (refresh/sync), compared with
the reference goldens and the oracle."""
import copy

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import glad_oracle as O
from rl_quant_b200 import (InferenceRunner, QuantCNN, QuantLinear, patch_encoder, swap, swap_cnn)
from rl_quant_b200.glad_model import build_glad
from rl_quant_b200.qconv import conv2_int8_acc
from rl_quant_b200.synthetic import glad_obs

from gpu_util import fp16_ulp_close, golden_model

pytestmark = pytest.mark.gpu
QL = O.GladWeights.QL


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float((a @ b) / np.sqrt((a @ a) * (b @ b)))


@pytest.fixture(scope="module")
def gm(golden_weights):
    return golden_model(golden_weights)


def test_requant_buffers_match_reference(gm, golden_weights):
    m, _ = gm
    w = golden_weights
    for p in QL:
        q = m.get_submodule(p)
        assert torch.equal(q.w8.cpu(), torch.from_numpy(w[f"{p}.w8"])), p
        assert torch.equal(q.s_w.cpu(), torch.from_numpy(w[f"{p}.s_w"])), p
        assert torch.equal(q.dq_scale.cpu(), torch.from_numpy(w[f"{p}.dq_scale"])), p
        np.testing.assert_allclose(q.b_prime.cpu().numpy(), w[f"{p}.b_prime"], atol=1e-6, rtol=0)
    for k in ("w1p", "b1f", "qa", "qc", "w8", "dq", "b2f", "a2", "c2"):
        assert np.array_equal(getattr(m.map_cnn, k).cpu().numpy(), w[f"map_cnn.{k}"]), k


@pytest.mark.parametrize("mode", ["static", "dynamic"])
@pytest.mark.parametrize("name,M", [("actor_proprio_embedding", 37), ("actor.0", 300), ("actor.2", 129),
                                    ("actor.6", 5)])
def test_quantlinear_forward_bit_exact(gm, golden_weights, mode, name, M):
    m, _ = gm
    q = m.get_submodule(name)
    q.act_mode = mode
    try:
        g = torch.Generator().manual_seed(M)
        x = (torch.randn(M, q.in_features, generator=g) * 0.7).half()
        with torch.inference_mode():
            y = q(x.cuda())
        # the oracle runs on this module's own buffers (bit-exactness is given identical weights)
        L = {k: getattr(q, k).cpu().numpy() for k in ("w8", "dq_scale", "s_w", "b_prime", "s_z", "inv_sz",
                                                      "alpha", "beta")}
        ref = O.qlinear_forward(x.numpy(), L, mode, q.out_features)
        assert y.dtype == torch.float16
        assert np.array_equal(y.cpu().numpy(), ref)
    finally:
        q.act_mode = "dynamic"


def test_quantlinear_training_branch_is_float(gm):
    m, _ = gm
    q = m.get_submodule("actor.2")
    x = torch.randn(4, 512, device="cuda", dtype=torch.float16)
    with torch.enable_grad():
        y = q(x)
    assert torch.equal(y, torch.nn.functional.linear(x, q.weight, q.bias))


def test_quantcnn_ops_match_oracle(gm, golden_weights, golden_conv):
    m, _ = gm
    c = m.map_cnn
    x = torch.from_numpy(golden_conv["x_nhwc"]).cuda()
    with torch.inference_mode():
        z8 = torch.ops.qrt.conv1_fused_q(x, c.w1p, c.b1f, c.qa, c.qc)
        feat = torch.ops.qrt.conv2_int8_fused(z8, c.w8, c.dq, c.b2f, c.a2, c.c2)
        out = c(x.permute(0, 3, 1, 2))
    assert torch.equal(z8.cpu(), torch.from_numpy(golden_conv["z8"]))
    fp16_ulp_close(feat.cpu().numpy(), golden_conv["feat"])
    assert out.shape == (4, 64, 11, 17)
    assert torch.equal(out.permute(0, 2, 3, 1).reshape(-1, 64), feat)
    acc = conv2_int8_acc(z8, c.w8)
    assert np.array_equal(acc.cpu().numpy(), O.conv2_acc(golden_conv["z8"], golden_weights["map_cnn.w8"]))


@pytest.mark.parametrize("mode", ["eager", "manual-graph", "max-autotune"])
def test_runner_act_matches_reference(gm, golden_fwd, mode):
    m, _ = gm
    r = InferenceRunner(m, mode=mode)
    for B in (3, 16):
        d = golden_fwd[B]
        po = torch.from_numpy(d["policy_obs"]).cuda().half()
        mean = r.act(po).float().cpu().numpy()
        ref = d["dynamic.mean"]
        assert np.abs(mean - ref).max() <= 1e-2 and cos(mean, ref) >= 0.99999


@pytest.mark.parametrize("mode", ["eager", "manual-graph"])
def test_runner_act_host_equals_act(gm, golden_fwd, mode):
    """act_host (host obs straight into the graph input, means straight back) gives the
    means of act on the same observations."""
    m, _ = gm
    r = InferenceRunner(m, mode=mode)
    d = golden_fwd[16]
    po = torch.from_numpy(d["policy_obs"]).float()
    out = r.act_host(po.pin_memory())
    torch.cuda.synchronize()
    assert torch.equal(out, r.act(po.cuda()).cpu())
    with pytest.raises(ValueError):
        r.act_host(po.cuda())


@pytest.mark.parametrize("lanes", [1, 2, 3])
def test_runner_act_host_pipelined_calls(gm, lanes):
    """Back-to-back act_host calls without a synchronise in between (the input copy of
    one call overlapping the forward of the previous one) each return act's means of
    their own observations."""
    m, _ = gm
    r = InferenceRunner(m, mode="manual-graph", host_lanes=lanes)
    obs = [glad_obs(64, seed=100 + i).float().pin_memory() for i in range(7)]
    outs = [torch.empty(64, 29, dtype=torch.float32).pin_memory() for _ in obs]
    for o, out in zip(obs, outs):
        r.act_host(o, out)
    torch.cuda.synchronize()
    for o, out in zip(obs, outs):
        assert torch.equal(out, r.act(o.cuda()).cpu())


def test_patched_encoder_outputs(gm, golden_fwd):
    m, _ = gm
    d = golden_fwd[16]
    with torch.inference_mode():
        enc, attn, idx, gcw = m._encode_terrain(torch.from_numpy(d["policy_obs"]).cuda().half())
        mean = m.actor(enc).float().cpu().numpy()
    assert enc.shape == (16, 224) and attn.shape == (16, 1, 32) and gcw.shape == (16, 187, 1)
    ref = d["dynamic.mean"]
    assert np.abs(mean - ref).max() <= 1e-2 and cos(mean, ref) >= 0.99999
    same = [set(a.tolist()) == set(b.tolist()) for a, b in zip(idx.cpu(), d["dynamic.topk_idx"])]
    assert np.mean(same) >= 0.9
    np.testing.assert_allclose(attn.float().cpu().numpy(), d["dynamic.attn_weights"].astype(np.float32),
                               atol=5e-3)


def test_refresh_quant_follows_weight_update(golden_weights, golden_fwd):
    """Perturb conv2's weight, refresh, outputs follow and two calls agree
    (qrt/bench/bench_rollout.py:174-179)."""
    m, _ = golden_model(golden_weights)
    r = InferenceRunner(m, mode="manual-graph")
    po = torch.from_numpy(golden_fwd[16]["policy_obs"]).cuda().half()
    before = r.act(po).clone()
    with torch.no_grad():
        m.map_cnn._modules["3"].weight.mul_(1.02)
        m.get_submodule("actor.0").weight.add_(1e-3)
    r.refresh_quant()
    o1 = r.act(po).clone()
    o2 = r.act(po).clone()
    assert torch.equal(o1, o2)
    assert not torch.equal(o1, before)
    # the refreshed buffers equal a fresh requantisation of the new weights
    sd = {k: v.detach().cpu().numpy() for k, v in m.state_dict().items()}
    c = O.requant_qcnn(sd, float(golden_weights["meta.s_cnn"]))
    assert np.array_equal(c["w8"], m.map_cnn.w8.cpu().numpy())
    q = m.get_submodule("actor.0")
    w8, dq, sw, bp = O.requant_qlinear(sd["actor.0.weight"], sd["actor.0.bias"], sd["actor.0.alpha"],
                                       sd["actor.0.beta"], sd["actor.0.s_z"])
    assert np.array_equal(w8, q.w8.cpu().numpy())


def test_sync_weights_from_master(golden_weights, golden_fwd):
    m, _ = golden_model(golden_weights)
    master = build_glad(seed=0, critic_seed=2).cuda()
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)).float() for k, v in golden_weights.items()
          if k in master.state_dict() and not k.endswith("num_batches_tracked")}
    master.load_state_dict(sd, strict=False)
    with torch.no_grad():
        for p in master.parameters():
            p.add_(1e-3 * torch.randn_like(p))
    r = InferenceRunner(m, mode="manual-graph")
    r.sync_weights_from(master)
    r.sync_weights_from(master)          # graph replay path
    for name, p in master.named_parameters():
        d = dict(m.named_parameters())[name]
        assert torch.equal(d, p.half()), name
    # buffers refreshed from the synced weights
    q = m.get_submodule("actor.2")
    w8, _, sw, _ = O.requant_qlinear(q.weight.cpu().numpy(), q.bias.cpu().numpy(), q.alpha.cpu().numpy(),
                                     q.beta.cpu().numpy(), float(q.s_z))
    assert np.array_equal(w8, q.w8.cpu().numpy()) and np.array_equal(sw, q.s_w.cpu().numpy())


def test_cpu_tensors_are_rejected(gm):
    m, _ = gm
    with torch.inference_mode(), pytest.raises(RuntimeError):
        m.get_submodule("actor.0")(torch.randn(4, 224).half())
    with pytest.raises(RuntimeError):
        QuantLinear(nn.Linear(16, 8))


@pytest.mark.parametrize("mode", ["eager", "manual-graph"])
def test_runner_evaluate_matches_reference(gm, golden_fwd, mode):
    m, _ = gm
    r = InferenceRunner(m, mode=mode, with_critic=True)
    assert r._fused_critic is not None
    for B in (3, 16):
        d = golden_fwd[B]
        v = r.evaluate(torch.from_numpy(d["critic_obs"]).cuda().half()).float().cpu().numpy()
        ref = d["dynamic.value"]
        assert v.shape == (B, 1)
        assert np.abs(v - ref).max() <= 1e-2
