"""The critic outside the shared-scan call: its train-mode Gumbel term drawn in the
kernel (glad_critic_forward_train), and critic-width observations through the
patched encoder (qrt/encoder_opt.py:57-66 routes both groups through the rewrite)."""
import numpy as np
import pytest
import torch

from oracle import glad_oracle as O
from rl_quant_b200 import _native as N
from rl_quant_b200.synthetic import glad_obs

from gpu_util import DeviceWeights, critic_forward, critic_weights, fp16_ulp_close, golden_model

pytestmark = pytest.mark.gpu


def _critic_train(dw, obs, seed, offset):
    B, dev = obs.shape[0], obs.device
    value = torch.empty(B, 1, dtype=torch.float32, device=dev)
    aux_t = {"topk_logits": torch.empty(B, 187, dtype=torch.float16, device=dev),
             "topk_idx": torch.empty(B, 32, dtype=torch.int64, device=dev)}
    aux = N.GladActorAux()
    for k, v in aux_t.items():
        setattr(aux, k, v.data_ptr())
    lib = N.load()
    nbytes = lib.glad_critic_workspace_size(B)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    N.check(lib.glad_critic_forward_train(critic_weights(dw), obs.data_ptr(), N.DTYPE_F32, B, obs.stride(0),
                                          N.ACT_DYNAMIC, seed, offset.data_ptr(), value.data_ptr(), aux,
                                          ws.data_ptr(), nbytes, N.stream_handle()), "glad_critic_forward_train")
    st = N.c_uint32(1)
    N.check(lib.glad_workspace_status(ws.data_ptr(), st, N.stream_handle()), "status")
    torch.cuda.synchronize()
    return value, aux_t


@pytest.mark.parametrize("B", [7, 300])
def test_critic_train_mode_gumbel_in_kernel(golden_weights, B):
    dw = DeviceWeights(golden_weights)
    obs = glad_obs(B, seed=61 + B, proprio_dim=99).cuda()
    _, clean = critic_forward(dw, obs, "dynamic")
    offset = torch.tensor([11], dtype=torch.int64, device="cuda")
    value, pert = _critic_train(dw, obs, 1234, offset)
    assert int(offset.item()) == 12
    assert torch.isfinite(value).all()
    expect = (clean["topk_logits"].cpu().numpy().astype(np.float32) + O.gumbel16(1234, 11, B)).astype(np.float16)
    got = pert["topk_logits"].cpu().numpy()
    fin = np.isfinite(expect)
    assert np.array_equal(np.isfinite(got), fin)
    fp16_ulp_close(got[fin], expect[fin])
    assert np.array_equal(pert["topk_idx"].cpu().numpy(), O.topk_lowest_index(got.astype(np.float32), 32))
    _, pert2 = _critic_train(dw, obs, 1234, offset)
    assert int(offset.item()) == 13 and not torch.equal(pert2["topk_logits"], pert["topk_logits"])


def test_patched_encoder_takes_critic_width_observations(golden_weights):
    m, _ = golden_model(golden_weights)
    B = 64
    obs = glad_obs(B, seed=71, proprio_dim=99)
    with torch.inference_mode():
        enc, attn, idx, gcw = m._encode_terrain(obs.half().cuda())
    assert enc.shape == (B, 128 + 99) and attn.shape == (B, 1, 32) and idx.shape == (B, 32)
    assert gcw.shape == (B, 187, 1)
    oaux = {}
    O.encode(obs.numpy(), O.GladWeights(golden_weights), "dynamic", "critic", aux=oaux)
    e = enc.float().cpu().numpy()
    ref = oaux["enc"].astype(np.float32)
    assert np.abs(e - ref).max() <= 2e-2
    assert float((e.ravel() @ ref.ravel()) / np.sqrt((e.ravel() @ e.ravel()) * (ref.ravel() @ ref.ravel()))) > 0.9999
    assert np.array_equal(enc[:, 128:].cpu(), obs[:, :99].half())
    # the same encoder pass as the fused critic's (bit for bit)
    _, aux = critic_forward(DeviceWeights(golden_weights), obs.cuda(), "dynamic")
    assert torch.equal(enc, aux["encoded"][:, :227])
    assert torch.equal(idx, aux["topk_idx"])
