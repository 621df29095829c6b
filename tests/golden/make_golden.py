"""Generate the golden fixtures under tests/golden/ by running the REFERENCE.

Run in a container that has a checkout of the reference (RLQ_REFERENCE names
its root; nothing here needs a GPU):

    RLQ_REFERENCE=<reference checkout> python tests/golden/make_golden.py [--parts ...]

What runs is the reference's own code, unmodified:
  * rsl_rl ``ActorCriticEncoder`` (fp32, seed 0) -- the GLAD model;
  * qrt ``calib.make_plan`` (LET, 200 Adam steps, 512 obs from seed 1),
    ``swap.apply``, ``calib_cnn_scale``, ``swap_cnn``, ``patch_encoder`` --
    the qrt full-mode setup (qrt/integration.py:100-126);
  * qrt ``QuantLinear`` forward (torch._int_mm on the CPU) and
    ``requantize_`` for every buffer;
  * the two Triton kernels of qrt/qconv.py executed by Triton's CPU
    interpreter (TRITON_INTERPRET=1), registered as the CPU kernels of the
    ``qrt::conv1_fused_q`` / ``qrt::conv2_int8_fused`` custom ops.

The only things this script adds are the seeded synthetic observations, the
mocks qrt's own bench harness uses for the absent ``git``/``tensordict``
modules (qrt/bench/_common.py:12-38) and the seeding of torch's global RNG
around ``make_plan`` (whose row sampling is unseeded, qrt/calib.py:80-81).

Outputs (numpy .npz, small):
  glad_weights.npz      fp16 inference-copy state dict + every qrt buffer
  glad_fwd_b{B}.npz     obs + qrt INT8-path outputs/intermediates (dynamic and
                        static s_z) + the fp32 eager outputs
  glad_conv_b4.npz      conv-chain op inputs/outputs from the Triton kernels
  glad_calib.npz        qrt ``calib.make_plan`` (seeded global RNG) run on an fp16
                        copy of this package's GLAD module: the LET alpha/beta and
                        s_z of every INT8 path, for tests/test_calib.py
"""
from __future__ import annotations

import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("RLQ_REFERENCE")
if not REF:
    raise SystemExit("set RLQ_REFERENCE to the root of a checkout of the reference (RL_Quant)")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, REF)
sys.path.insert(0, os.path.join(REF, "rsl_rl"))

for _name in ("git", "tensordict"):
    try:
        __import__(_name)
    except ImportError:
        _m = types.ModuleType(_name)
        if _name == "git":
            _m.Repo = type("Repo", (), {"__init__": lambda self, *a, **k: None})
            _m.InvalidGitRepositoryError = Exception
        else:
            _m.TensorDict = type("TensorDict", (dict,), {})
        sys.modules[_name] = _m

import copy  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn as nn  # noqa: E402

from rsl_rl.modules.actor_critic_encoder import ActorCriticEncoder  # noqa: E402
import qrt.qconv as qconv  # noqa: E402
from qrt import calib, swap, patch_encoder  # noqa: E402
from qrt.qconv import swap_cnn, calib_cnn_scale  # noqa: E402
from qrt.qlinear import QuantLinear  # noqa: E402

from rl_quant_b200.synthetic import glad_obs, glad_obs_pair, ACTOR_PROPRIO, MAP_SIZE  # noqa: E402
from rl_quant_b200.glad_model import build_glad  # noqa: E402

INT8_PATHS = ["actor.0", "actor.2", "actor.4", "actor.6",
              "actor_proprio_embedding", "query_projector"]


# -- the Triton kernels as CPU kernels of the qrt custom ops ----------------
@qconv._op_conv1.register_kernel("cpu")
def _conv1_cpu(x_nhwc, w1p, b1, qa, qc):
    M = x_nhwc.shape[0] * qconv.P
    out = torch.empty(M, qconv.C2, dtype=torch.int8)
    qconv._k_conv1_fused_q.fn[((M + 127) // 128,)](
        x_nhwc.contiguous(), w1p, b1, qa, qc, out, M, BLOCK_M=128)
    return out


@qconv._op_conv2.register_kernel("cpu")
def _conv2_cpu(z8, w8, dq, b2, a2, c2):
    M = z8.shape[0]
    out = torch.empty(M, qconv.N2, dtype=torch.float16)
    qconv._k_conv2_int8_fused.fn[((M + 127) // 128,)](
        z8.contiguous(), w8, dq, b2, a2, c2, out, M, BLOCK_M=128)
    return out


def build_reference_model() -> ActorCriticEncoder:
    """GLAD main config, seed 0; critic-only modules re-initialised from seed 2."""
    torch.manual_seed(0)
    dummy = {"policy_obs": torch.zeros(1, ACTOR_PROPRIO + MAP_SIZE),
             "critic_obs": torch.zeros(1, ACTOR_PROPRIO + 3 + MAP_SIZE)}
    m = ActorCriticEncoder(obs=dummy, obs_groups={"policy": ["policy_obs"], "critic": ["critic_obs"]},
                           num_actions=29, map_scan_dim=(33, 21, 3), mha_dim=64, num_heads=16,
                           cnn_downsample=True, use_global_context=True, topk=32)
    torch.manual_seed(2)
    m.critic_proprio_embedding.reset_parameters()
    for layer in m.critic:
        if isinstance(layer, nn.Linear):
            layer.reset_parameters()
    return m.eval()


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy()


# the calibration golden: qrt's make_plan on the package's own GLAD module
CALIB_SEED, CALIB_OBS_SEED, CALIB_BATCHES, CALIB_ROWS, CALIB_STEPS = 77, 11, 2, 64, 25


def calib_golden():
    """Run qrt ``calib.make_plan`` with torch's global RNG seeded by CALIB_SEED on an
    fp16 copy of ``build_glad(seed=0, critic_seed=2)`` (equal to the reference model,
    checked in main), CALIB_BATCHES batches of CALIB_ROWS observations, LET with
    CALIB_STEPS Adam steps, dynamic act mode; save every path's alpha, beta, s_z."""
    model = build_glad(seed=0, critic_seed=2).half().eval()
    obs = glad_obs(CALIB_BATCHES * CALIB_ROWS, seed=CALIB_OBS_SEED).half()
    batches = [{"policy_obs": obs[i * CALIB_ROWS:(i + 1) * CALIB_ROWS]} for i in range(CALIB_BATCHES)]
    it = iter(batches)
    torch.manual_seed(CALIB_SEED)
    plan = calib.make_plan(model, INT8_PATHS, obs_fn=lambda: next(it), n_calib=CALIB_BATCHES, use_let=True,
                           let_steps=CALIB_STEPS, act_mode="dynamic", verbose=False)
    out = {"meta.seed": np.int64(CALIB_SEED), "meta.obs_seed": np.int64(CALIB_OBS_SEED),
           "meta.batches": np.int64(CALIB_BATCHES), "meta.rows": np.int64(CALIB_ROWS),
           "meta.steps": np.int64(CALIB_STEPS)}
    for p in INT8_PATHS:
        out[f"{p}.alpha"] = to_np(plan[p]["alpha"])
        out[f"{p}.beta"] = to_np(plan[p]["beta"])
        out[f"{p}.s_z"] = np.float64(plan[p]["s_z"])
    np.savez_compressed(os.path.join(HERE, "glad_calib.npz"), **out)
    print(f"[golden] qrt make_plan (seed {CALIB_SEED}) on the package GLAD module: {list(plan)}")


def main(parts):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if "calib" in parts:
        calib_golden()
    if not parts & {"weights", "fwd", "conv"}:
        return
    m32 = build_reference_model()
    # The package's own GLAD module must reproduce the same initialisation.
    mine = build_glad(seed=0, critic_seed=2)
    sd_ref, sd_mine = m32.state_dict(), mine.state_dict()
    assert sd_ref.keys() == sd_mine.keys(), "parameter names differ from the reference"
    for k in sd_ref:
        assert torch.equal(sd_ref[k], sd_mine[k]), f"init differs at {k}"
    print("[golden] package GLAD init == reference init (seed 0 / critic seed 2)")

    # -- qrt full-mode setup on an fp16 copy (qrt/integration.py:100-126) --
    infer = copy.deepcopy(m32).half().eval()
    calib_all = glad_obs(512, seed=1).half()
    batches = [{"policy_obs": calib_all[i * 64:(i + 1) * 64]} for i in range(8)]
    it = iter(batches * 64)
    obs_fn = lambda: next(it)  # noqa: E731
    torch.manual_seed(1234)
    plan = calib.make_plan(infer, INT8_PATHS, obs_fn=obs_fn, n_calib=8, use_let=True,
                           let_steps=200, act_mode="dynamic", verbose=False)
    swapped = swap.apply(infer, plan)
    it = iter(batches * 64)
    s_cnn = calib_cnn_scale(infer, obs_fn, n_batches=8)
    qcnn = swap_cnn(infer, s_cnn)
    patch_encoder(infer)
    infer.eval()
    print(f"[golden] s_cnn={s_cnn:.6g}; LET plan for {list(plan)}")

    w = {}
    for k, v in infer.state_dict().items():
        w[k] = to_np(v)
    w["meta.s_cnn"] = np.float32(s_cnn)
    for p in INT8_PATHS:
        w[f"plan.{p}.s_z"] = np.float64(plan[p]["s_z"])
    np.savez_compressed(os.path.join(HERE, "glad_weights.npz"), **w)

    # -- conv chain op fixture (config 2 semantics, reference kernels) -----
    x_map = glad_obs(4, seed=7)[:, ACTOR_PROPRIO:].half().reshape(4, 21, 33, 3)
    with torch.inference_mode():
        z8 = torch.ops.qrt.conv1_fused_q(x_map, qcnn.w1p, qcnn.b1f, qcnn.qa, qcnn.qc)
        feat = torch.ops.qrt.conv2_int8_fused(z8, qcnn.w8, qcnn.dq, qcnn.b2f, qcnn.a2, qcnn.c2)
        # fp32 float chain for the _test_qconv.py:57-67 style bound
        xm32 = x_map.float().permute(0, 3, 1, 2)
        ref_z = m32.map_cnn[2](torch.relu(m32.map_cnn[0](xm32)))
        ref_full = m32.map_cnn(xm32)
    np.savez_compressed(os.path.join(HERE, "glad_conv_b4.npz"),
                        x_nhwc=to_np(x_map), z8=to_np(z8), feat=to_np(feat),
                        ref_bn1_fp32=to_np(ref_z), ref_chain_fp32=to_np(ref_full))

    # -- end-to-end forwards ------------------------------------------------
    captured: dict[str, torch.Tensor] = {}

    def hook(name):
        def fn(mod, inp, out):
            captured[name + ".in"] = inp[0].detach().clone()
            captured[name + ".out"] = out.detach().clone()
        return fn

    hooks = [infer.get_submodule(p).register_forward_hook(hook(p)) for p in INT8_PATHS]
    hooks.append(qcnn.register_forward_hook(hook("map_cnn")))
    hooks.append(infer.critic_proprio_embedding.register_forward_hook(hook("critic_proprio_embedding")))

    for B, seed in ((16, 1234), (3, 99), (1, 5)):
        po, co = glad_obs_pair(B, seed)
        out = {"policy_obs": to_np(po), "critic_obs": to_np(co)}
        for mode in ("dynamic", "static"):
            for ql in swapped.values():
                ql.act_mode = mode
            captured.clear()
            with torch.inference_mode():
                mean, att_w, idx, gc_w = infer.act_inference({"policy_obs": po.half()})
            out[f"{mode}.mean"] = to_np(mean.float())
            out[f"{mode}.attn_weights"] = to_np(att_w)
            out[f"{mode}.topk_idx"] = to_np(idx)
            out[f"{mode}.gc_weights"] = to_np(gc_w)
            for k, v in captured.items():
                if k.startswith("map_cnn") and B > 4:
                    v = v[:2]
                out[f"{mode}.{k}"] = to_np(v)
            with torch.inference_mode():
                enc, _, idx_c, _ = infer._encode_terrain(co.half())
                value = infer.critic(enc)
            out[f"{mode}.value"] = to_np(value.float())
            out[f"{mode}.critic_topk_idx"] = to_np(idx_c)
        for ql in swapped.values():
            ql.act_mode = "dynamic"
        with torch.inference_mode():
            m_fp32, _, idx32, _ = m32.act_inference({"policy_obs": po})
            v_fp32 = m32.evaluate({"critic_obs": co})
        out["fp32.mean"] = to_np(m_fp32)
        out["fp32.topk_idx"] = to_np(idx32)
        out["fp32.value"] = to_np(v_fp32)
        np.savez_compressed(os.path.join(HERE, f"glad_fwd_b{B}.npz"), **out)
        cos = torch.nn.functional.cosine_similarity(
            torch.from_numpy(out["dynamic.mean"]).flatten(), m_fp32.flatten(), dim=0).item()
        print(f"[golden] B={B}: qrt INT8 (dynamic) vs fp32 eager mean cos={cos:.6f}")
    for h in hooks:
        h.remove()


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--parts", default="weights,fwd,conv,calib",
                    help="comma-separated subset of weights,fwd,conv,calib (weights, fwd and conv "
                         "are written together)")
    main(set(ap.parse_args().parts.split(",")))
