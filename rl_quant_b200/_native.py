"""ctypes binding of the C ABI in ``include/glad_b200.h`` (``libglad_b200.so``).

There is no fallback: if the library is missing or the device is not an
sm_100 part, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p

import torch

LIB_NAME = "libglad_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

GLAD_OK = 0
GLAD_ERR_INVALID_ARG = -1
GLAD_ERR_CUDA = -2
GLAD_ERR_DEVICE = -3
GLAD_ERR_UNSUPPORTED = -4
GLAD_ERR_WORKSPACE = -5

DTYPE_F32 = 0
DTYPE_F16 = 1
ACT_STATIC = 0
ACT_DYNAMIC = 1
ACT_MODES = {"static": ACT_STATIC, "dynamic": ACT_DYNAMIC}
NOALLOC_MAX_B = 2048      # GLAD_NOALLOC_MAX_B


class GladConvWeights(Structure):
    _fields_ = [(n, c_void_p) for n in ("w1p", "b1f", "qa", "qc", "w8", "dq", "b2f", "a2", "c2")]


class GladQLinear(Structure):
    _fields_ = [(n, c_void_p) for n in ("w8", "dq_scale", "s_w", "b_prime", "alpha", "beta", "s_z", "inv_sz")] + [
        ("in_features", c_int32), ("out_features", c_int32)]


class GladObsNorm(Structure):
    _fields_ = [("mean", c_void_p), ("var", c_void_p), ("eps", c_float), ("n", c_int32)]


class GladActorWeights(Structure):
    _fields_ = [("conv", GladConvWeights), ("proprio_emb", GladQLinear), ("query_proj", GladQLinear)] + [
        (n, c_void_p) for n in ("gps_w", "gps_b", "scorer_w", "scorer_b", "mha_in_w", "mha_in_b",
                                "mha_out_w", "mha_out_b")] + [("mlp", GladQLinear * 4), ("obs_norm", GladObsNorm)]


class GladLinear16(Structure):
    _fields_ = [("weight", c_void_p), ("bias", c_void_p), ("in_features", c_int32), ("out_features", c_int32)]


class GladCriticWeights(Structure):
    _fields_ = [("conv", GladConvWeights), ("proprio_emb", GladLinear16), ("proprio_emb_q", GladQLinear),
                ("query_proj", GladQLinear)] + [
        (n, c_void_p) for n in ("gps_w", "gps_b", "scorer_w", "scorer_b", "mha_in_w", "mha_in_b",
                                "mha_out_w", "mha_out_b")] + [("mlp", GladLinear16 * 4), ("obs_norm", GladObsNorm)]


class GladActorAux(Structure):
    _fields_ = [(n, c_void_p) for n in ("z8", "local", "gc_weights", "score_local", "topk_logits",
                                        "topk_idx", "attn_weights", "encoded", "act_scales",
                                        "proprio_emb", "query")]


class GladQLinearSrc(Structure):
    _fields_ = [("weight", c_void_p), ("bias", c_void_p), ("w_dtype", c_int32), ("N", c_int32),
                ("K", c_int32), ("Np", c_int32)] + [
        (n, c_void_p) for n in ("alpha", "beta", "s_z", "w8", "dq_scale", "s_w", "b_prime")]


class GladQCNNSrc(Structure):
    _fields_ = [(n, c_void_p) for n in (
        "conv1_w", "conv1_b", "bn1_w", "bn1_b", "bn1_mean", "bn1_var",
        "conv2_w", "conv2_b", "bn2_w", "bn2_b", "bn2_mean", "bn2_var", "s_z")] + [
        ("eps1", c_float), ("eps2", c_float)] + [
        (n, c_void_p) for n in ("w1p", "b1f", "qa", "qc", "w8", "dq", "b2f", "a2", "c2")] + [
        ("dtype", c_int32), ("alpha", c_void_p), ("beta", c_void_p)]


class GladW4Linear(Structure):
    _fields_ = [("packed", c_void_p), ("scales", c_void_p), ("bias", c_void_p), ("in_features", c_int),
                ("out_features", c_int)]


class GladPackItem(Structure):
    _fields_ = [("tensor", c_void_p), ("nbytes", c_size_t), ("offset", c_size_t)]


class GladCastCopy(Structure):
    _fields_ = [("src", c_void_p), ("dst", c_void_p), ("n", c_int64), ("src_dtype", c_int32),
                ("dst_dtype", c_int32)]


# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "glad_last_error": (c_char_p, []),
    "glad_abi_version": (c_int, []),
    "glad_conv1_fused_q": (c_int, [c_void_p, c_int64, POINTER(GladConvWeights), c_void_p, c_void_p]),
    "glad_conv2_int8_fused": (c_int, [c_void_p, c_int64, POINTER(GladConvWeights), c_void_p, c_void_p, c_void_p]),
    "glad_conv_chain": (c_int, [c_void_p, c_int64, POINTER(GladConvWeights), c_void_p, c_void_p, c_void_p]),
    "glad_qlinear_workspace_size": (c_size_t, []),
    "glad_qlinear_forward": (c_int, [POINTER(GladQLinear), c_int, c_void_p, c_int, c_int64, c_int64, c_void_p,
                                     c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "glad_actor_workspace_size": (c_size_t, [c_int64]),
    "glad_actor_forward": (c_int, [POINTER(GladActorWeights), c_void_p, c_int, c_int64, c_int64, c_int, c_void_p,
                                   c_void_p, POINTER(GladActorAux), c_void_p, c_size_t, c_void_p]),
    "glad_actor_forward_train": (c_int, [POINTER(GladActorWeights), c_void_p, c_int, c_int64, c_int64, c_int,
                                         c_uint64, c_void_p, c_void_p, POINTER(GladActorAux), c_void_p,
                                         c_size_t, c_void_p]),
    "glad_w4a16_mlp_forward": (c_int, [POINTER(GladW4Linear), c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    "glad_actor_forward_w4a16": (c_int, [POINTER(GladActorWeights), POINTER(GladW4Linear), c_void_p, c_int,
                                         c_int64, c_int64, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "glad_actor_critic_workspace_size": (c_size_t, [c_int64]),
    "glad_actor_critic_forward": (c_int, [POINTER(GladActorWeights), POINTER(GladCriticWeights), c_void_p,
                                          c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_void_p, c_void_p,
                                          c_void_p, c_size_t, c_void_p]),
    "glad_actor_critic_forward_train": (c_int, [POINTER(GladActorWeights), POINTER(GladCriticWeights), c_void_p,
                                                c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_uint64,
                                                c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "glad_ppo_epilogue": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int, c_uint64, c_void_p, c_void_p,
                                  c_int64, c_void_p, c_void_p, c_void_p]),
    "glad_critic_workspace_size": (c_size_t, [c_int64]),
    "glad_critic_forward_train": (c_int, [POINTER(GladCriticWeights), c_void_p, c_int, c_int64, c_int64, c_int,
                                          c_uint64, c_void_p, c_void_p, POINTER(GladActorAux), c_void_p, c_size_t,
                                          c_void_p]),
    "glad_pack_layout": (c_size_t, [POINTER(GladPackItem), c_int]),
    "glad_pack_weights": (c_int, [POINTER(GladPackItem), c_int, c_void_p, c_size_t, c_void_p]),
    "glad_unpack_weights": (c_int, [POINTER(GladPackItem), c_int, c_void_p, c_size_t, c_void_p]),
    "glad_critic_forward": (c_int, [POINTER(GladCriticWeights), c_void_p, c_int, c_int64, c_int64, c_int,
                                    c_void_p, c_void_p, POINTER(GladActorAux), c_void_p, c_size_t, c_void_p]),
    "glad_actor_forward_noalloc": (c_int, [POINTER(GladActorWeights), c_void_p, c_int, c_int64, c_int64, c_int,
                                           c_void_p, c_void_p, POINTER(GladActorAux), c_void_p]),
    "glad_actor_noalloc_status": (c_int, [POINTER(c_uint32), c_void_p]),
    "glad_actor_stage_events": (c_int, [POINTER(c_void_p), c_int]),
    "glad_actor_mlp_fused": (c_int, [c_int64, c_int]),
    "glad_actor_kernel_count": (c_int, [c_int64, c_int]),
    "glad_workspace_status": (c_int, [c_void_p, POINTER(c_uint32), c_void_p]),
    "glad_debug_mlp_barrier": (c_int, [c_uint32, c_uint64]),
    "glad_requant_qlinear": (c_int, [POINTER(GladQLinearSrc), c_int, c_void_p]),
    "glad_requant_qcnn": (c_int, [POINTER(GladQCNNSrc), c_void_p]),
    "glad_cast_copy": (c_int, [POINTER(GladCastCopy), c_int, c_void_p]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the library (once). Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{LIB_NAME} is not built ({path}); run `python -m rl_quant_b200.build` "
                           "(nvcc, sm_100a) -- the GLAD B200 path has no CPU or eager fallback")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc == GLAD_OK:
        return
    msg = load().glad_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == GLAD_ERR_INVALID_ARG:
        raise ValueError(text)
    raise RuntimeError(f"{text} (status {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    """The product path runs on the GPU only; CPU tensors are an error."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("rl_quant_b200 kernels need CUDA tensors on an sm_100 device "
                               "(there is no CPU implementation)")


def conv_weights(w1p, b1f, qa, qc, w8, dq, b2f, a2, c2) -> GladConvWeights:
    return GladConvWeights(ptr(w1p), ptr(b1f), ptr(qa), ptr(qc), ptr(w8), ptr(dq), ptr(b2f), ptr(a2), ptr(c2))


def qlinear_struct(m) -> GladQLinear:
    """GladQLinear view of a QuantLinear-like module's buffers."""
    alpha = getattr(m, "alpha", None) if getattr(m, "has_let", False) else None
    beta = getattr(m, "beta", None) if getattr(m, "has_let", False) else None
    return GladQLinear(ptr(m.w8), ptr(m.dq_scale), ptr(m.s_w), ptr(m.b_prime), ptr(alpha), ptr(beta),
                       ptr(m.s_z), ptr(m.inv_sz), int(m.in_features), int(m.out_features))
