"""Numpy restatement of the qrt INT8 GLAD forward (test infrastructure only).

Arithmetic follows PyTorch eager semantics of the reference on each op:
fp16 tensors are rounded to fp16 after every op, fp32 where the reference
promotes, int8 x int8 products accumulate exactly in int32. Summation order
inside float dot products is whatever numpy's BLAS picks -- the reference's
own order is unspecified as well -- so only integer results are expected to
match bit for bit; float results match within rounding.
"""
from __future__ import annotations

import numpy as np

f16, f32, i8, i32 = np.float16, np.float32, np.int8, np.int32
H1, W1, C1 = 21, 33, 3        # conv1 input (NHWC)           qrt/qconv.py:32
H2, W2, C2 = 11, 17, 16       # conv1 output / conv2 input    qrt/qconv.py:33
P = H2 * W2                   # 187 tokens                    qrt/qconv.py:34
N2 = 64                       # conv2 output channels         qrt/qconv.py:35
K1, K2S = 128, 64             # packed K sizes                qrt/qconv.py:37-38
MAP = H1 * W1 * C1            # 2079
INV127 = f32(1.0 / 127.0)


def _mm16(a, b):
    """fp16 @ fp16 -> fp16 with fp32 accumulation (torch CPU half matmul)."""
    return np.matmul(a.astype(f32), b.astype(f32)).astype(f16)


def _softmax16(x, axis):
    """torch.softmax on fp16: computed in fp32, result rounded to fp16."""
    x = x.astype(f32)
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return (e / e.sum(axis=axis, keepdims=True)).astype(f16)


def _elu16(x):
    x32 = x.astype(f32)
    return np.where(x32 > 0, x32, np.expm1(x32)).astype(f16)


def round_half_away(z):
    """``where(z>=0, floor(z+0.5), ceil(z-0.5))`` in fp32 (qrt/qconv.py:100)."""
    z = z.astype(f32)
    return np.where(z >= 0, np.floor(z + f32(0.5)), np.ceil(z - f32(0.5))).astype(f32)


# -- weight quantisation ------------------------------------------------------
def requant_qlinear(weight, bias, alpha=None, beta=None, s_z=1.0):
    """``QuantLinear.requantize_`` (qrt/qlinear.py:84-102).

    Returns ``w8 [Np,K] int8, dq_scale [Np], s_w [Np], b_prime [Np]`` with the
    rows padded to a multiple of 8 (qrt/qlinear.py:56,76-80; pad rows keep the
    constructor's values: w8 0, scales 1, bias 0).
    """
    W = np.asarray(weight).astype(f32)
    N, K = W.shape
    b = np.asarray(bias).astype(f32) if bias is not None else np.zeros(N, f32)
    if alpha is not None:
        W = W / np.asarray(alpha, f32)[None, :]
        beta = np.asarray(beta, f32) if beta is not None else np.zeros(K, f32)
        b = (b - (W * beta[None, :]).sum(axis=1, dtype=f32)).astype(f32)
    s_w = (np.maximum(np.abs(W).max(axis=1), f32(1e-8)) / f32(127.0)).astype(f32)
    w8 = np.clip(np.rint(W / s_w[:, None]), -128, 127).astype(i8)
    Np = N + (-N) % 8
    w8p = np.zeros((Np, K), i8)
    w8p[:N] = w8
    dq = np.ones(Np, f32)
    dq[:N] = s_w * f32(s_z)
    swp = np.ones(Np, f32)
    swp[:N] = s_w
    bp = np.zeros(Np, f32)
    bp[:N] = b
    return w8p, dq, swp, bp


def bn_affine16(weight, bias, mean, var, eps=1e-5):
    """Eval BatchNorm as ``a*x+c``, evaluated on the fp16 copy's tensors:
    ``a`` is computed in fp16 then widened (qrt/qconv.py:252-255)."""
    w, bb, mu, v = (np.asarray(t).astype(f16) for t in (weight, bias, mean, var))
    # fp16 tensor + python float: computed in fp32, rounded to fp16
    den = np.sqrt((v.astype(f32) + f32(eps)).astype(f16)).astype(f16)
    a = (w / den).astype(f16).astype(f32)
    c = (bb.astype(f32) - a * mu.astype(f32)).astype(f32)
    return a, c


def requant_qcnn(sd, s_z, prefix="map_cnn."):
    """``QuantCNN.requantize_`` without LET (qrt/qconv.py:247-284).

    ``sd`` maps the fp16 model's names (``map_cnn.0.weight``...) to arrays.
    """
    g = lambda k: np.asarray(sd[prefix + k])  # noqa: E731
    a1, c1 = bn_affine16(g("2.weight"), g("2.bias"), g("2.running_mean"), g("2.running_var"))
    a2, c2 = bn_affine16(g("5.weight"), g("5.bias"), g("5.running_mean"), g("5.running_var"))
    s_z = f32(s_z)
    W1 = g("0.weight").astype(f32)                                 # [16,3,5,5]
    w1p = np.zeros((8, 16, C2), f32)
    w1p[:5, :15, :] = W1.transpose(2, 3, 1, 0).reshape(5, 15, C2)
    W2 = g("3.weight").astype(f32)                                 # [64,16,3,3]
    Wp = W2.transpose(2, 3, 1, 0).reshape(3, 48, N2)
    s_w = (np.maximum(np.abs(Wp).max(axis=(0, 1)), f32(1e-8)) / f32(127.0)).astype(f32)
    w8 = np.zeros((3, K2S, N2), i8)
    w8[:, :48, :] = np.clip(np.rint(Wp / s_w[None, None, :]), -128, 127).astype(i8)
    return {
        "w1p": w1p.reshape(K1, C2).astype(f16), "b1f": g("0.bias").astype(f32),
        "qa": (a1 / s_z).astype(f32), "qc": (c1 / s_z).astype(f32),
        "w8": w8, "dq": (s_w * s_z).astype(f32), "b2f": g("3.bias").astype(f32),
        "a2": a2, "c2": c2,
    }


# -- conv chain ---------------------------------------------------------------
def conv1_im2col(x_nhwc):
    """``[B*187, 128]`` fp16 A tile of ``_k_conv1_fused_q`` (qrt/qconv.py:64-87)."""
    x = np.asarray(x_nhwc).astype(f16)
    B = x.shape[0]
    xp = np.zeros((B, H1 + 4, W1 + 4, C1), f16)                   # pad 2 each side
    xp[:, 2:2 + H1, 2:2 + W1, :] = x
    A = np.zeros((B, H2, W2, 8, 16), f16)
    for kh in range(5):
        for kw in range(5):
            patch = xp[:, kh:kh + 2 * H2:2, kw:kw + 2 * W2:2, :]   # [B,11,17,3]
            A[:, :, :, kh, kw * 3:kw * 3 + 3] = patch
    return A.reshape(B * P, K1)


def conv1_fused_q(x_nhwc, w1p, b1, qa, qc, return_z=False):
    """Op ``qrt::conv1_fused_q`` -> z8 ``[B*187,16]`` (qrt/qconv.py:54-103)."""
    A = conv1_im2col(x_nhwc)
    acc = np.matmul(A.astype(f32), np.asarray(w1p).astype(f32), dtype=f32)
    z = np.maximum(acc + np.asarray(b1, f32)[None, :], f32(0.0)).astype(f32)
    z = (z * np.asarray(qa, f32)[None, :] + np.asarray(qc, f32)[None, :]).astype(f32)
    q = np.clip(round_half_away(z), -128.0, 127.0).astype(i8)
    return (q, z) if return_z else q


def conv2_acc(z8, w8):
    """int32 accumulators of ``_k_conv2_int8_fused`` (qrt/qconv.py:135-153).

    The nine taps run as fp32 matrix products: every product of two int8 values
    is at most 2^14 in magnitude and a sum of 144 of them stays below 2^22, so
    every partial sum is an integer that fp32 holds exactly, in any order."""
    z = np.asarray(z8).astype(f32).reshape(-1, H2, W2, C2)
    B = z.shape[0]
    zp = np.zeros((B, H2 + 2, W2 + 2, C2), f32)
    zp[:, 1:1 + H2, 1:1 + W2, :] = z
    w = np.asarray(w8).astype(f32)                                # [3, 64(ks), 64(n)]
    acc = np.zeros((B * P, N2), f32)
    for kh in range(3):
        for kw in range(3):
            tap = np.ascontiguousarray(zp[:, kh:kh + H2, kw:kw + W2, :]).reshape(B * P, C2)
            acc += tap @ w[kh, kw * 16:kw * 16 + 16, :]
    return acc.astype(i32)


def conv2_epilogue(acc, dq, b2, a2, c2):
    """``acc*dq + b`` -> ReLU -> BN2 -> fp16 (qrt/qconv.py:155-163)."""
    y = (acc.astype(f32) * np.asarray(dq, f32)[None, :] + np.asarray(b2, f32)[None, :]).astype(f32)
    y = np.maximum(y, f32(0.0))
    y = (y * np.asarray(a2, f32)[None, :] + np.asarray(c2, f32)[None, :]).astype(f32)
    return y.astype(f16)


def conv2_int8_fused(z8, w8, dq, b2, a2, c2, return_acc=False):
    """Op ``qrt::conv2_int8_fused`` -> ``[B*187,64]`` fp16 (qrt/qconv.py:116-163)."""
    acc = conv2_acc(z8, w8)
    y = conv2_epilogue(acc, dq, b2, a2, c2)
    return (y, acc) if return_acc else y


# -- QuantLinear --------------------------------------------------------------
def qlinear_forward(x, L, act_mode="dynamic", out_features=None, aux=None):
    """``QuantLinear.forward`` inference branch (qrt/qlinear.py:111-138).

    ``L`` holds ``w8, dq_scale, s_w, b_prime, s_z, inv_sz`` and optionally
    ``alpha, beta``. Returns fp16 ``[M, out_features]``.
    """
    x = np.asarray(x).astype(f16)
    has_let = L.get("alpha") is not None
    if has_let:
        z = (x.astype(f32) * np.asarray(L["alpha"], f32)[None, :]).astype(f32)
        z = (z + np.asarray(L["beta"], f32)[None, :]).astype(f32)
    else:
        z = x                                    # stays fp16 (0-d scale does not promote)
    zt = z.dtype.type
    if act_mode == "dynamic":
        amax = np.abs(z).max() if z.size else zt(0)
        s_z = (np.maximum(amax, zt(1e-8)) * zt(1.0 / 127.0)).astype(zt)
        q = np.clip(np.rint((z / s_z).astype(zt)), -128, 127).astype(i8)
        scale = (np.asarray(L["s_w"], f32) * f32(s_z)).astype(f32)
    elif act_mode == "static":
        s_z = f32(L["s_z"])
        q = np.clip(np.rint((z * zt(L["inv_sz"])).astype(zt)), -128, 127).astype(i8)
        scale = np.asarray(L["dq_scale"], f32)
    else:
        raise ValueError(f"unknown act_mode: {act_mode}")
    acc = np.matmul(q.astype(np.int64), np.asarray(L["w8"]).astype(np.int64).T).astype(i32)
    y = (acc.astype(f32) * scale[None, :]).astype(f32)
    y = (y + np.asarray(L["b_prime"], f32)[None, :]).astype(f32)
    n = out_features or y.shape[1]
    if aux is not None:
        aux.update(q=q, acc=acc, s_z=f32(s_z))
    return y[:, :n].astype(f16)


def linear16(x, w, b):
    """fp16 ``F.linear`` (addmm, fp32 accumulation, one rounding)."""
    y = np.matmul(np.asarray(x).astype(f32), np.asarray(w).astype(f32).T)
    if b is not None:
        y = y + np.asarray(b).astype(f32)[None, :]
    return y.astype(f16)


# -- top-k ----------------------------------------------------------------------
def philox4x32_10(ctr, key):
    """Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, "Parallel random
    numbers: as easy as 1, 2, 3", SC 2011), vectorised: ctr is four uint32
    arrays, key two uint32 scalars; returns the four output words."""
    c0, c1, c2, c3 = (np.asarray(x, dtype=np.uint32).copy() for x in ctr)
    k0, k1 = np.uint32(key[0]), np.uint32(key[1])
    m0, m1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
    with np.errstate(over="ignore"):
        for r in range(10):
            if r > 0:
                k0 = np.uint32((int(k0) + 0x9E3779B9) & 0xFFFFFFFF)
                k1 = np.uint32((int(k1) + 0xBB67AE85) & 0xFFFFFFFF)
            p0 = m0 * c0.astype(np.uint64)
            p1 = m1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return c0, c1, c2, c3


def gumbel16(seed, offset, B, n_tok=187):
    """The Gumbel term glad_actor_forward_train adds to the top-k logits: token i
    of env e takes word (i & 3) of philox({i>>2, e, e>>32, offset}, {seed,
    seed>>32}); U = (word >> 21) / 2048 (the fp16 grid of torch.rand on fp16,
    qrt/encoder_opt.py:88); noise = -log(-log(U + 1e-10) + 1e-10) in fp16 steps
    (each log evaluated in fp32 and rounded to fp16; the 1e-10 terms vanish)."""
    env = np.arange(B, dtype=np.uint64)[:, None] * np.ones((1, n_tok), np.uint64)
    tok = np.arange(n_tok, dtype=np.uint64)[None, :] * np.ones((B, 1), np.uint64)
    ctr = [(tok >> np.uint64(2)).astype(np.uint32), (env & np.uint64(0xFFFFFFFF)).astype(np.uint32),
           (env >> np.uint64(32)).astype(np.uint32), np.full(env.shape, offset & 0xFFFFFFFF, np.uint32)]
    words = np.stack(philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)))
    w = np.take_along_axis(words, (tok & np.uint64(3)).astype(np.int64)[None], axis=0)[0]
    u = (w >> np.uint32(21)).astype(np.float32) / np.float32(2048.0)
    with np.errstate(divide="ignore"):
        a = np.log(u).astype(np.float16).astype(np.float32)
        b = np.log(-a).astype(np.float16).astype(np.float32)
    return -b


def obs_normalize(x, mean, var, eps):
    """rsl_rl EmpiricalNormalization.forward (rsl_rl/networks/normalization.py:44-47) with
    std = sqrt(var) as the module keeps it (:67-68): (x - mean) / (std + eps), each step an
    fp32 operation."""
    x, mean, var = (np.asarray(t, f32) for t in (x, mean, var))
    std = np.sqrt(var).astype(f32)
    return ((x - mean).astype(f32) / (std + f32(eps)).astype(f32)).astype(f32)


def ppo_normal(seed, offset, B, n):
    """The N(0,1) draws of glad_ppo_epilogue: pair q = j // 2 of env e takes words
    (2(q&1), 2(q&1)+1) of philox({0x80000000 | q>>1, e, e>>32, offset}, {seed, seed>>32});
    u1 = ((w0 >> 8) + 1) / 2^24, u2 = (w1 >> 8) / 2^24, r = sqrt(-2 log u1) in fp32,
    z[2q] = r cos(2 pi u2), z[2q+1] = r sin(2 pi u2) (Box-Muller; the sine and cosine
    evaluated in float64 and rounded, CUDA's sincospif is within 2 ulp of that)."""
    j = np.arange(n)
    q = j // 2
    env = np.arange(B, dtype=np.uint64)[:, None] * np.ones((1, n), np.uint64)
    qq = np.broadcast_to(q[None, :], (B, n)).astype(np.uint64)
    ctr = [(np.uint64(0x80000000) | (qq >> np.uint64(1))).astype(np.uint32),
           (env & np.uint64(0xFFFFFFFF)).astype(np.uint32), (env >> np.uint64(32)).astype(np.uint32),
           np.full(env.shape, offset & 0xFFFFFFFF, np.uint32)]
    words = np.stack(philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)))
    h = (qq & np.uint64(1)).astype(np.int64)
    w0 = np.take_along_axis(words, (2 * h)[None], axis=0)[0]
    w1 = np.take_along_axis(words, (2 * h + 1)[None], axis=0)[0]
    u1 = ((w0 >> np.uint32(8)) + np.uint32(1)).astype(f32) * f32(2.0 ** -24)
    u2 = (w1 >> np.uint32(8)).astype(f32) * f32(2.0 ** -24)
    r = np.sqrt(f32(-2.0) * np.log(u1).astype(f32)).astype(f32)
    ang = 2.0 * np.pi * u2.astype(np.float64)
    trig = np.where(j[None, :] % 2 == 1, np.sin(ang), np.cos(ang)).astype(f32)
    return (r * trig).astype(f32)


def ppo_log_prob_terms(mean, std, actions):
    """Per-action terms of torch.distributions.Normal(mean, std).log_prob(actions) in fp32:
    (-(a - mean)^2) / (2 std^2) - log(std) - log(sqrt(2 pi))."""
    d = (actions.astype(f32) - mean.astype(f32)).astype(f32)
    var = (std.astype(f32) * std.astype(f32)).astype(f32)
    t = ((-(d * d)).astype(f32) / (f32(2.0) * var)).astype(f32)
    return ((t - np.log(std.astype(f32)).astype(f32)).astype(f32) - f32(0.9189385332046727)).astype(f32)


def butterfly_sum32(terms):
    """Sum of up to 64 terms per row in glad_ppo_epilogue's order: lane l holds terms l and
    l + 32, then five xor butterflies (partners 16, 8, 4, 2, 1 apart), all in fp32."""
    B, n = terms.shape
    v = np.zeros((B, 64), f32)
    v[:, :n] = terms
    lanes = (v[:, :32] + v[:, 32:]).astype(f32)
    idx = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        lanes = (lanes + lanes[:, idx ^ o]).astype(f32)
    return lanes[:, 0]


def ppo_epilogue(mean, std, seed, offset):
    """PPO.act epilogue (rsl_rl/algorithms/ppo.py:129-140; Normal sample and log_prob,
    rsl_rl/modules/actor_critic_encoder.py:329-335,366-367): actions = mean + std z,
    log_prob = the butterfly sum of the per-action log-density terms."""
    mean = np.asarray(mean, f32)
    std = np.asarray(std, f32)
    B, n = mean.shape
    z = ppo_normal(seed, offset, B, n)
    a = (mean + (std[None, :] * z).astype(f32)).astype(f32)
    lp = butterfly_sum32(ppo_log_prob_terms(mean, np.broadcast_to(std[None, :], (B, n)), a))
    return a, lp


def topk_lowest_index(logits, k):
    """Top-k indices ordered by value descending, ties by index ascending."""
    lg = np.asarray(logits).astype(f32)
    order = np.lexsort((np.broadcast_to(np.arange(lg.shape[-1]), lg.shape), -lg), axis=-1)
    return order[..., :k].astype(np.int64)


# -- model-level forward --------------------------------------------------------
class GladWeights:
    """fp16 inference-copy parameters + qrt quantised buffers by qrt name."""

    QL = ("actor_proprio_embedding", "query_projector", "actor.0", "actor.2", "actor.4", "actor.6")

    def __init__(self, sd):
        self.sd = {k: np.asarray(v) for k, v in sd.items()}

    def ql(self, name):
        s = self.sd
        d = {k: s[f"{name}.{k}"] for k in ("w8", "dq_scale", "s_w", "b_prime", "s_z", "inv_sz")}
        d["alpha"] = s.get(f"{name}.alpha")
        d["beta"] = s.get(f"{name}.beta")
        d["out_features"] = s[f"{name}.weight"].shape[0]
        return d

    def cnn(self):
        return {k: self.sd[f"map_cnn.{k}"] for k in ("w1p", "b1f", "qa", "qc", "w8", "dq", "b2f", "a2", "c2")}

    def __getitem__(self, k):
        return self.sd[k]


def encode(obs, Wt: GladWeights, act_mode="dynamic", proprio="actor", noise=None, aux=None):
    """``_encode_terrain_opt`` over QuantCNN / QuantLinear (qrt/encoder_opt.py:41-123).

    ``obs`` is the observation group (fp32 or fp16); it is cast to fp16 first,
    as ``update_distribution_qrt`` does (qrt/integration.py:206). ``noise`` is
    an optional additive perturbation of the top-k logits (the Gumbel term of
    train-mode rollouts, qrt/encoder_opt.py:87-91).
    """
    obs16 = np.asarray(obs).astype(f16)
    B = obs16.shape[0]
    x_nhwc = obs16[:, -MAP:].reshape(B, H1, W1, C1)
    c = Wt.cnn()
    z8 = conv1_fused_q(x_nhwc, c["w1p"], c["b1f"], c["qa"], c["qc"])
    local = conv2_int8_fused(z8, c["w8"], c["dq"], c["b2f"], c["a2"], c["c2"]).reshape(B, P, N2)
    prop = obs16[:, :-MAP]
    if proprio == "actor":
        pe_aux = {}
        L = Wt.ql("actor_proprio_embedding")
        emb = qlinear_forward(prop, L, act_mode, L["out_features"], pe_aux)
    else:
        emb = linear16(prop, Wt["critic_proprio_embedding.weight"], Wt["critic_proprio_embedding.bias"])
        pe_aux = {}
    D = N2
    w2 = np.concatenate([Wt["global_pool_selector.weight"], Wt["topk_scorer.weight"][:, :D]], 0)
    logits2 = _mm16(local.reshape(B * P, D), w2.T).reshape(B, P, 2)
    gc_logits = (logits2[..., 0].astype(f32) + Wt["global_pool_selector.bias"].astype(f32)).astype(f16)
    score_local = logits2[..., 1]
    gc_w = _softmax16(gc_logits, axis=1)                                      # [B,N]
    gc = np.einsum("bn,bnd->bd", gc_w.astype(f32), local.astype(f32)).astype(f16)
    qp_aux = {}
    L = Wt.ql("query_projector")
    qin = np.concatenate([gc, emb], axis=1)
    query = qlinear_forward(qin, L, act_mode, L["out_features"], qp_aux)
    sq = _mm16(query, Wt["topk_scorer.weight"][:, D:].T)
    score_query = (sq.astype(f32) + Wt["topk_scorer.bias"].astype(f32)).astype(f16)   # [B,1]
    topk_logits = (score_local.astype(f32) + score_query.astype(f32)).astype(f16)
    pert = topk_logits if noise is None else (topk_logits.astype(f32) + np.asarray(noise, f32)).astype(f16)
    idx = topk_lowest_index(pert, 32)
    sparse = np.take_along_axis(local, idx[..., None], axis=1)               # [B,32,D]
    foot, attn_w = mha(query, sparse, Wt)
    enc = np.concatenate([foot, gc, prop], axis=1)
    if aux is not None:
        aux.update(z8=z8, local=local, emb=emb, gc_logits=gc_logits, score_local=score_local,
                   gc_w=gc_w, gc=gc, query=query, score_query=score_query,
                   topk_logits=topk_logits, topk_idx=idx, foothold=foot, attn_weights=attn_w,
                   enc=enc, s_pe=pe_aux.get("s_z"), s_qp=qp_aux.get("s_z"),
                   q_pe=pe_aux.get("q"), acc_pe=pe_aux.get("acc"),
                   q_qp=qp_aux.get("q"), acc_qp=qp_aux.get("acc"))
    return enc


def mha(query, sparse, Wt: GladWeights):
    """The encoder's single-query cross-attention (qrt/encoder_opt.py:104-119): query
    ``[B,64]`` over the 32 gathered tokens ``[B,32,64]`` (fp16), 16 heads of 4. Returns
    ``foothold [B,64]`` and the head-mean attention weights ``[B,1,32]``, both fp16."""
    query = np.asarray(query).astype(f16)
    sparse = np.asarray(sparse).astype(f16)
    B, D = query.shape
    Win, bin_ = Wt["mha.in_proj_weight"], Wt["mha.in_proj_bias"]
    q = linear16_2step(query, Win[:D], bin_[:D])
    k = linear16_2step(sparse.reshape(-1, D), Win[D:2 * D], bin_[D:2 * D]).reshape(B, 32, D)
    v = linear16_2step(sparse.reshape(-1, D), Win[2 * D:], bin_[2 * D:]).reshape(B, 32, D)
    H, hd = 16, 4
    qh = q.reshape(B, H, 1, hd)
    kh = k.reshape(B, 32, H, hd).transpose(0, 2, 1, 3)
    vh = v.reshape(B, 32, H, hd).transpose(0, 2, 1, 3)
    scores = (_mm16(qh, kh.transpose(0, 1, 3, 2)).astype(f32) * f32(0.5)).astype(f16)
    attn = _softmax16(scores, axis=-1)                                        # [B,H,1,32]
    oh = _mm16(attn, vh)                                                      # [B,H,1,4]
    foot = linear16_2step(oh.reshape(B, D), Wt["mha.out_proj.weight"], Wt["mha.out_proj.bias"])
    attn_w = attn[:, :, 0, :].astype(f32).mean(axis=1, keepdims=True).astype(f16)
    return foot, attn_w


def actor_mlp(enc, Wt: GladWeights, act_mode="dynamic", aux=None):
    """The INT8 actor MLP of qrt full mode (``actor.0/2/4/6`` QuantLinear with ELU between,
    rsl_rl/networks/mlp.py:59-83 with qrt/integration.py:42-43) on the fp16 ``encoded`` rows;
    returns the fp16 head output as fp32 ``[B, 29]`` (``.float()``, qrt/integration.py:206)."""
    h = np.asarray(enc).astype(f16)
    for i, n in enumerate(("actor.0", "actor.2", "actor.4", "actor.6")):
        L = Wt.ql(n)
        la = {}
        h = qlinear_forward(h, L, act_mode, L["out_features"], la)
        if aux is not None:
            aux[f"{n}.q"], aux[f"{n}.acc"], aux[f"{n}.s_z"] = la["q"], la["acc"], la["s_z"]
        if i < 3:
            h = _elu16(h)
        if aux is not None:
            aux[f"{n}.out"] = h
    return h.astype(f32)


def critic_mlp(enc, Wt: GladWeights):
    """The fp16 critic MLP (``critic.0/2/4/6``, not quantised, qrt/integration.py:42-43,133-135)
    on the fp16 critic ``encoded`` rows; returns ``[B,1]`` fp32."""
    h = np.asarray(enc).astype(f16)
    for i, n in enumerate(("critic.0", "critic.2", "critic.4", "critic.6")):
        h = linear16(h, Wt[f"{n}.weight"], Wt[f"{n}.bias"])
        if i < 3:
            h = _elu16(h)
    return h.astype(f32)


def linear16_2step(x, w, b):
    """``x @ W.t() + b`` in fp16 as two eager ops (matmul, then add)
    (qrt/encoder_opt.py:108-118)."""
    y = _mm16(np.asarray(x), np.asarray(w).T)
    return (y.astype(f32) + np.asarray(b).astype(f32)[None, :]).astype(f16)


def actor_forward(obs, Wt: GladWeights, act_mode="dynamic", noise=None, aux=None):
    """Compiled ``f_act`` of qrt (qrt/integration.py:129-131): encoder + the
    INT8 actor MLP (``actor.0/2/4/6`` with ELU between, rsl_rl/networks/mlp.py:59-83).
    Returns the action mean ``[B, 29]`` in fp32 (``.float()``, integration.py:206)."""
    h = encode(obs, Wt, act_mode, "actor", noise, aux)
    return actor_mlp(h, Wt, act_mode, aux)


def critic_forward(obs, Wt: GladWeights, act_mode="dynamic", aux=None):
    """Compiled ``f_val`` (qrt/integration.py:133-135): same encoder with the
    fp16 critic proprio embedding, fp16 critic MLP. Returns ``[B,1]`` fp32."""
    h = encode(obs, Wt, act_mode, "critic", None, aux)
    return critic_mlp(h, Wt)


# -- W4A16 actor MLP ----------------------------------------------------------------
# No reference implementation exists (INT4 is future work in README.md:259); this is
# the restatement of the format documented in include/glad_b200.h (GladW4Linear).
def w4_quantize(W, group=64):
    """W [N,K] -> (packed uint8 [N,K/2], scales fp16 [N,ceil(K/group)]): s = absmax/7
    (fp16), q = clamp(rint(W / s), -8, 7), even k in the low nibble."""
    W = np.asarray(W, np.float32)
    n, K = W.shape
    G = -(-K // group)
    Wp = np.zeros((n, G * group), np.float32)
    Wp[:, :K] = W
    s16 = (np.abs(Wp.reshape(n, G, group)).max(axis=-1) / np.float32(7.0)).astype(np.float16)
    sf = s16.astype(np.float32)
    sf = np.where(sf > 0, sf, np.float32(1.0))
    q = np.clip(np.rint(Wp.reshape(n, G, group) / sf[..., None]), -8, 7).astype(np.int16).reshape(n, -1)[:, :K]
    q = (q & 0xF).astype(np.uint8)
    return (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8), s16


def w4_dequant(packed, scales, K, group=64):
    """fp16 W' = fp16(q * s)."""
    lo = (packed & 0xF).astype(np.int16)
    hi = (packed >> 4).astype(np.int16)
    q = np.empty((packed.shape[0], K), np.int16)
    q[:, 0::2] = np.where(lo >= 8, lo - 16, lo)
    q[:, 1::2] = np.where(hi >= 8, hi - 16, hi)
    s = np.asarray(scales, np.float16).astype(np.float32)[:, np.arange(K) // group]
    return (q.astype(np.float32) * s).astype(np.float16)


def w4a16_mlp(x16, layers):
    """layers: 4 x (packed, scales, bias fp16, K). Hidden: fp16(x W'^T + b) then ELU in
    fp16; head: float(fp16(x W'^T + b)). Accumulation in float64 (the kernel: fp32)."""
    h = np.asarray(x16, np.float16)
    for i, (packed, scales, bias, K) in enumerate(layers):
        Wd = w4_dequant(packed, scales, K).astype(np.float64)
        y = (h[:, :K].astype(np.float64) @ Wd.T + np.asarray(bias, np.float16).astype(np.float64)).astype(np.float16)
        if i < 3:
            yf = y.astype(np.float32)
            y = np.where(yf > 0, yf, np.expm1(yf)).astype(np.float16)
        h = y
    return h.astype(np.float32)
