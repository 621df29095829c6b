// Shared definitions of the GLAD kernels: shapes, parameter blocks and the
// element-wise arithmetic that must agree with the reference's qrt semantics.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "../../include/glad_b200.h"
#include "tc05.cuh"

namespace glad {

// GLAD shapes (qrt/qconv.py:32-38, rsl_rl actor_critic_encoder.py:33-38).
constexpr int kH1 = 21, kW1 = 33, kC1 = 3;      // height map, NHWC
constexpr int kH2 = 11, kW2 = 17, kC2 = 16;     // conv1 output
constexpr int kTok = kH2 * kW2;                 // 187 tokens
constexpr int kD = 64;                          // embedding / conv2 channels
constexpr int kMap = kH1 * kW1 * kC1;           // 2079
constexpr int kTopK = 32;
constexpr int kHeads = 16;
constexpr int kEnc = 224;                       // cat(foothold, gc, proprio[96])
constexpr int kActions = 29;

// ---- fused-forward workspace slots --------------------------------------------
// slots[0..5] : running absmax of each quantised layer's input z (dynamic s_z)
//   0 actor_proprio_embedding, 1 query_projector, 2 actor.0, 3 actor.2,
//   4 actor.4, 5 actor.6
// slots[63]   : device status word (DeviceError bits); outside the per-call clear, so it
//               collects every launch since glad_workspace_status last read (and cleared) it
constexpr int kSlotStatus = 63;
constexpr int kSlotCriticQp = 7;        // critic query projector absmax (fused actor + critic)
// slots[16..18] : arrival counters of the fused MLP's grid barriers
// slots[19]     : arrival counter of the front kernel's proprio-absmax grid barrier
constexpr int kSlotMlpBarrier = 16;
constexpr int kSlotFrontBarrier = 19;
constexpr int kSlotTailDone = 20;       // CTAs of the tail kernel that finished (Gumbel offset)
constexpr int kSlotCriticTailDone = 21; // the same for the critic tail of a fused actor + critic call
constexpr int kSlotsBytes = 256;
constexpr int kSlotsClearBytes = kSlotStatus * 4;   // what each call zeroes: everything but the status
static_assert(kDevErrMmaTimeout == GLAD_DEVERR_MMA_TIMEOUT && kDevErrCopyTimeout == GLAD_DEVERR_COPY_TIMEOUT &&
                  kDevErrBadShape == GLAD_DEVERR_BAD_SHAPE && kDevErrBarrierTimeout == GLAD_DEVERR_BARRIER_TIMEOUT,
              "device status bits and their C-ABI names agree");

__device__ __forceinline__ float fp16r(float x) { return __half2float(__float2half_rn(x)); }

// Activation quantisation of QuantLinear (qrt/qlinear.py:123-133).
//  with LET: z = x*alpha + beta in fp32 (two roundings), q = rint(z/s) (dynamic)
//            or rint(z*inv_sz) (static);
//  without : z stays fp16 and the scaled value is rounded to fp16 before rint.
//
// rint(z/s) needs the correctly rounded quotient only near a rounding
// boundary: t = z*RN(1/s) differs from RN(z/s) by at most ~1.8e-7*|z/s|, so
// rint(t) == rint(RN(z/s)) unless t lies within that distance of a
// half-integer; only then is the IEEE division evaluated.
struct ActQuant {
  bool let;
  bool dyn;
  float s;      // dynamic scale (fp32 with LET; fp16-valued without)
  float rcp;    // RN(1/s)
  float inv;    // static inv_sz (fp32 with LET; fp16-valued without)
  __device__ __forceinline__ int quant(float x, float alpha, float beta) const {
    float r;
    if (let) {
      const float z = __fadd_rn(__fmul_rn(x, alpha), beta);
      if (dyn) {
        const float t = __fmul_rn(z, rcp);
        r = rintf(t);
        if (0.5f - fabsf(t - r) <= fabsf(t) * 4.8e-7f) r = rintf(__fdiv_rn(z, s));
      } else {
        r = rintf(__fmul_rn(z, inv));
      }
    } else {
      r = rintf(fp16r(dyn ? __fdiv_rn(x, s) : __fmul_rn(x, inv)));
    }
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int)r;
  }
  // quant() as the low byte of an fp32 bit pattern: the clamped value plus 1.5*2^23
  // rounds to the nearest even integer in the mantissa (equal to rintf for |t| < 2^22,
  // and clamping before rounding equals clamping after, the bounds being integers), so
  // no float->int conversion is needed. The dynamic LET path tests the fast quotient on
  // the clamped value with the wider bound |t - rint(t)| >= 0.4999, which contains every
  // case quant() re-evaluates (|t| <= 128 there, 128*4.8e-7 < 1e-4); a clamped value has
  // no fraction, and both give the clamp bound whenever the fast quotient is outside
  // [-128, 127].
  __device__ __forceinline__ uint32_t qbits(float x, float alpha, float beta) const {
    constexpr float kMagic = 12582912.0f;
    float t;
    if (let) {
      const float z = __fadd_rn(__fmul_rn(x, alpha), beta);
      if (dyn) {
        t = fminf(fmaxf(__fmul_rn(z, rcp), -128.0f), 127.0f);
        const float u = __fadd_rn(t, kMagic);
        if (fabsf(__fsub_rn(t, __fsub_rn(u, kMagic))) < 0.4999f) return __float_as_uint(u);
        t = fminf(fmaxf(rintf(__fdiv_rn(z, s)), -128.0f), 127.0f);
      } else {
        t = fminf(fmaxf(__fmul_rn(z, inv), -128.0f), 127.0f);
      }
    } else {
      t = fminf(fmaxf(fp16r(dyn ? __fdiv_rn(x, s) : __fmul_rn(x, inv)), -128.0f), 127.0f);
    }
    return __float_as_uint(__fadd_rn(t, kMagic));
  }
  // |z| of one input element (what the dynamic absmax reduces).
  __device__ __forceinline__ float absz(float x, float alpha, float beta) const {
    return let ? fabsf(__fadd_rn(__fmul_rn(x, alpha), beta)) : fabsf(x);
  }
};

// Scale of a dynamic layer from its reduced absmax:
//   s_z = absmax.clamp_min(1e-8) * (1/127)      (qrt/qlinear.py:128)
__device__ __forceinline__ float dyn_scale(float amax, bool let) {
  if (let) return __fmul_rn(fmaxf(amax, 1e-8f), (float)(1.0 / 127.0));
  // fp16 tensor: 1e-8 rounds to 0 in fp16; product rounded to fp16.
  return fp16r(__fmul_rn(fmaxf(amax, 0.0f), (float)(1.0 / 127.0)));
}

__device__ __forceinline__ ActQuant make_act_quant(const GladQLinear& L, int act_mode,
                                                   const float* slots, int slot) {
  ActQuant a;
  a.let = L.alpha != nullptr;
  a.dyn = act_mode == GLAD_ACT_DYNAMIC;
  a.s = a.dyn ? dyn_scale(slots[slot], a.let) : 1.0f;
  a.rcp = __fdiv_rn(1.0f, a.s);
  a.inv = a.let ? *L.inv_sz : fp16r(*L.inv_sz);
  return a;
}

// Output scale of row n: s_w*s_z (dynamic) or dq_scale (static) (qlinear.py:130,135).
__device__ __forceinline__ float out_scale(const GladQLinear& L, const ActQuant& a, int n) {
  return a.dyn ? __fmul_rn(L.s_w[n], a.s) : L.dq_scale[n];
}

// int32 accumulator -> output: y = acc*scale + b' in fp32 (qrt/qlinear.py:135).
__device__ __forceinline__ float qlinear_out32(int32_t acc, float scale, float bprime) {
  return __fadd_rn(__fmul_rn((float)acc, scale), bprime);
}
// ... then cast to the fp16 input dtype (qrt/qlinear.py:138).
__device__ __forceinline__ __half qlinear_out(int32_t acc, float scale, float bprime) {
  return __float2half_rn(qlinear_out32(acc, scale, bprime));
}

// ELU on an fp16 value (computed in fp32, rounded to fp16).
__device__ __forceinline__ __half elu16(__half h) {
  float x = __half2float(h);
  return __float2half_rn(x > 0.0f ? x : expm1f(x));
}

// conv2 epilogue (qrt/qconv.py:159-161): ((acc*dq + b) relu) * a2 + c2 with fused
// multiply-adds, as the compiled Triton kernel contracts them; the fp16 rounding is the
// caller's (paired conversions).
__device__ __forceinline__ float conv2_val(int32_t acc, float dq, float b, float a2, float c2) {
  return fmaf(fmaxf(fmaf(i2f_small(acc), dq, b), 0.0f), a2, c2);
}

// fp16 rounding of two fp32 values, back in fp32 (one paired conversion).
__device__ __forceinline__ float2 fp16r2(float x, float y) { return __half22float2(__floats2half2_rn(x, y)); }

// conv1 epilogue (qrt/qconv.py:96-101): relu(acc+b)*qa + qc, round half away
// from zero, clamp to int8.
__device__ __forceinline__ int conv1_quant(float acc, float b, float qa, float qc) {
  float z = fmaxf(__fadd_rn(acc, b), 0.0f);
  z = __fadd_rn(__fmul_rn(z, qa), qc);
  float q = z >= 0.0f ? floorf(__fadd_rn(z, 0.5f)) : ceilf(__fsub_rn(z, 0.5f));
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return (int)q;
}
// conv1_quant() as the low byte of the returned word, without the conversion unit:
// clamping first changes nothing (integer bounds), floor(|z| + 0.5) is the mantissa of
// (|z| + 0.5) + 2^23 added with rounding toward zero, and the sign is applied to the
// integer (two's complement in the low byte).
__device__ __forceinline__ uint32_t conv1_qbits(float acc, float b, float qa, float qc) {
  float z = fmaxf(__fadd_rn(acc, b), 0.0f);
  z = fminf(fmaxf(__fadd_rn(__fmul_rn(z, qa), qc), -128.0f), 127.0f);
  const uint32_t t = __float_as_uint(__fadd_rz(__fadd_rn(fabsf(z), 0.5f), 8388608.0f));
  const uint32_t sgn = (uint32_t)(__float_as_int(z) >> 31);
  return (t ^ sgn) - sgn;
}

// ---- 64-wide cross-lane reduction -----------------------------------------------
// On return lane L holds the warp sums of channels c0 and c0+1 with
// c0 = 32*b4 + 16*b3 + 8*b2 + 4*b1 + 2*b0 (b_i = bit i of L) in v[0], v[1].
__device__ __forceinline__ void warp_reduce64(float (&v)[64], int lane) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const bool up = lane & 16;
    float send = up ? v[i] : v[i + 32];
    float keep = up ? v[i + 32] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const bool up = lane & 8;
    float send = up ? v[i] : v[i + 16];
    float keep = up ? v[i + 16] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 4;
    float send = up ? v[i] : v[i + 8];
    float keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 2;
    float send = up ? v[i] : v[i + 4];
    float keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 1;
    float send = up ? v[i] : v[i + 2];
    float keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
  }
}
__device__ __forceinline__ int reduce64_channel(int lane) {
  return ((lane >> 4) & 1) * 32 + ((lane >> 3) & 1) * 16 + ((lane >> 2) & 1) * 8 +
         ((lane >> 1) & 1) * 4 + (lane & 1) * 2;
}

// 16 values -> warp sums: lanes L and L^16 end with the sum of channel L & 15.
__device__ __forceinline__ float warp_reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 8];
    const float keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 4];
    const float keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 2;
    const float send = up ? v[i] : v[i + 2];
    const float keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  const bool up = lane & 1;
  const float send = up ? v[0] : v[1];
  const float keep = up ? v[1] : v[0];
  const float r = keep + __shfl_xor_sync(0xffffffffu, send, 1);
  return r + __shfl_xor_sync(0xffffffffu, r, 16);
}

// 16 per-lane values v[h] -> every lane gets op over the 32 lanes of each h, combined in
// the butterfly order (partners L^16, L^8, L^4, L^2, L^1) and so bit-identical to 16
// separate xor-butterflies, in 32 shuffles instead of 80: each step hands half of the
// still-open values to the partner (after step k a lane holds 16 >> k of them), the last
// step leaves value h on lanes 2h and 2h+1, and 16 shuffles broadcast the results.
template <bool kMax>
__device__ __forceinline__ void warp_allreduce16(float (&v)[16], int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    w[i] = op(up ? v[i + 8] : v[i], __shfl_xor_sync(0xffffffffu, up ? v[i] : v[i + 8], 16));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    w[i] = op(up ? w[i + 4] : w[i], __shfl_xor_sync(0xffffffffu, up ? w[i] : w[i + 4], 8));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    w[i] = op(up ? w[i + 2] : w[i], __shfl_xor_sync(0xffffffffu, up ? w[i] : w[i + 2], 4));
  }
  {
    const bool up = lane & 2;
    w[0] = op(up ? w[1] : w[0], __shfl_xor_sync(0xffffffffu, up ? w[0] : w[1], 2));
  }
  w[0] = op(w[0], __shfl_xor_sync(0xffffffffu, w[0], 1));
  // lane L now holds the result of h = 8*b4 + 4*b3 + 2*b2 + b1 (bk = bit k of L)
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    const int src = ((h >> 3) & 1) << 4 | ((h >> 2) & 1) << 3 | ((h >> 1) & 1) << 2 | (h & 1) << 1;
    v[h] = __shfl_sync(0xffffffffu, w[0], src);
  }
}

// conv2 weights w8 [3][64 (kw*16 + c)][64 n] (qrt/qconv.py:270-284) -> the MMA B operand
// [5 K-steps][2 taps][64 n][16 c] (tap q = kh*3 + kw; tap 9 is zero filler). One thread
// builds one 4-byte word; a warp reads 32 consecutive n (no bank conflicts in shared
// memory, coalesced in global memory).
__device__ __forceinline__ void conv2_b_relayout(uint8_t* dst, const uint8_t* w8, int tid, int nthr) {
  for (int j = tid; j < 5 * 2 * 64 * 4; j += nthr) {
    const int n = j & 63, g = (j >> 6) & 3, q = j >> 8;     // q = 2*pr + c
    uint32_t word = 0;
    if (q < 9) {
      const uint8_t* src = w8 + ((q / 3) * 64 + (q % 3) * 16 + 4 * g) * 64 + n;
      word = (uint32_t)src[0] | ((uint32_t)src[64] << 8) | ((uint32_t)src[128] << 16) |
             ((uint32_t)src[192] << 24);
    }
    *reinterpret_cast<uint32_t*>(dst + q * 1024 + n * 16 + 4 * g) = word;
  }
}

// ---- Gumbel noise for train-mode rollouts (qrt/encoder_opt.py:87-91) ------------------
// Counter-based generator: Philox4x32 with 10 rounds, the published method of Salmon,
// Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011).
// Token i of environment e draws word (i & 3) of philox(counter = {i >> 2, e_lo, e_hi,
// offset}, key = {seed_lo, seed_hi}); the word's top 11 bits give U on the fp16 grid
// k * 2^-11 in [0, 1), and the noise follows the reference's fp16 steps
// -log(-log(U + 1e-10) + 1e-10) (the 1e-10 terms vanish in fp16).
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
  }
}

__device__ __forceinline__ float gumbel16(uint64_t seed, uint64_t offset, int64_t env, int tok) {
  uint32_t c[4] = {(uint32_t)(tok >> 2), (uint32_t)env, (uint32_t)((uint64_t)env >> 32), (uint32_t)offset};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const uint32_t w = c[tok & 3];
  const float u = (float)(w >> 21) * (1.0f / 2048.0f);
  const float a = fp16r(logf(u));          // log(0) = -inf
  const float b = fp16r(logf(-a));
  return -b;
}

// rsl_rl EmpiricalNormalization of column k (rsl_rl/networks/normalization.py:44-47):
// (x - mean) / (std + eps) with std = sqrt(var) as the module computes it, every step
// an fp32 operation.
__device__ __forceinline__ float obs_norm(float x, const float* mean, const float* var, float eps, int k) {
  return __fdiv_rn(__fsub_rn(x, __ldg(mean + k)), __fadd_rn(__fsqrt_rn(__ldg(var + k)), eps));
}

// ---- kernel parameter blocks -------------------------------------------------------
enum FrontMode : int { kModeConv1 = 0, kModeConv2 = 1, kModeChain = 2, kModeFront = 3 };

struct FrontParams {
  const void* in;          // obs / x_nhwc rows (kModeConv2: z8)
  int64_t ld;              // row stride in elements
  int in_dtype;            // GLAD_DTYPE_*
  int prop_dim;            // columns before the map (0 for the conv operators)
  int64_t B;
  GladConvWeights conv;
  // kModeFront only
  const __half* gps_w;
  const __half* gps_b;
  const __half* scorer_w;
  GladQLinear pe;          // int8 proprio embedding (pe_f16 == 0)
  const __half* pe16_w;    // fp16 proprio embedding [64, prop_dim] (pe_f16 != 0)
  const __half* pe16_b;    // [64]
  int pe_f16;
  int pe_absmax;           // dynamic int8 embedding: reduce slot 0 in-kernel (grid barrier)
  // actor + critic from one read of the scan (dual != 0): the critic group's proprio
  // columns come from `in_c`, its fp16 embedding and encoded row are written too
  int dual;
  const void* in_c;        // critic obs rows (same dtype as `in`)
  int64_t ld_c;
  int prop_dim_c;
  const __half* pec_w;     // critic proprio embedding fp16 [64, prop_dim_c]
  const __half* pec_b;     // [64] or null
  int ld_enc_c;            // row stride of enc_c
  __half* enc_c;           // [B, ld_enc_c]: writes columns 64..127+prop_dim_c
  __half* pe_c_out;        // [B, 64]
  GladQLinear qp;          // only alpha/beta are read (absmax of its input)
  int act_mode;
  int ld_enc;              // row stride of `enc` (>= 128 + prop_dim)
  // observation normaliser of the `in` rows (norm_mean NULL: identity; f32 rows only)
  const float* norm_mean;
  const float* norm_var;
  float norm_eps;
  // outputs
  int8_t* z8_out;          // [B*187,16]
  __half* feat_out;        // [B*187,64]
  int32_t* acc_out;        // [B*187,64]
  __half* score_local;     // [B,187]
  __half* gc_w_out;        // [B,187]
  __half* enc;             // [B,ld_enc]: writes columns 64..127+prop_dim (gc, proprio)
  __half* pe_out;          // [B,64]
  float* slots;
};

struct TailParams {
  int64_t B;
  GladConvWeights conv;
  GladQLinear qp;          // query_projector
  const __half* scorer_w;  // [128]
  const __half* scorer_b;  // [1]
  const __half* in_w;      // [192,64]
  const __half* in_b;      // [192]
  const __half* out_w;     // [64,64]
  const __half* out_b;     // [64]
  const float* a0_alpha;   // LET of the layer after the encoder (absmax of its input)
  const float* a0_beta;
  int a0_absmax;           // reduce that absmax (an INT8 layer follows the encoder)
  int qp_slot;             // slot holding the query projector's input absmax
  int act_mode;
  int ld_enc;              // row stride of `enc`
  int prop_dim;            // proprio columns of `enc` (from column 128)
  const float* noise;      // [B,187] or null
  int gumbel;              // draw the noise in-kernel (Philox4x32-10) instead of reading `noise`
  uint64_t gumbel_seed;
  unsigned long long* gumbel_offset;   // device word: this call's counter offset; advanced by one per call
  int done_slot;           // slot counting finished CTAs (the last one advances the offset)
  const int8_t* z8;        // [B*187,16]
  const __half* score_local;
  const __half* pe;        // [B,64]
  __half* enc;             // [B,ld_enc]: reads 64..127+prop_dim, writes 0..63
  __half* topk_logits_out; // [B,187] or null
  int64_t* topk_idx_out;   // [B,32] or null
  __half* attn_w_out;      // [B,32] or null
  __half* query_out;       // [B,64] query projector output or null
  float* slots;
};

struct PpoParams {
  const float* mean;       // [B, ld_mean]
  int64_t ld_mean;
  const float* std;        // [n]
  int n;                   // actions, 1..64
  int64_t B;
  uint64_t seed;
  unsigned long long* rng; // {offset, finished-block counter}
  float* actions;          // [B, ld_act]
  int64_t ld_act;
  float* log_prob;         // [B]
  float* sigma;            // [B, n] or null
};

struct GemmParams {
  GladQLinear L;
  int act_mode;
  int slot;                // slot of this layer's absmax (dynamic)
  const void* x;           // [M,K]
  int x_dtype;
  int64_t M, ldx;
  __half* y;               // [M,ldy] f16 output (or null)
  int64_t ldy;
  float* y32;              // [M,ldy32] f32 output (or null)
  int64_t ldy32;
  int y32_round16;         // y32 holds float(fp16(y)) instead of the fp32 y
  int elu;                 // apply ELU to the fp16 output
  const float* next_alpha; // LET of the consumer layer (absmax of its input)
  const float* next_beta;
  int next_let;
  int next_slot;           // -1: no absmax for a consumer
  float* slots;
};

}  // namespace glad
