// Encoder front: conv1 (fp16 tcgen05) -> conv2 (int8 tcgen05) and, in the
// fused mode, the global softmax pool, the scorer's local logits and the
// proprio embedding, one environment at a time per CTA.
//
// Reference: qrt/qconv.py:54-163 (the two Triton kernels), qrt/encoder_opt.py:
// 41-77 (GPS + scorer-local merged GEMM, softmax pool), qrt/qlinear.py:111-138
// (actor_proprio_embedding).
//
// Shared-memory operand layouts (no swizzle, K-major core matrices of
// 8 rows x 16 bytes). Neither GEMM materialises an im2col matrix: the A
// operand descriptors point into layouts in which consecutive GEMM rows are
// 16 bytes apart, so one descriptor per K chunk walks the whole tile.
//
// conv1 planes (fp16): input rows split by parity, each pixel padded to four
//   halves (x,y,z,0). Plane p, row r holds input row ih = 2r-2+p; pixel slot
//   s holds column iw = s-2; a row is 38 slots = 304 bytes. GEMM row
//   m = oh*19 + ow (ow < 17 valid). The 16-byte chunk (kh, j) of row m (pixels
//   kw = 2j, 2j+1) sits at plane(kh&1) + (kh>>1)*304 + j*16 + m*16.
// conv2 strip (int8): z8 at padded position (oh+1)*18 + (ow+1), 16 channels =
//   16 bytes per position; row 0 / column 0 are zero halo and column 18 wraps
//   onto the next row's halo. GEMM row m = oh*18 + ow; tap (kh,kw) of row m
//   sits at (m + kh*18 + kw)*16.
// Each environment owns two M=128 tiles per GEMM (conv1: 209 rows, conv2:
// 198 rows); rows outside the 11x17 grid are computed and discarded.
#include <cuda_runtime.h>

#include <cstddef>

#include "glad_common.cuh"
#include "front_layout.cuh"

namespace glad {

constexpr int kTmemCols = 128;
constexpr int kFrontThreads = 256;
#ifndef FRONT_MIN_BLOCKS
#define FRONT_MIN_BLOCKS 2
#endif

struct __align__(128) FrontSmem {
  uint8_t planes[kPlanesBytes];
  uint8_t w1s[kW1sBytes];
  uint8_t strip[kStripBytes];
  uint8_t w2s[kW2sBytes];
  uint8_t stage[kStageBytes];
  alignas(16) float b1[16];
  alignas(16) float qa[16];
  alignas(16) float qc[16];
  alignas(16) float dq[64];
  alignas(16) float b2[64];
  alignas(16) float a2[64];
  alignas(16) float c2[64];
  alignas(16) float wg[64];             // GPS weight (local half of the merged GEMM)
  alignas(16) float ws[64];             // scorer weight, local half
  float2 lpart[2][2][128];              // [tile][channel half][row] partial (gps, scorer) logits
  __half wt16[2][128];                  // softmax weights per row of each tile
  float pool[2][4][64];                 // [tile][lane quarter][channel] pooled partial sums
  float wmax[8], wsum[8];
  __half prop16[128];                   // proprio (fp16)
  __half pe16[64];
  __half gc16[64];
  alignas(16) int8_t q8[128];           // quantised proprio
  alignas(16) uint8_t pe_w[64 * kMaxProp * 2];  // proprio embedding rows: int8 or fp16
  float pe_a[kMaxProp], pe_b[kMaxProp]; // int8 embedding: LET alpha / beta
  float pe_scale[64], pe_bp[64];        // its output scale and bias
  float qp_a[128], qp_b[128];           // query_projector LET (absmax of its input)
  uint64_t mbar;
  uint32_t tmem_base;
  int abort_flag;
};


// 32 values -> one warp sum per lane: lane L ends with the sum of channel L.
__device__ __forceinline__ float warp_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 16];
    const float keep = up ? v[i + 16] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
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
  return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

template <int MODE>
__global__ void __launch_bounds__(kFrontThreads, FRONT_MIN_BLOCKS) front_kernel(const __grid_constant__ FrontParams p) {
  extern __shared__ uint8_t smem_raw[];
  FrontSmem& s = *reinterpret_cast<FrontSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;     // TMEM lane quarter, column half / tile
  constexpr int NT = kFrontThreads;
  constexpr bool kConv1 = MODE != kModeConv2;
  constexpr bool kConv2 = MODE != kModeConv1;
  constexpr bool kFront = MODE == kModeFront;

  grid_dep_launch();                    // the next kernel may start its prologue
  // ---- one-time set-up ------------------------------------------------------
  if (warp == 0) tmem_alloc(&s.tmem_base, kTmemCols);
  if (tid == 0) {
    mbar_init(&s.mbar, 1);
    fence_mbar_init();
    s.abort_flag = 0;
  }
  {
    uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < kPlanesBytes / 16; i += NT) reinterpret_cast<uint4*>(s.planes)[i] = z;
    for (int i = tid; i < kStripBytes / 16; i += NT) reinterpret_cast<uint4*>(s.strip)[i] = z;
  }
  if (kConv1) {
    const __half* w1p = reinterpret_cast<const __half*>(p.conv.w1p);
    __half* dst = reinterpret_cast<__half*>(s.w1s);
    for (int idx = tid; idx < kW1sBytes / 2; idx += NT) {
      const int pr = idx >> 8, c = (idx >> 7) & 1, n = (idx >> 3) & 15, e = idx & 7;
      const int q = 2 * pr + c;
      __half v = __float2half(0.0f);
      if (q < 15) {
        const int kh = q / 3, kw = 2 * (q % 3) + (e >> 2), ch = e & 3;
        if (kw < 5 && ch < 3) v = w1p[(kh * 16 + kw * 3 + ch) * 16 + n];
      }
      dst[idx] = v;
    }
    if (tid < 16) {
      s.b1[tid] = p.conv.b1f[tid];
      s.qa[tid] = p.conv.qa[tid];
      s.qc[tid] = p.conv.qc[tid];
    }
  }
  if (kConv2) {
    conv2_b_relayout(s.w2s, reinterpret_cast<const uint8_t*>(p.conv.w8), tid, NT);
    if (tid < 64) {
      s.dq[tid] = p.conv.dq[tid];
      s.b2[tid] = p.conv.b2f[tid];
      s.a2[tid] = p.conv.a2[tid];
      s.c2[tid] = p.conv.c2[tid];
      if (kFront) {
        s.wg[tid] = __half2float(p.gps_w[tid]);
        s.ws[tid] = __half2float(p.scorer_w[tid]);
      }
    }
  }
  grid_dep_wait();                      // inputs of the preceding kernel are visible from here
  // Front-mode constants.
  ActQuant aq_pe{};
  ActQuant aq_qp{};
  float gb = 0.0f;
  float zmax_qp = 0.0f;
  const int P = p.prop_dim;
  if (kFront) {
    if (!p.pe_f16) aq_pe = make_act_quant(p.pe, p.act_mode, p.slots, 0);
    aq_qp.let = p.qp.alpha != nullptr;
    gb = __half2float(p.gps_b[0]);
    if (p.pe_f16) {
      __half* dst = reinterpret_cast<__half*>(s.pe_w);
      for (int i = tid; i < kD * P; i += NT) dst[i] = p.pe16_w[i];
      if (tid < kD) s.pe_bp[tid] = p.pe16_b ? __half2float(p.pe16_b[tid]) : 0.0f;
    } else {
      for (int i = tid; i < kD * P / 4; i += NT)
        reinterpret_cast<int*>(s.pe_w)[i] = reinterpret_cast<const int*>(p.pe.w8)[i];
      for (int k = tid; k < P; k += NT) {
        s.pe_a[k] = aq_pe.let ? p.pe.alpha[k] : 0.0f;
        s.pe_b[k] = aq_pe.let ? p.pe.beta[k] : 0.0f;
      }
      if (tid < kD) {
        s.pe_scale[tid] = out_scale(p.pe, aq_pe, tid);
        s.pe_bp[tid] = p.pe.b_prime[tid];
      }
    }
    if (tid < 128) {
      s.qp_a[tid] = aq_qp.let ? p.qp.alpha[tid] : 0.0f;
      s.qp_b[tid] = aq_qp.let ? p.qp.beta[tid] : 0.0f;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
  uint32_t phase = 0;

  const int esz = (MODE == kModeConv2) ? 1 : (p.in_dtype == GLAD_DTYPE_F32 ? 4 : 2);
  const int row_elems = (MODE == kModeConv2) ? kTok * kC2 : p.prop_dim + kMap;
  int64_t env = blockIdx.x;
  if (env < p.B) row_issue(row_stage(p.in, env, p.ld, esz, row_elems, s.stage), tid, NT);
  cp_async_commit();

  for (; env < p.B; env += gridDim.x) {
    cp_async_wait_all();
    __syncthreads();
    const RowStage rs = row_stage(p.in, env, p.ld, esz, row_elems, s.stage);
    const int64_t nxt = env + gridDim.x;

    if (kConv1) {
      // ---- input -> conv1 planes (fp16) -------------------------------------------
      const int moff = p.prop_dim;
      for (int px = tid; px < kH1 * kW1; px += NT) {
        const int ih = px / kW1, iw = px - ih * kW1;
        float v0, v1, v2;
        if (esz == 4) {
          v0 = row_elem<4>(rs, moff + px * 3);
          v1 = row_elem<4>(rs, moff + px * 3 + 1);
          v2 = row_elem<4>(rs, moff + px * 3 + 2);
        } else {
          v0 = row_elem<2>(rs, moff + px * 3);
          v1 = row_elem<2>(rs, moff + px * 3 + 1);
          v2 = row_elem<2>(rs, moff + px * 3 + 2);
        }
        const int pl = ih & 1, r = ((ih - pl) >> 1) + 1, slot = iw + 2;
        __half2 h01 = __floats2half2_rn(v0, v1);
        __half2 h2z = __floats2half2_rn(v2, 0.0f);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&h01);
        pk.y = *reinterpret_cast<uint32_t*>(&h2z);
        *reinterpret_cast<uint2*>(s.planes + pl * kPlaneBytes + r * kRowBytes + slot * 8) = pk;
      }
      if (kFront) {
        for (int k = tid; k < P; k += NT)
          s.prop16[k] = __float2half_rn(esz == 4 ? row_elem<4>(rs, k) : row_elem<2>(rs, k));
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // stage is free: prefetch the next environment while this one computes
      if (nxt < p.B) row_issue(row_stage(p.in, nxt, p.ld, esz, row_elems, s.stage), tid, NT);
      cp_async_commit();

      if (tid == 0) {
        tc_fence_after();
        const uint32_t pb = smem_u32(s.planes), wb = smem_u32(s.w1s);
        constexpr uint32_t idesc = idesc_f16(128, 16);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int pr = 0; pr < 8; ++pr) {
            const uint32_t c0 = conv1_chunk_off(2 * pr), c1 = conv1_chunk_off(2 * pr + 1);
            const uint64_t ad = smem_desc(pb + c0 + t * 128 * 16, c1 - c0, 128);
            const uint64_t bd = smem_desc(wb + pr * 512, 256, 128);
            mma_f16(tmem + t * 16, ad, bd, idesc, pr > 0 ? 1u : 0u);
          }
        }
        mma_commit(&s.mbar);
      }

      if (kFront) {
        // proprio embedding while the tensor core runs
        if (p.pe_f16) {
          // fp16 nn.Linear: fp32 accumulation, bias, one rounding
          if (tid < 2 * kD) {
            const int n = tid >> 1, part = tid & 1;
            const __half* wrow = reinterpret_cast<const __half*>(s.pe_w) + n * P;
            const int half_k = (P + 1) >> 1;
            const int k0 = part * half_k, k1 = min(P, k0 + half_k);
            float a = 0.0f;
            for (int k = k0; k < k1; ++k) a = fmaf(__half2float(s.prop16[k]), __half2float(wrow[k]), a);
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            if (part == 0) s.pe16[n] = __float2half_rn(a + s.pe_bp[n]);
          }
        } else {
          // W8A8 QuantLinear (qrt/qlinear.py:123-138)
          for (int k = tid; k < P; k += NT)
            s.q8[k] = (int8_t)aq_pe.quant(__half2float(s.prop16[k]), s.pe_a[k], s.pe_b[k]);
          __syncthreads();
          if (tid < 2 * kD) {
            // two threads per output row, each half of K
            const int n = tid >> 1, part = tid & 1;
            const int* wrow = reinterpret_cast<const int*>(s.pe_w + n * P) + part * (P / 8);
            const int* qw = reinterpret_cast<const int*>(s.q8) + part * (P / 8);
            int acc = 0;
            for (int k4 = 0; k4 < P / 8; ++k4) acc = __dp4a(qw[k4], wrow[k4], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            if (part == 0) s.pe16[n] = qlinear_out(acc, s.pe_scale[n], s.pe_bp[n]);
          }
        }
      }

      const bool ok = mbar_wait_bounded(&s.mbar, phase);
      phase ^= 1;
      if (!ok) s.abort_flag = 1;
      tc_fence_after();
      __syncthreads();
      if (s.abort_flag) break;

      // ---- conv1 epilogue: warp half = tile; TMEM -> int8 z8 -> strip / global -------
      {
        const int t = half;
        const int m = t * 128 + 32 * quarter + lane;
        if (t * 128 + 32 * quarter < 11 * 19) {            // warp has rows inside the grid
          uint32_t r[16];
          tmem_ld16(tmem + lane_base + t * 16, r);
          tmem_ld_wait();
          const int oh = m / 19, ow = m - oh * 19;
          if (oh < kH2 && ow < kW2) {
            uint32_t pk[4];
#pragma unroll
            for (int w4 = 0; w4 < 4; ++w4) {
              const float4 b4 = *reinterpret_cast<const float4*>(&s.b1[4 * w4]);
              const float4 qa4 = *reinterpret_cast<const float4*>(&s.qa[4 * w4]);
              const float4 qc4 = *reinterpret_cast<const float4*>(&s.qc[4 * w4]);
              const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
              const float aa[4] = {qa4.x, qa4.y, qa4.z, qa4.w};
              const float cc[4] = {qc4.x, qc4.y, qc4.z, qc4.w};
              uint32_t q4[4];
#pragma unroll
              for (int b = 0; b < 4; ++b)
                q4[b] = conv1_qbits(__uint_as_float(r[4 * w4 + b]), bb[b], aa[b], cc[b]);
              pk[w4] = __byte_perm(__byte_perm(q4[0], q4[1], 0x0040), __byte_perm(q4[2], q4[3], 0x0040), 0x5410);
            }
            const uint4 v = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            if (kConv2)
              *reinterpret_cast<uint4*>(s.strip + ((oh + 1) * kStripCols + ow + 1) * 16) = v;
            if (p.z8_out)
              reinterpret_cast<uint4*>(p.z8_out)[env * kTok + oh * kW2 + ow] = v;
          }
        }
      }
      tc_fence_before();
    } else {
      // kModeConv2: z8 rows of this environment -> strip
      for (int t = tid; t < kTok; t += NT) {
        const int oh = t / kW2, ow = t - oh * kW2;
        const uint32_t b = (uint32_t)t * 16;
        const uint8_t* src = (b >= rs.body_lo && b + 16 <= rs.body_hi) ? rs.stage + b : rs.src + b;
        *reinterpret_cast<uint4*>(s.strip + ((oh + 1) * kStripCols + ow + 1) * 16) =
            *reinterpret_cast<const uint4*>(src);
      }
      __syncthreads();
      if (nxt < p.B) row_issue(row_stage(p.in, nxt, p.ld, esz, row_elems, s.stage), tid, NT);
      cp_async_commit();
    }

    if (kConv2) {
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint32_t sb = smem_u32(s.strip), wb = smem_u32(s.w2s);
        constexpr uint32_t idesc = idesc_i8(128, 64);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int pr = 0; pr < 5; ++pr) {
            const int o0 = conv2_tap_off(2 * pr), o1 = conv2_tap_off(2 * pr + 1);
            const uint64_t ad = smem_desc(sb + (t * 128 + o0) * 16, (o1 - o0) * 16, 128);
            const uint64_t bd = smem_desc(wb + pr * 2048, 1024, 128);
            mma_i8(tmem + t * 64, ad, bd, idesc, pr > 0 ? 1u : 0u);
          }
        }
        mma_commit(&s.mbar);
      }
      const bool ok = mbar_wait_bounded(&s.mbar, phase);
      phase ^= 1;
      if (!ok) s.abort_flag = 1;
      tc_fence_after();
      __syncthreads();
      if (s.abort_flag) break;

      // ---- conv2 epilogue, pass 1: thread = (row, 32-channel half) -------------------
      uint32_t loc[2][16];                 // fp16 local features, packed in pairs
      const int c0 = 32 * half;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = 32 * quarter + lane;
        const int m = t * 128 + i;
        const int oh = m / kStripCols, ow = m - oh * kStripCols;
        const bool valid = oh < kH2 && ow < kW2;
        const int tok = oh * kW2 + ow;
        if (t * 128 + 32 * quarter < 11 * kStripCols) {   // warp has rows inside the grid
          float l0 = 0.0f, l1 = 0.0f;
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            uint32_t r[16];
            tmem_ld16(tmem + lane_base + t * 64 + c0 + 16 * hb, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              const int c = c0 + 16 * hb + j;
              // per-channel constants, four channels per 16-byte shared load
              const float4 dq4 = *reinterpret_cast<const float4*>(&s.dq[c]);
              const float4 b24 = *reinterpret_cast<const float4*>(&s.b2[c]);
              const float4 a24 = *reinterpret_cast<const float4*>(&s.a2[c]);
              const float4 c24 = *reinterpret_cast<const float4*>(&s.c2[c]);
              const float y0 = conv2_val((int32_t)r[j], dq4.x, b24.x, a24.x, c24.x);
              const float y1 = conv2_val((int32_t)r[j + 1], dq4.y, b24.y, a24.y, c24.y);
              const float y2 = conv2_val((int32_t)r[j + 2], dq4.z, b24.z, a24.z, c24.z);
              const float y3 = conv2_val((int32_t)r[j + 3], dq4.w, b24.w, a24.w, c24.w);
              __half2 h01 = __floats2half2_rn(y0, y1), h23 = __floats2half2_rn(y2, y3);
              loc[t][8 * hb + (j >> 1)] = *reinterpret_cast<uint32_t*>(&h01);
              loc[t][8 * hb + (j >> 1) + 1] = *reinterpret_cast<uint32_t*>(&h23);
              if (kFront) {
                const float4 wg4 = *reinterpret_cast<const float4*>(&s.wg[c]);
                const float4 ws4 = *reinterpret_cast<const float4*>(&s.ws[c]);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                l0 = fmaf(f01.x, wg4.x, l0);
                l0 = fmaf(f01.y, wg4.y, l0);
                l0 = fmaf(f23.x, wg4.z, l0);
                l0 = fmaf(f23.y, wg4.w, l0);
                l1 = fmaf(f01.x, ws4.x, l1);
                l1 = fmaf(f01.y, ws4.y, l1);
                l1 = fmaf(f23.x, ws4.z, l1);
                l1 = fmaf(f23.y, ws4.w, l1);
              }
            }
            if (valid && p.acc_out) {
              int4* dst = reinterpret_cast<int4*>(p.acc_out + (env * kTok + tok) * kD + c0 + 16 * hb);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
                dst[q4] = make_int4((int)r[4 * q4], (int)r[4 * q4 + 1], (int)r[4 * q4 + 2], (int)r[4 * q4 + 3]);
            }
          }
          if (kFront) s.lpart[t][half][i] = make_float2(l0, l1);
          if (valid && p.feat_out) {
            uint4* dst = reinterpret_cast<uint4*>(p.feat_out + (env * kTok + tok) * kD + c0);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
              dst[q4] = make_uint4(loc[t][4 * q4], loc[t][4 * q4 + 1], loc[t][4 * q4 + 2], loc[t][4 * q4 + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) loc[t][j] = 0;
        }
      }
      tc_fence_before();

      if (kFront) {
        __syncthreads();
        // ---- logits (fp16, qrt/encoder_opt.py:69-73) and softmax over 187 tokens --------
        // warps 0-3: tile 0 rows, warps 4-7: tile 1 rows
        float my_logit;
        {
          const int t = half, i = 32 * quarter + lane;
          const int m = t * 128 + i;
          const int oh = m / kStripCols, ow = m - oh * kStripCols;
          const bool valid = oh < kH2 && ow < kW2;
          float g = -INFINITY;
          if (valid) {
            const float2 a = s.lpart[t][0][i], b = s.lpart[t][1][i];
            g = fp16r(__fadd_rn(fp16r(a.x + b.x), gb));
            p.score_local[env * kTok + oh * kW2 + ow] = __float2half_rn(a.y + b.y);
          }
          my_logit = g;
        }
        float mx = warp_max(my_logit);
        if (lane == 0) s.wmax[warp] = mx;
        __syncthreads();
        mx = s.wmax[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s.wmax[w]);
        const float e = my_logit == -INFINITY ? 0.0f : expf(my_logit - mx);
        float sm = warp_sum(e);
        if (lane == 0) s.wsum[warp] = sm;
        __syncthreads();
        sm = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sm += s.wsum[w];
        {
          const int t = half, i = 32 * quarter + lane;
          const int m = t * 128 + i;
          const int oh = m / kStripCols, ow = m - oh * kStripCols;
          const bool valid = oh < kH2 && ow < kW2;
          const __half wh = __float2half_rn(__fdiv_rn(e, sm));
          s.wt16[t][i] = valid ? wh : __float2half(0.0f);
          if (valid && p.gc_w_out) p.gc_w_out[env * kTok + oh * kW2 + ow] = wh;
        }
        __syncthreads();
        // ---- pass 2: gc = sum_i w_i * local_i over this thread's 32 channels ------------
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (t * 128 + 32 * quarter < 11 * kStripCols) {
            const float wt = __half2float(s.wt16[t][32 * quarter + lane]);
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              float v[16];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&loc[t][8 * hb + j]));
                v[2 * j] = wt * f.x;
                v[2 * j + 1] = wt * f.y;
              }
              const float r = warp_reduce16(v, lane);     // lanes L and L^16 hold channel L&15
              if (lane < 16) s.pool[t][quarter][c0 + 16 * hb + lane] = r;
            }
          } else {
            s.pool[t][quarter][c0 + lane] = 0.0f;
          }
        }
        __syncthreads();
        if (tid < kD) {
          float g = 0.0f;
#pragma unroll
          for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int q = 0; q < 4; ++q) g += s.pool[t][q][tid];
          const __half gh = __float2half_rn(g);
          s.gc16[tid] = gh;
          p.enc[env * p.ld_enc + 64 + tid] = gh;
          p.pe_out[env * kD + tid] = s.pe16[tid];
        }
        for (int k = tid; k < P; k += NT) p.enc[env * p.ld_enc + 128 + k] = s.prop16[k];
        __syncthreads();
        if (p.act_mode == GLAD_ACT_DYNAMIC && tid < 2 * kD) {
          // |alpha*cat(gc, pe) + beta| for the query projector's dynamic s_z
          const float x = __half2float(tid < kD ? s.gc16[tid] : s.pe16[tid - kD]);
          zmax_qp = fmaxf(zmax_qp, aq_qp.absz(x, s.qp_a[tid], s.qp_b[tid]));
        }
      }
    }
  }

  // ---- teardown --------------------------------------------------------------------------
  cp_async_wait_all();
  if (s.abort_flag) {
    // give an MMA still in flight one more bounded wait before TMEM is released
    mbar_wait_bounded(&s.mbar, phase);
  }
  if (kFront && p.act_mode == GLAD_ACT_DYNAMIC) {
    const float m = warp_max(zmax_qp);
    if (lane == 0 && m > 0.0f) atomic_max_nonneg(&p.slots[1], m);
  }
  if (s.abort_flag && tid == 0 && p.slots)
    atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrMmaTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================================================
// Fused encoder front, software-pipelined across environments.
//
// Per iteration (environment e, planes buffer b = e & 1):
//   wait conv1(e) -> conv1 epilogue -> issue conv2(e)
//   stage -> planes[b^1] for e+1, prefetch e+2, issue conv1(e+1), proprio emb(e+1)
//   wait conv2(e) -> logits, softmax, pooled gc, outputs of e
// so the tensor core works on one environment while the CUDA cores convert
// the next or finish the previous. conv1 accumulators live in TMEM columns
// [128,160), conv2's in [0,128). All MMA descriptors are built once.
// ============================================================================================
constexpr int kFusedTmemCols = 256;
// Warps 6 and 7 issue the conv MMAs (tile t by warp 6 + t, each from one elected lane):
// a warp's MMA issue takes ~140 cycles, so two issuers halve the chain.
constexpr int kIssuerWarp0 = 6;
constexpr int kConverters = 6 * 32;      // warps 0-5 stage observation rows (all warps convert them)

struct __align__(128) FusedSmem {
  uint8_t planes[1][kPlanesBytes];     // conv1(e) completes before the conversion of e+1 writes it
  uint8_t w1s[kW1sBytes];
  uint8_t strip[kStripBytes];
  uint8_t w2s[kW2sBytes];
  uint8_t stage[kStageBytes];
  alignas(16) float b1[16];
  alignas(16) float qa[16];
  alignas(16) float qc[16];
  alignas(16) float dq[64];
  alignas(16) float b2[64];
  alignas(16) float a2[64];
  alignas(16) float c2[64];
  // fp16 local features of one environment [tile][8-channel chunk][128 rows][16 B]:
  // A operand (K-major) of the logits GEMM and (M-major) of the pooling GEMM
  alignas(128) uint8_t local16[2 * 8 * 128 * 16];
  alignas(128) uint8_t blog[8 * 16 * 16];     // logits B: [chunk][n: gps, scorer, 0...][16 B]
  alignas(128) uint8_t bpool[16 * 16 * 16];   // pooling B: [8-row chunk][n: tile 0, tile 1, 0...][16 B]
  float poolv[128];                           // pooled partial sums, row = tile*64 + channel
  float wmax[8], wsum[8];
  __half prop16[2][128];
  __half pe16[2][64];
  __half gc16[64];
  alignas(16) int8_t q8[128];
  alignas(16) uint8_t pe_w[64 * kMaxProp * 2];
  float pe_a[kMaxProp], pe_b[kMaxProp];
  float pe_scale[64], pe_bp[64];
  float qp_a[128], qp_b[128];
  uint64_t c1_adesc[2][16];            // [planes buffer][tile*8 + K-step]
  uint64_t c1_bdesc[8];
  uint64_t c2_adesc[10];               // [tile*5 + K-step]
  uint64_t c2_bdesc[5];
  uint64_t lg_adesc[2][4];             // logits GEMM [tile][K-step]
  uint64_t lg_bdesc[4];
  uint64_t pl_adesc[8];                // pooling GEMM [K-step]
  uint64_t pl_bdesc[8];
  uint64_t bar1, bar2, bar3;           // conv1 (2 issuers) / conv2 (warp 7) / logits and pooling (2 issuers)
  uint64_t bar_pe;                     // batched proprio embedding
  uint64_t bar_row;                    // bulk copy of the next observation row
  uint32_t tmem_base;
  int abort_flag;
  // fused actor + critic only (launches without it allocate up to `pec_w`): the critic
  // group's proprio and its fp16 embedding
  alignas(128) uint8_t pec_w[64 * kMaxProp * 2];
  float pec_bp[64];
  __half prop16c[2][128];
  __half pe16c[2][64];
  alignas(16) uint8_t stage_c[kMaxProp * 4 + 32];
};
// dynamic shared memory of a launch (+128 for the in-kernel alignment)
constexpr size_t kFusedSmemSingle = offsetof(FusedSmem, pec_w) + 128;
constexpr size_t kFusedSmemDual = sizeof(FusedSmem) + 128;

// FULL = false: the QuantCNN chain alone (x_nhwc -> z8 -> fp16 local features), the same
// pipeline without the pooling / embedding stages.
// DUAL (with FULL): also the critic head's proprio embedding and encoded row.
// NORM (with FULL, not DUAL): the observation normaliser runs in the row loads.
template <bool FULL, bool DUAL, bool NORM = false>
__global__ void __launch_bounds__(kFrontThreads, FRONT_MIN_BLOCKS)
front_fused_kernel(const __grid_constant__ FrontParams p) {
  extern __shared__ uint8_t smem_raw[];
  FusedSmem& s = *reinterpret_cast<FusedSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  constexpr int NT = kFrontThreads;
  grid_dep_launch();

  // ---- one-time set-up: every global read is issued before the first wait -----------------
  if (warp == 0) tmem_alloc(&s.tmem_base, kFusedTmemCols);
  if (tid == 0) {
    mbar_init(&s.bar1, 2);
    mbar_init(&s.bar2, 1);
    mbar_init(&s.bar3, 2);
    mbar_init(&s.bar_pe, 1);
    mbar_init(&s.bar_row, 1);
    fence_mbar_init();
    s.abort_flag = 0;
  }
  const int P = p.prop_dim;
  const int esz = p.in_dtype == GLAD_DTYPE_F32 ? 4 : 2;
  const int row_elems = P + kMap;
  const bool dyn = p.act_mode == GLAD_ACT_DYNAMIC;
  constexpr bool dual = FULL && DUAL;
  // int8 proprio embedding: one batched GEMM over all of this CTA's environments
  // before the loop (fp16 embeddings keep the per-environment path)
  const bool pe_batch = FULL && !p.pe_f16;
  const int Pc = dual ? p.prop_dim_c : 0;
  // raw conv weights -> scratch (the local-feature tile is unused until the loop)
  uint8_t* scratch = s.local16;
  #pragma unroll 1
  for (int i = tid; i < 3 * 64 * 64 / 16; i += NT)
    cp_async16(scratch + 16 * i, reinterpret_cast<const uint4*>(p.conv.w8) + i);
  #pragma unroll 1
  for (int i = tid; i < 128 * 16 * 2 / 16; i += NT)
    cp_async16(scratch + 12288 + 16 * i, reinterpret_cast<const uint4*>(p.conv.w1p) + i);
  #pragma unroll 1
  for (int i = tid; i < 16; i += NT) {
    cp_async4(&s.b1[i], p.conv.b1f + i);
    cp_async4(&s.qa[i], p.conv.qa + i);
    cp_async4(&s.qc[i], p.conv.qc + i);
  }
  #pragma unroll 1
  for (int i = tid; i < 64; i += NT) {
    cp_async4(&s.dq[i], p.conv.dq + i);
    cp_async4(&s.b2[i], p.conv.b2f + i);
    cp_async4(&s.a2[i], p.conv.a2 + i);
    cp_async4(&s.c2[i], p.conv.c2 + i);
  }
  // proprio embedding weights and constants
  bool pe_w_async = false;
  if (!FULL) {
  } else if (p.pe_f16) {
    pe_w_async = (kD * P) % 8 == 0 && (reinterpret_cast<uintptr_t>(p.pe16_w) & 15) == 0;
    if (pe_w_async)
      #pragma unroll 1
      for (int i = tid; i < kD * P / 8; i += NT)
        cp_async16(s.pe_w + 16 * i, reinterpret_cast<const uint4*>(p.pe16_w) + i);
  } else {
    // int8 embedding weights as the B operand of the batched GEMM: [16-byte K chunk]
    // [64 n][16 B], K zero-padded to a multiple of 32 (P % 4 == 0, w8 16-byte aligned)
    const int KC = ((P + 31) >> 5) * 2;
    #pragma unroll 1
    for (int idx = tid; idx < KC * kD * 4; idx += NT) {
      const int c = idx / (kD * 4), n = (idx >> 2) % kD, t4 = idx & 3;
      const int k = c * 16 + 4 * t4;
      uint8_t* dst = s.pe_w + c * 1024 + n * 16 + 4 * t4;
      if (k < P) cp_async4(dst, p.pe.w8 + (size_t)n * P + k);
      else *reinterpret_cast<uint32_t*>(dst) = 0u;
    }
    #pragma unroll 1
    for (int k = tid; k < P; k += NT) {
      if (p.pe.alpha) {
        cp_async4(&s.pe_a[k], p.pe.alpha + k);
        cp_async4(&s.pe_b[k], p.pe.beta + k);
      } else {
        s.pe_a[k] = 0.0f;
        s.pe_b[k] = 0.0f;
      }
    }
    #pragma unroll 1
    for (int i = tid; i < kD; i += NT) {
      cp_async4(&s.pe_scale[i], (dyn ? p.pe.s_w : p.pe.dq_scale) + i);   // raw; scaled below
      cp_async4(&s.pe_bp[i], p.pe.b_prime + i);
    }
  }
  #pragma unroll 1
  for (int k = tid; k < 128; k += NT) {
    if (FULL && p.qp.alpha) {
      cp_async4(&s.qp_a[k], p.qp.alpha + k);
      cp_async4(&s.qp_b[k], p.qp.beta + k);
    } else {
      s.qp_a[k] = 0.0f;
      s.qp_b[k] = 0.0f;
    }
  }
  bool pec_w_async = false;
  if (dual) {
    pec_w_async = (kD * Pc) % 8 == 0 && (reinterpret_cast<uintptr_t>(p.pec_w) & 15) == 0;
    if (pec_w_async)
      #pragma unroll 1
      for (int i = tid; i < kD * Pc / 8; i += NT)
        cp_async16(s.pec_w + 16 * i, reinterpret_cast<const uint4*>(p.pec_w) + i);
  }
  // the first environment's observation row (and the critic group's proprio columns)
  int64_t env = blockIdx.x;
  if (env < p.B) row_issue(row_stage(p.in, env, p.ld, esz, row_elems, s.stage), tid, NT);
  if (dual && env < p.B) row_issue(row_stage(p.in_c, env, p.ld_c, esz, Pc, s.stage_c), tid, NT);
  cp_async_commit();
  // dynamic int8 proprio embedding: this CTA's part of the batch absmax of
  // |alpha*fp16(x) + beta| over the proprio columns (qrt/qlinear.py:124-128)
  const bool grid_absmax = FULL && dyn && !p.pe_f16 && p.pe_absmax;
  if (grid_absmax) {
    // warp w takes this CTA's environments w, w+8, ...; lanes walk the proprio columns
    float m = 0.0f;
    for (int64_t row = (int64_t)blockIdx.x + (int64_t)warp * gridDim.x; row < p.B;
         row += (int64_t)8 * gridDim.x) {
#pragma unroll 4
      for (int k = lane; k < P; k += 32) {
        float x = esz == 4 ? reinterpret_cast<const float*>(p.in)[row * p.ld + k]
                           : __half2float(reinterpret_cast<const __half*>(p.in)[row * p.ld + k]);
        if constexpr (NORM) x = obs_norm(x, p.norm_mean, p.norm_var, p.norm_eps, k);
        const float xr = fp16r(x);
        m = fmaxf(m, p.pe.alpha ? fabsf(__fadd_rn(__fmul_rn(xr, p.pe.alpha[k]), p.pe.beta[k])) : fabsf(xr));
      }
    }
    m = warp_max(m);
    if (lane == 0) s.wmax[warp] = m;
  }
  // small fp16 vectors through registers: logits operand rows, biases
  __half lgw = __float2half(0.0f);
  if (FULL && tid < 2 * kD) lgw = tid < kD ? p.gps_w[tid] : p.scorer_w[tid - kD];
  const float gb = FULL ? __half2float(p.gps_b[0]) : 0.0f;
  float pe16b = 0.0f;
  if (FULL && p.pe_f16 && tid < kD && p.pe16_b) pe16b = __half2float(p.pe16_b[tid]);
  {
    const uint4 z = make_uint4(0, 0, 0, 0);
    #pragma unroll 1
    for (int i = tid; i < kPlanesBytes / 16; i += NT) reinterpret_cast<uint4*>(&s.planes[0][0])[i] = z;
    #pragma unroll 1
    for (int i = tid; i < kStripBytes / 16; i += NT) reinterpret_cast<uint4*>(s.strip)[i] = z;
    #pragma unroll 1
    for (int i = tid; i < 16 * 16 * 16 / 16; i += NT) reinterpret_cast<uint4*>(s.bpool)[i] = z;
    #pragma unroll 1
    for (int i = tid; i < 8 * 16 * 16 / 16; i += NT) reinterpret_cast<uint4*>(s.blog)[i] = z;
  }
  grid_dep_wait();                      // slots written by the preceding kernel are visible from here
  ActQuant aq_pe{};
  ActQuant aq_qp{};
  if (FULL && !p.pe_f16 && !grid_absmax) aq_pe = make_act_quant(p.pe, p.act_mode, p.slots, 0);
  aq_qp.let = FULL && p.qp.alpha != nullptr;
  cp_async_wait_all();
  __syncthreads();
  if (grid_absmax && tid == 0) {
    // publish this CTA's maximum and arrive; the wait comes just before the first use
    float m = s.wmax[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, s.wmax[w]);
    if (m > 0.0f) atomic_max_nonneg(&p.slots[0], m);
    red_release_add(reinterpret_cast<uint32_t*>(&p.slots[kSlotFrontBarrier]), 1u);
  }

  // ---- derived operands ------------------------------------------------------------------
  {
    const __half* w1p = reinterpret_cast<const __half*>(scratch + 12288);
    __half* dst = reinterpret_cast<__half*>(s.w1s);
    #pragma unroll 1
    for (int idx = tid; idx < kW1sBytes / 2; idx += NT) {
      const int pr = idx >> 8, c = (idx >> 7) & 1, n = (idx >> 3) & 15, e = idx & 7;
      const int q = 2 * pr + c;
      __half v = __float2half(0.0f);
      if (q < 15) {
        const int kh = q / 3, kw = 2 * (q % 3) + (e >> 2), ch = e & 3;
        if (kw < 5 && ch < 3) v = w1p[(kh * 16 + kw * 3 + ch) * 16 + n];
      }
      dst[idx] = v;
    }
    conv2_b_relayout(s.w2s, scratch, tid, NT);
    // logits B operand: row 0 = global_pool_selector weight, row 1 = scorer weight (local half)
    if (tid < 2 * kD) {
      const int n = tid >> 6, c = (tid & 63) >> 3, e = tid & 7;
      reinterpret_cast<__half*>(s.blog)[(c * 16 + n) * 8 + e] = lgw;
    }
    if (dual) {
      if (!pec_w_async) {
        __half* dw = reinterpret_cast<__half*>(s.pec_w);
        #pragma unroll 1
        for (int i = tid; i < kD * Pc; i += NT) dw[i] = p.pec_w[i];
      }
      if (tid < kD) s.pec_bp[tid] = p.pec_b ? __half2float(p.pec_b[tid]) : 0.0f;
    }
    if (!FULL) {
    } else if (p.pe_f16) {
      if (!pe_w_async) {
        __half* dw = reinterpret_cast<__half*>(s.pe_w);
        #pragma unroll 1
        for (int i = tid; i < kD * P; i += NT) dw[i] = p.pe16_w[i];
      }
      if (tid < kD) s.pe_bp[tid] = pe16b;
    } else {
      if (dyn && !grid_absmax && tid < kD) s.pe_scale[tid] = __fmul_rn(s.pe_scale[tid], aq_pe.s);   // s_w * s_z
    }
    // every MMA descriptor of the loop, one per thread
    const uint32_t lb = smem_u32(s.local16);
    if (tid < 32) {
      const int bb = tid >> 4, t = (tid >> 3) & 1, pr = tid & 7;
      const uint32_t c0 = conv1_chunk_off(2 * pr), c1 = conv1_chunk_off(2 * pr + 1);
      s.c1_adesc[bb][t * 8 + pr] = smem_desc(smem_u32(s.planes[0]) + c0 + t * 128 * 16, c1 - c0, 128);
    } else if (tid < 40) {
      const int pr = tid - 32;
      s.c1_bdesc[pr] = smem_desc(smem_u32(s.w1s) + pr * 512, 256, 128);
    } else if (tid < 50) {
      const int t = (tid - 40) / 5, pr = (tid - 40) % 5;
      const int o0 = conv2_tap_off(2 * pr), o1 = conv2_tap_off(2 * pr + 1);
      s.c2_adesc[t * 5 + pr] = smem_desc(smem_u32(s.strip) + (t * 128 + o0) * 16, (o1 - o0) * 16, 128);
    } else if (tid < 55) {
      const int pr = tid - 50;
      s.c2_bdesc[pr] = smem_desc(smem_u32(s.w2s) + pr * 2048, 1024, 128);
    } else if (tid < 63) {
      // logits: A = local16 tile t, K-major (chunk stride 2048 B, 8-row groups 128 B)
      const int t = (tid - 55) >> 2, kk = (tid - 55) & 3;
      s.lg_adesc[t][kk] = smem_desc(lb + t * 16384 + kk * 2 * 2048, 2048, 128);
    } else if (tid < 67) {
      const int kk = tid - 63;
      s.lg_bdesc[kk] = smem_desc(smem_u32(s.blog) + kk * 2 * 256, 256, 128);
    } else if (tid < 75) {
      // pooling: A = local16 read M-major (M = tile*64 + channel: 8-channel blocks 2048 B
      // apart, K = row: 8-row blocks 128 B apart), B = softmax weights, K-major
      const int kk = tid - 67;
      s.pl_adesc[kk] = smem_desc(lb + kk * 256, 128, 2048);
    } else if (tid < 83) {
      const int kk = tid - 75;
      s.pl_bdesc[kk] = smem_desc(smem_u32(s.bpool) + kk * 2 * 256, 256, 128);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t tmem_c1 = tmem + 128;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
  uint32_t ph1 = 0, ph2 = 0, ph3 = 0, ph_pe = 0;
  uint32_t ph_row = 0;                  // next phase of bar_row the converters consume
  bool row_pending = false;             // a bulk row copy is in flight (converters)
  float zmax_qp = 0.0f;
  float zmax_qpc = 0.0f;                // critic query projector input (dual)

  // observation normaliser of column k (identity without one)
  auto nz = [&](float x, int k) {
    if constexpr (NORM) return obs_norm(x, p.norm_mean, p.norm_var, p.norm_eps, k);
    return x;
  };
  // convert the staged row of `e` into planes[b] / prop16[b]
  auto convert = [&](int64_t e, int b, int nthr) {
    if (dual) {
      const RowStage rc = row_stage(p.in_c, e, p.ld_c, esz, Pc, s.stage_c);
      for (int k = tid; k < Pc; k += nthr)
        s.prop16c[b][k] = __float2half_rn(esz == 4 ? row_elem<4>(rc, k) : row_elem<2>(rc, k));
    }
    const RowStage rs = row_stage(p.in, e, p.ld, esz, row_elems, s.stage);
    if (esz == 4 && rs.lo == 0 && rs.hi == (uint32_t)row_elems * 4) {
      // the whole fp32 row is in shared memory
      const float* st = reinterpret_cast<const float*>(s.stage + (rs.stage - s.stage));
      auto put = [&](int px, float v0, float v1, float v2) {
        const int ih = px / kW1, iw = px - ih * kW1;
        const int pl = ih & 1, r = ((ih - pl) >> 1) + 1, slot = iw + 2;
        const __half2 h01 = __floats2half2_rn(v0, v1);
        const __half2 h2z = __floats2half2_rn(v2, 0.0f);
        *reinterpret_cast<uint2*>(s.planes[0] + pl * kPlaneBytes + r * kRowBytes + slot * 8) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h2z));
      };
      if constexpr (NORM) {
        for (int px = tid; px < kH1 * kW1; px += nthr) {
          const int c0 = P + px * 3;
          put(px, nz(st[c0], c0), nz(st[c0 + 1], c0 + 1), nz(st[c0 + 2], c0 + 2));
        }
        if (!pe_batch)
          for (int k = tid; k < P; k += nthr) s.prop16[b][k] = __float2half_rn(nz(st[k], k));
      } else {
        for (int px = tid; px < kH1 * kW1; px += nthr)
          put(px, st[P + px * 3], st[P + px * 3 + 1], st[P + px * 3 + 2]);
        if (!pe_batch)
          for (int k = tid; k < P; k += nthr) s.prop16[b][k] = __float2half_rn(st[k]);
      }
      return;
    }
    for (int px = tid; px < kH1 * kW1; px += nthr) {
      const int ih = px / kW1, iw = px - ih * kW1;
      float v0, v1, v2;
      if (esz == 4) {
        const int c0 = P + px * 3;
        v0 = nz(row_elem<4>(rs, c0), c0);
        v1 = nz(row_elem<4>(rs, c0 + 1), c0 + 1);
        v2 = nz(row_elem<4>(rs, c0 + 2), c0 + 2);
      } else {
        v0 = row_elem<2>(rs, P + px * 3);
        v1 = row_elem<2>(rs, P + px * 3 + 1);
        v2 = row_elem<2>(rs, P + px * 3 + 2);
      }
      const int pl = ih & 1, r = ((ih - pl) >> 1) + 1, slot = iw + 2;
      __half2 h01 = __floats2half2_rn(v0, v1);
      __half2 h2z = __floats2half2_rn(v2, 0.0f);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&h01);
      pk.y = *reinterpret_cast<uint32_t*>(&h2z);
      *reinterpret_cast<uint2*>(s.planes[0] + pl * kPlaneBytes + r * kRowBytes + slot * 8) = pk;
    }
    if (!pe_batch)
      for (int k = tid; k < P; k += nthr)
        s.prop16[b][k] = __float2half_rn(esz == 4 ? nz(row_elem<4>(rs, k), k) : row_elem<2>(rs, k));
  };
  auto issue_conv1 = [&](int b) {      // tile t by warp 6 + t (one elected lane each)
    if (warp >= kIssuerWarp0) {
      const int t = warp - kIssuerWarp0;
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16(128, 16);
#pragma unroll
      for (int pr = 0; pr < 8; ++pr)
        mma_f16_warp(tmem_c1 + t * 16, s.c1_adesc[b][t * 8 + pr], s.c1_bdesc[pr], idesc, pr > 0 ? 1u : 0u);
      mma_commit_warp(&s.bar1);
    }
  };
  // critic proprio embedding (fp16 nn.Linear) of buffer b on threads 128-255
  auto critic_emb = [&](int b) {
    if (tid >= 2 * kD) {
      const int t = tid - 2 * kD, n = t >> 1, part = t & 1;
      const __half* wrow = reinterpret_cast<const __half*>(s.pec_w) + n * Pc;
      const int half_k = (Pc + 1) >> 1;
      const int k0 = part * half_k, k1 = min(Pc, k0 + half_k);
      float a = 0.0f;
      for (int k = k0; k < k1; ++k) a = fmaf(__half2float(s.prop16c[b][k]), __half2float(wrow[k]), a);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      if (part == 0) s.pe16c[b][n] = __float2half_rn(a + s.pec_bp[n]);
    }
  };
  // fp16 proprio embedding (nn.Linear) of the environment in buffer b (threads 0-127)
  auto proprio_emb = [&](int b) {
    if (tid < 2 * kD) {
      const int n = tid >> 1, part = tid & 1;
      const __half* wrow = reinterpret_cast<const __half*>(s.pe_w) + n * P;
      const int half_k = (P + 1) >> 1;
      const int k0 = part * half_k, k1 = min(P, k0 + half_k);
      float a = 0.0f;
      for (int k = k0; k < k1; ++k) a = fmaf(__half2float(s.prop16[b][k]), __half2float(wrow[k]), a);
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      if (part == 0) s.pe16[b][n] = __float2half_rn(a + s.pe_bp[n]);
    }
  };
  // int8 proprio embedding of ALL of this CTA's environments (qrt/qlinear.py:111-138),
  // in batches of 128: the quantised rows [env][k] form the A operand (K-major, the
  // local-feature tile is free until the loop), w8 the B operand, the int32 products
  // land in TMEM columns [160, 224) and the row's thread dequantises them into pe_out.
  // The same pass writes each row's fp16 proprio into `enc` and folds the embedding
  // into the query projector's absmax.
  // the 4 proprio values of item `item` (row item / (4 KC), columns 4 * (item % (4 KC))
  // + 0..3) of the batch starting at local row j0
  const int pe_kc = ((P + 31) >> 5) * 2;
  const int pe_q = pe_kc * 4;
  const int64_t pe_nloc = blockIdx.x < p.B ? (p.B - 1 - (int64_t)blockIdx.x) / gridDim.x + 1 : 0;
  auto pe_load = [&](int item, int64_t j0) -> float4 {
    const int r = item / pe_q, k0 = 4 * (item - r * pe_q);
    const int64_t e = (int64_t)blockIdx.x + (j0 + r) * gridDim.x;
    auto ld = [&](int k) {
      if (k >= P) return 0.0f;
      return esz == 4 ? reinterpret_cast<const float*>(p.in)[e * p.ld + k]
                      : __half2float(reinterpret_cast<const __half*>(p.in)[e * p.ld + k]);
    };
    return make_float4(ld(k0), ld(k0 + 1), ld(k0 + 2), ld(k0 + 3));
  };
  // int8 proprio embedding of ALL of this CTA's environments (qrt/qlinear.py:111-138),
  // in batches of 128: the quantised rows [env][k] form the A operand (K-major, the
  // local-feature tile is free until the loop), w8 the B operand, the int32 products
  // land in TMEM columns [160, 224); the rows' threads dequantise them into pe_out and
  // an fp16 copy from which every thread folds the embedding into the query
  // projector's absmax. The same pass writes each row's fp16 proprio into `enc`.
  // `pre` holds item `tid` of the first batch, loaded before the absmax barrier.
  auto pe_batched = [&](float4 pre) {
    uint8_t* A = s.local16;                                   // [chunk][128 rows][16 B]
    __half* pes = reinterpret_cast<__half*>(s.local16 + 16384);   // [row][64] fp16
    for (int64_t j0 = 0; j0 < pe_nloc; j0 += 128) {
      const int nb = (int)(pe_nloc - j0 < 128 ? pe_nloc - j0 : 128);
      // rows past nb keep whatever bytes the tile holds (their products are never read)
      for (int item = tid; item < nb * pe_q; item += NT) {
        const int r = item / pe_q, k0 = 4 * (item - r * pe_q);
        const int64_t e = (int64_t)blockIdx.x + (j0 + r) * gridDim.x;
        const float4 x = (j0 == 0 && item == tid) ? pre : pe_load(item, j0);
        auto cv = [&](float v, int k) { return __float2half_rn(esz == 4 ? nz(v, k) : v); };
        const __half h0 = cv(x.x, k0), h1 = cv(x.y, k0 + 1), h2 = cv(x.z, k0 + 2), h3 = cv(x.w, k0 + 3);
        auto qz = [&](__half h, int k) {
          return k < P ? ((uint32_t)aq_pe.quant(__half2float(h), s.pe_a[k], s.pe_b[k]) & 0xFFu) : 0u;
        };
        const uint32_t w = qz(h0, k0) | (qz(h1, k0 + 1) << 8) | (qz(h2, k0 + 2) << 16) | (qz(h3, k0 + 3) << 24);
        *reinterpret_cast<uint32_t*>(A + (k0 >> 4) * 2048 + r * 16 + (k0 & 15)) = w;
        __half* er = p.enc + e * p.ld_enc + 128 + k0;
        if (k0 + 4 <= P && (reinterpret_cast<uintptr_t>(er) & 7) == 0) {
          const __half2 a01 = __halves2half2(h0, h1), a23 = __halves2half2(h2, h3);
          *reinterpret_cast<uint2*>(er) = make_uint2(*reinterpret_cast<const uint32_t*>(&a01),
                                                     *reinterpret_cast<const uint32_t*>(&a23));
        } else {
          if (k0 < P) er[0] = h0;
          if (k0 + 1 < P) er[1] = h1;
          if (k0 + 2 < P) er[2] = h2;
          if (k0 + 3 < P) er[3] = h3;
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (warp == 7) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_i8(128, 64);
        for (int kk = 0; kk < pe_kc / 2; ++kk)
          mma_i8_warp(tmem + 160, smem_desc(smem_u32(A) + kk * 4096, 2048, 128),
                      smem_desc(smem_u32(s.pe_w) + kk * 2048, 1024, 128), idesc, kk > 0 ? 1u : 0u);
        mma_commit_warp(&s.bar_pe);
      }
      if (!mbar_wait_bounded(&s.bar_pe, ph_pe)) s.abort_flag = 1;
      ph_pe ^= 1;
      tc_fence_after();
      __syncthreads();
      if (s.abort_flag) return;
      if (32 * quarter < nb) {
        // warps w and w + 4 share TMEM lanes 32*(w & 3)..: each takes two of the four
        // 16-column chunks of its rows
        const int r = 32 * quarter + lane;
        const int64_t e = (int64_t)blockIdx.x + (j0 + r) * gridDim.x;
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          uint32_t acc[16];
          tmem_ld16(tmem + lane_base + 160 + 16 * c, acc);
          tmem_ld_wait();
          if (r < nb) {
            uint32_t hw[8];
#pragma unroll
            for (int t = 0; t < 16; t += 2) {
              const int n = 16 * c + t;
              const __half2 h2 = __halves2half2(qlinear_out((int32_t)acc[t], s.pe_scale[n], s.pe_bp[n]),
                                                qlinear_out((int32_t)acc[t + 1], s.pe_scale[n + 1], s.pe_bp[n + 1]));
              hw[t >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            const uint4 v0 = make_uint4(hw[0], hw[1], hw[2], hw[3]), v1 = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            uint4* dst = reinterpret_cast<uint4*>(p.pe_out + e * kD + 16 * c);
            dst[0] = v0;
            dst[1] = v1;
            uint4* sp = reinterpret_cast<uint4*>(pes + r * kD + 16 * c);
            sp[0] = v0;
            sp[1] = v1;
          }
        }
      }
      tc_fence_before();
      __syncthreads();
      if (dyn)
        for (int idx = tid; idx < nb * kD; idx += NT) {
          const int n = idx & (kD - 1);
          zmax_qp = fmaxf(zmax_qp, aq_qp.absz(__half2float(pes[idx]), s.qp_a[kD + n], s.qp_b[kD + n]));
        }
      __syncthreads();                  // A, pes and the TMEM columns are reused by the next batch
    }
  };

  // conv1(e) accumulators -> z8 -> conv2's strip (and z8_out); warps 0-6 own rows
  auto conv1_epi = [&](int64_t e) {
    {
      const int t = half;
      const int m = t * 128 + 32 * quarter + lane;
      if (t * 128 + 32 * quarter < 11 * 19) {
        uint32_t r[16];
        tmem_ld16(tmem_c1 + lane_base + t * 16, r);
        tmem_ld_wait();
        const int oh = m / 19, ow = m - oh * 19;
        if (oh < kH2 && ow < kW2) {
          uint32_t pk[4];
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const float4 b4 = *reinterpret_cast<const float4*>(&s.b1[4 * w4]);
            const float4 qa4 = *reinterpret_cast<const float4*>(&s.qa[4 * w4]);
            const float4 qc4 = *reinterpret_cast<const float4*>(&s.qc[4 * w4]);
            const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
            const float aa[4] = {qa4.x, qa4.y, qa4.z, qa4.w};
            const float cc[4] = {qc4.x, qc4.y, qc4.z, qc4.w};
            uint32_t q4[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              q4[k] = conv1_qbits(__uint_as_float(r[4 * w4 + k]), bb[k], aa[k], cc[k]);
            pk[w4] = __byte_perm(__byte_perm(q4[0], q4[1], 0x0040), __byte_perm(q4[2], q4[3], 0x0040), 0x5410);
          }
          const uint4 v = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(s.strip + ((oh + 1) * kStripCols + ow + 1) * 16) = v;
          if (p.z8_out) reinterpret_cast<uint4*>(p.z8_out)[e * kTok + oh * kW2 + ow] = v;   // optional for the chain
        }
      }
    }
  };
  // conv2 of the strip's environment: warp 7 (one elected lane) issues both tiles
  auto issue_conv2 = [&]() {
    if (warp == 7) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_i8(128, 64);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int pr = 0; pr < 5; ++pr)
          mma_i8_warp(tmem + t * 64, s.c2_adesc[t * 5 + pr], s.c2_bdesc[pr], idesc, pr > 0 ? 1u : 0u);
      mma_commit_warp(&s.bar2);
    }
  };
  // conv1(e) done -> strip (warps 0-6) -> conv2(e) issued by warp 7 once the strip is
  // complete (named barrier 3: 224 arrivals + warp 7); warp 7 has no conv1 rows
  auto stage_conv2 = [&](int64_t e) {
    if (warp < 7) {
      if (!mbar_wait_bounded(&s.bar1, ph1)) s.abort_flag = 1;
      tc_fence_after();
      conv1_epi(e);
      tc_fence_before();
      fence_async_smem();
      named_bar_arrive(3, NT);
    } else {
      named_bar_sync(3, NT);
      issue_conv2();
    }
    ph1 ^= 1;
  };

  // ---- prologue: first environment through conv1 issue ---------------------------------
  // In the loop, warps 0-5 stage and convert observation rows (named barrier 1) while
  // warps 6 and 7 issue the conv MMAs; only warps 0-5 own cp.async groups there.
  if (env < p.B) {
    convert(env, 0, NT);                // its row was staged with the set-up copies
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    const int64_t nx = env + gridDim.x;
    if (nx < p.B && tid < kConverters) {
      row_issue_bulk(row_stage(p.in, nx, p.ld, esz, row_elems, s.stage), &s.bar_row, tid);
      row_pending = true;
    }
    if (dual && nx < p.B && tid < kConverters)
      row_issue(row_stage(p.in_c, nx, p.ld_c, esz, Pc, s.stage_c), tid, kConverters);
    cp_async_commit();
    issue_conv1(0);
    // the first embedding batch's proprio values, in flight while the barrier is awaited
    float4 pe_pre = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (pe_batch && tid < (pe_nloc < 128 ? (int)pe_nloc : 128) * pe_q) pe_pre = pe_load(tid, 0);
    if (grid_absmax) {
      // every CTA has added its part of the proprio absmax (bounded spin, 2 s)
      if (tid == 0) {
        const uint32_t* ctr = reinterpret_cast<const uint32_t*>(&p.slots[kSlotFrontBarrier]);
        const uint64_t t0 = global_timer_ns();
        while (ld_acquire_gpu(ctr) < gridDim.x) {
          if (global_timer_ns() - t0 > 2000000000ull) {
            s.abort_flag = 1;
            atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrBarrierTimeout);
            break;
          }
        }
      }
      __syncthreads();
      aq_pe.let = p.pe.alpha != nullptr;
      aq_pe.dyn = true;
      aq_pe.s = dyn_scale(ld_relaxed_gpu(&p.slots[0]), aq_pe.let);
      aq_pe.rcp = __fdiv_rn(1.0f, aq_pe.s);
      aq_pe.inv = 0.0f;
      if (tid < kD) s.pe_scale[tid] = __fmul_rn(s.pe_scale[tid], aq_pe.s);   // s_w * s_z
      __syncthreads();
    }
    if (pe_batch) pe_batched(pe_pre);
    else if (FULL) proprio_emb(0);
    if (dual) critic_emb(0);
    stage_conv2(env);                   // conv2 of the first environment, ahead of the loop
  }

  int b = 0;
  for (; env < p.B; env += gridDim.x, b ^= 1) {
    const int64_t nxt = env + gridDim.x;
    // ---- next environment: warps 0-5 convert and prefetch it, then warps 6-7 issue its conv1
    //      (warps 0-3 compute an fp16 proprio embedding); conv2(e) is in flight ----------------
    if (nxt < p.B) {
      // all eight warps convert the staged row of e+1; then warps 6-7 issue its conv1 while
      // warps 0-5 start the copy of row e+2
      if (warp < kIssuerWarp0) {
        cp_async_wait_all();
        if (mbar_wait_bounded(&s.bar_row, ph_row)) {   // the bulk body of row e+1
          ph_row ^= 1;
          row_pending = false;
        } else {
          s.abort_flag = 1;                 // the teardown waits for it once more
        }
      }
      __syncthreads();                    // the staged row of e+1 is complete
      convert(nxt, b ^ 1, NT);
      fence_async_smem();
      tc_fence_before();
      __syncthreads();                    // planes ready; the stage buffer is free
      if (warp >= kIssuerWarp0) {
        issue_conv1(b ^ 1);
        if (dual) critic_emb(b ^ 1);
      } else {
        const int64_t nn = nxt + gridDim.x;
        if (nn < p.B) {
          row_issue_bulk(row_stage(p.in, nn, p.ld, esz, row_elems, s.stage), &s.bar_row, tid);
          row_pending = true;
        }
        if (dual && nn < p.B) row_issue(row_stage(p.in_c, nn, p.ld_c, esz, Pc, s.stage_c), tid, kConverters);
        cp_async_commit();
        if (FULL && !pe_batch) proprio_emb(b ^ 1);
        if (dual) critic_emb(b ^ 1);
      }
    }

    // ---- conv2(e) done -> local features -> logits, softmax pool ---------------------------
    if (!mbar_wait_bounded(&s.bar2, ph2)) s.abort_flag = 1;
    ph2 ^= 1;
    tc_fence_after();
    __syncthreads();
    if (s.abort_flag) break;

    // fp16 local features -> local16 (operand of the logits and pooling GEMMs). A thread
    // owns row i of both tiles and 32 channels; each channel's constants serve both tiles.
    {
      const int c0 = 32 * half;
      const int i = 32 * quarter + lane;
      const bool live1 = 128 + 32 * quarter < 11 * kStripCols;   // tile-1 rows of this warp in the grid
      const int m1 = 128 + i;
      const int oh0 = i / kStripCols, ow0 = i - oh0 * kStripCols;
      const int oh1 = m1 / kStripCols, ow1 = m1 - oh1 * kStripCols;
      const bool valid0 = oh0 < kH2 && ow0 < kW2;
      const bool valid1 = oh1 < kH2 && ow1 < kW2;
      uint8_t* lrow0 = s.local16 + i * 16;
      uint8_t* lrow1 = s.local16 + 16384 + i * 16;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t r0[16], r1[16];
        tmem_ld16(tmem + lane_base + c0 + 16 * hb, r0);
        if (live1) tmem_ld16(tmem + lane_base + 64 + c0 + 16 * hb, r1);
        tmem_ld_wait();
        uint32_t hw0[8], hw1[8];
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          const int c = c0 + 16 * hb + j;
          const float4 dq4 = *reinterpret_cast<const float4*>(&s.dq[c]);
          const float4 b24 = *reinterpret_cast<const float4*>(&s.b2[c]);
          const float4 a24 = *reinterpret_cast<const float4*>(&s.a2[c]);
          const float4 c24 = *reinterpret_cast<const float4*>(&s.c2[c]);
          {
            const __half2 h01 = __floats2half2_rn(conv2_val((int32_t)r0[j], dq4.x, b24.x, a24.x, c24.x),
                                                  conv2_val((int32_t)r0[j + 1], dq4.y, b24.y, a24.y, c24.y));
            const __half2 h23 = __floats2half2_rn(conv2_val((int32_t)r0[j + 2], dq4.z, b24.z, a24.z, c24.z),
                                                  conv2_val((int32_t)r0[j + 3], dq4.w, b24.w, a24.w, c24.w));
            hw0[j >> 1] = *reinterpret_cast<const uint32_t*>(&h01);
            hw0[(j >> 1) + 1] = *reinterpret_cast<const uint32_t*>(&h23);
          }
          if (live1) {
            const __half2 h01 = __floats2half2_rn(conv2_val((int32_t)r1[j], dq4.x, b24.x, a24.x, c24.x),
                                                  conv2_val((int32_t)r1[j + 1], dq4.y, b24.y, a24.y, c24.y));
            const __half2 h23 = __floats2half2_rn(conv2_val((int32_t)r1[j + 2], dq4.z, b24.z, a24.z, c24.z),
                                                  conv2_val((int32_t)r1[j + 3], dq4.w, b24.w, a24.w, c24.w));
            hw1[j >> 1] = *reinterpret_cast<const uint32_t*>(&h01);
            hw1[(j >> 1) + 1] = *reinterpret_cast<const uint32_t*>(&h23);
          } else {
            // rows past the grid: zero (their pooling weight is 0, the operand must be finite)
            hw1[j >> 1] = 0u;
            hw1[(j >> 1) + 1] = 0u;
          }
        }
        const int ch = (c0 + 16 * hb) >> 3;
        const uint4 v00 = make_uint4(hw0[0], hw0[1], hw0[2], hw0[3]);
        const uint4 v01 = make_uint4(hw0[4], hw0[5], hw0[6], hw0[7]);
        const uint4 v10 = make_uint4(hw1[0], hw1[1], hw1[2], hw1[3]);
        const uint4 v11 = make_uint4(hw1[4], hw1[5], hw1[6], hw1[7]);
        if (FULL) {
          *reinterpret_cast<uint4*>(lrow0 + ch * 2048) = v00;
          *reinterpret_cast<uint4*>(lrow0 + (ch + 1) * 2048) = v01;
          *reinterpret_cast<uint4*>(lrow1 + ch * 2048) = v10;
          *reinterpret_cast<uint4*>(lrow1 + (ch + 1) * 2048) = v11;
        }
        if (p.feat_out) {
          if (valid0) {
            uint4* dst = reinterpret_cast<uint4*>(p.feat_out + (env * kTok + oh0 * kW2 + ow0) * kD + c0 + 16 * hb);
            dst[0] = v00;
            dst[1] = v01;
          }
          if (valid1) {
            uint4* dst = reinterpret_cast<uint4*>(p.feat_out + (env * kTok + oh1 * kW2 + ow1) * kD + c0 + 16 * hb);
            dst[0] = v10;
            dst[1] = v11;
          }
        }
      }
    }
    if constexpr (!FULL) {
      // chain only: conv1(e+1) -> strip -> conv2(e+1) while the next row is converted
      tc_fence_before();
      __syncthreads();
      if (nxt < p.B) stage_conv2(nxt);
      continue;
    }
    tc_fence_before();
    fence_async_smem();
    __syncthreads();
    // logits of both heads for every row: [gps, scorer-local] = local @ [w_g; w_s]^T (fp32 in
    // TMEM), tile t issued by warp t
    if (warp < 2) {
      const int t = warp;
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16(128, 16);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_warp(tmem + 160 + 16 * t, s.lg_adesc[t][kk], s.lg_bdesc[kk], idesc, kk > 0 ? 1u : 0u);
      mma_commit_warp(&s.bar3);
    }
    // while the logits GEMM runs: conv1(e+1) -> strip, and warp 7 issues conv2(e+1); warp 7
    // owns no valid token rows, so the softmax and pooling below run on warps 0-6 (named
    // barrier 4) while it issues, and it rejoins at the CTA barrier before the outputs
    if (nxt < p.B) stage_conv2(nxt);
    if (warp < 7) {
      if (!mbar_wait_bounded(&s.bar3, ph3)) s.abort_flag = 1;
      tc_fence_after();
      named_bar_sync(4, 7 * 32);
      // logits (qrt/encoder_opt.py:69-73) and the softmax over the 187 tokens (:75)
      float my_logit;
      int my_tok = -1;
      {
        const int t = half, i = 32 * quarter + lane;
        const int m = t * 128 + i;
        const int oh = m / kStripCols, ow = m - oh * kStripCols;
        uint32_t l0 = 0, l1 = 0;
        if (t * 128 + 32 * quarter < 11 * kStripCols) {
          tmem_ld2(tmem + lane_base + 160 + 16 * t, l0, l1);
          tmem_ld_wait();
        }
        float g = -INFINITY;
        if (oh < kH2 && ow < kW2) {
          my_tok = oh * kW2 + ow;
          g = fp16r(__fadd_rn(fp16r(__uint_as_float(l0)), gb));
          p.score_local[env * kTok + my_tok] = __float2half_rn(__uint_as_float(l1));
        }
        my_logit = g;
      }
      tc_fence_before();
      float mx = warp_max(my_logit);
      if (lane == 0) s.wmax[warp] = mx;
      named_bar_sync(4, 7 * 32);
      mx = s.wmax[0];
#pragma unroll
      for (int w = 1; w < 7; ++w) mx = fmaxf(mx, s.wmax[w]);
      const float ex = my_tok < 0 ? 0.0f : expf(my_logit - mx);
      float sm = warp_sum(ex);
      if (lane == 0) s.wsum[warp] = sm;
      named_bar_sync(4, 7 * 32);
      sm = 0.0f;
#pragma unroll
      for (int w = 0; w < 7; ++w) sm += s.wsum[w];
      {
        const __half wh = __float2half_rn(__fdiv_rn(ex, sm));
        const int i = 32 * quarter + lane;
        // pooling B: column n = tile, K = row within the tile
        reinterpret_cast<__half*>(s.bpool + (i >> 3) * 256 + half * 16)[i & 7] =
            my_tok < 0 ? __float2half(0.0f) : wh;
        if (my_tok >= 0 && p.gc_w_out) p.gc_w_out[env * kTok + my_tok] = wh;
      }
      fence_async_smem();
      named_bar_sync(4, 7 * 32);
      // pooled global context gc = sum_i w_i local_i (qrt/encoder_opt.py:76-77): row
      // tile*64 + c of the pooling GEMM, column `tile`; warp h sums the rows 64h..64h+63 of
      // each tile into its own accumulator (TMEM columns 192 + 16h)
      if (warp < 2) {
        const int h = warp;
        tc_fence_after();
        constexpr uint32_t idesc = idesc_f16_amajor_m(128, 16);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_warp(tmem + 192 + 16 * h, s.pl_adesc[4 * h + kk], s.pl_bdesc[4 * h + kk], idesc,
                       kk > 0 ? 1u : 0u);
        mma_commit_warp(&s.bar3);
      }
      if (!mbar_wait_bounded(&s.bar3, ph3 ^ 1)) s.abort_flag = 1;
      tc_fence_after();
      named_bar_sync(4, 7 * 32);
      if (warp < 4) {
        uint32_t d0, d1, e0, e1;
        tmem_ld2(tmem + lane_base + 192, d0, d1);
        tmem_ld2(tmem + lane_base + 208, e0, e1);
        tmem_ld_wait();
        const int mrow = 32 * warp + lane;
        s.poolv[mrow] = __fadd_rn(__uint_as_float(mrow < 64 ? d0 : d1), __uint_as_float(mrow < 64 ? e0 : e1));
      }
      tc_fence_before();
    }                                   // softmax group
    // bar3 completed two phases (logits, pooling) this iteration: ph3 is unchanged
    __syncthreads();                    // warp 7 rejoins
    if (s.abort_flag) break;
    if (tid < kD) {
      const float g = s.poolv[tid] + s.poolv[64 + tid];
      const __half gh = __float2half_rn(g);
      s.gc16[tid] = gh;
      p.enc[env * p.ld_enc + 64 + tid] = gh;
      if (!pe_batch) p.pe_out[env * kD + tid] = s.pe16[b][tid];
      if (dual) {
        p.enc_c[env * p.ld_enc_c + 64 + tid] = gh;
        p.pe_c_out[env * kD + tid] = s.pe16c[b][tid];
      }
    }
    if (!pe_batch)
      for (int k = tid; k < P; k += NT) p.enc[env * p.ld_enc + 128 + k] = s.prop16[b][k];
    for (int k = tid; k < Pc; k += NT) p.enc_c[env * p.ld_enc_c + 128 + k] = s.prop16c[b][k];
    __syncthreads();
    if (p.act_mode == GLAD_ACT_DYNAMIC && tid < (pe_batch ? kD : 2 * kD)) {
      const float x = __half2float(tid < kD ? s.gc16[tid] : s.pe16[b][tid - kD]);
      zmax_qp = fmaxf(zmax_qp, aq_qp.absz(x, s.qp_a[tid], s.qp_b[tid]));
    }
    if (dual && p.act_mode == GLAD_ACT_DYNAMIC && tid >= 2 * kD) {
      // the critic's query projector input cat(gc, pe_critic)
      const int t = tid - 2 * kD;
      const float x = __half2float(t < kD ? s.gc16[t] : s.pe16c[b][t - kD]);
      zmax_qpc = fmaxf(zmax_qpc, aq_qp.absz(x, s.qp_a[t], s.qp_b[t]));
    }
  }

  // ---- teardown ----------------------------------------------------------------------------
  cp_async_wait_all();
  if (row_pending) mbar_wait_bounded(&s.bar_row, ph_row);   // an aborted loop's row copy in flight
  if (s.abort_flag) {
    mbar_wait_bounded(&s.bar1, ph1);
    mbar_wait_bounded(&s.bar2, ph2);
    mbar_wait_bounded(&s.bar3, ph3);
    mbar_wait_bounded(&s.bar_pe, ph_pe);
  }
  if (FULL && p.act_mode == GLAD_ACT_DYNAMIC) {
    // one atomic per CTA on the query projector's absmax slot
    const float m = warp_max(zmax_qp);
    __syncthreads();
    if (lane == 0) s.wmax[warp] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = s.wmax[0];
#pragma unroll
      for (int w = 1; w < 8; ++w) mm = fmaxf(mm, s.wmax[w]);
      if (mm > 0.0f) atomic_max_nonneg(&p.slots[1], mm);
    }
    if (dual) {
      const float mc = warp_max(zmax_qpc);
      __syncthreads();
      if (lane == 0) s.wmax[warp] = mc;
      __syncthreads();
      if (tid == 0) {
        float mm = s.wmax[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) mm = fmaxf(mm, s.wmax[w]);
        if (mm > 0.0f) atomic_max_nonneg(&p.slots[kSlotCriticQp], mm);
      }
    }
  }
  if (s.abort_flag && tid == 0 && p.slots)
    atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrMmaTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kFusedTmemCols);
  }
}

size_t front_smem_bytes() { return sizeof(FrontSmem) + 128; }

// Resident CTAs of the fused front kernel per SM (its in-kernel grid barrier needs
// the whole grid resident), cached per device. Computed from the kernel's own
// resources -- shared memory, registers, threads and TMEM columns (512 per SM) --
// because the runtime's occupancy query answers 1 for this kernel while two CTAs
// per SM run side by side.
int front_fused_blocks_per_sm() {
  static int cached[64];
  static bool have[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (have[dev]) return cached[dev];
  static bool done[64] = {false};
  if (allow_max_smem((const void*)front_fused_kernel<true, false>, done) != cudaSuccess) return 0;
  cudaFuncAttributes a;
  cudaDeviceProp pr;
  if (cudaFuncGetAttributes(&a, (const void*)front_fused_kernel<true, false>) != cudaSuccess ||
      cudaGetDeviceProperties(&pr, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const size_t smem = sizeof(FusedSmem) + 128 + a.sharedSizeBytes + pr.reservedSharedMemPerBlock;
  const int by_smem = (int)(pr.sharedMemPerMultiprocessor / smem);
  const int regs_warp = ((a.numRegs * 32 + 255) / 256) * 256;           // 256-register granules
  const int by_regs = pr.regsPerMultiprocessor / (regs_warp * (kFrontThreads / 32));
  const int by_threads = pr.maxThreadsPerMultiProcessor / kFrontThreads;
  const int by_tmem = 512 / kFusedTmemCols;
  int n = by_smem < by_regs ? by_smem : by_regs;
  n = n < by_threads ? n : by_threads;
  n = n < by_tmem ? n : by_tmem;
  cached[dev] = n;
  have[dev] = true;
  return n;
}

// The QuantCNN chain through the pipelined kernel (x_nhwc rows, P = 0).
cudaError_t launch_chain(const FrontParams& p, int grid, cudaStream_t st) {
  static bool done_c[64] = {false};
  cudaError_t e = allow_max_smem((const void*)front_fused_kernel<false, false>, done_c);
  if (e != cudaSuccess) return e;
  return launch_k(front_fused_kernel<false, false>, dim3(grid), dim3(kFrontThreads), kFusedSmemSingle, st, false, p);
}

template <int MODE>
cudaError_t launch_front(const FrontParams& p, int grid, cudaStream_t st, bool pdl) {
  if constexpr (MODE == kModeFront) {
    // the fused forward's front runs the pipelined kernel
    static bool done_f[64] = {false};
    static bool done_d[64] = {false};
    if (p.dual) {
      cudaError_t e = allow_max_smem((const void*)front_fused_kernel<true, true>, done_d);
      if (e != cudaSuccess) return e;
      return launch_k(front_fused_kernel<true, true>, dim3(grid), dim3(kFrontThreads), kFusedSmemDual, st,
                      pdl, p);
    }
    if (p.norm_mean) {
      static bool done_n[64] = {false};
      cudaError_t e = allow_max_smem((const void*)front_fused_kernel<true, false, true>, done_n);
      if (e != cudaSuccess) return e;
      return launch_k(front_fused_kernel<true, false, true>, dim3(grid), dim3(kFrontThreads), kFusedSmemSingle,
                      st, pdl, p);
    }
    cudaError_t e = allow_max_smem((const void*)front_fused_kernel<true, false>, done_f);
    if (e != cudaSuccess) return e;
    return launch_k(front_fused_kernel<true, false>, dim3(grid), dim3(kFrontThreads), kFusedSmemSingle, st,
                    pdl, p);
  } else {
    const size_t smem = front_smem_bytes();
    static bool done[64] = {false};
    cudaError_t e = allow_max_smem((const void*)front_kernel<MODE>, done);
    if (e != cudaSuccess) return e;
    return launch_k(front_kernel<MODE>, dim3(grid), dim3(kFrontThreads), smem, st, pdl, p);
  }
}

template cudaError_t launch_front<kModeConv1>(const FrontParams&, int, cudaStream_t, bool);
template cudaError_t launch_front<kModeConv2>(const FrontParams&, int, cudaStream_t, bool);
template cudaError_t launch_front<kModeChain>(const FrontParams&, int, cudaStream_t, bool);
template cudaError_t launch_front<kModeFront>(const FrontParams&, int, cudaStream_t, bool);

}  // namespace glad
