// Encoder tail, four environments per CTA (one warp each):
//   query = QuantLinear(cat(gc, proprio_emb))            qrt/encoder_opt.py:78-79
//   score_query, top-32 of score_local + score_query     qrt/encoder_opt.py:82-95
//   local features of the 32 selected tokens             (conv2 recomputed from z8)
//   16-head single-query attention + out projection      qrt/encoder_opt.py:104-119
//   encoded[:, 0:64] = foothold; absmax for actor.0      qrt/encoder_opt.py:122
//
// The 187 local features are never stored: the front kernel keeps z8 (16 bytes
// per token) and this kernel recomputes conv2 for the 32 selected tokens only
// (identical integer arithmetic and epilogue, so identical fp16 values).
// GEMM rows here are r = 32*warp + slot (M = 128 = 4 environments x 32 tokens).
#include <cuda_runtime.h>

#include "glad_common.cuh"

namespace glad {

constexpr int kTailTmemCols = 256;   // [0,64) conv2 recompute, [64,192) K|V projection

struct __align__(128) TailSmem {
  uint8_t w2s[5 * 2048];          // conv2 B operand (same layout as the front kernel)
  uint8_t a1[10 * 2048];          // im2col rows of the selected tokens: [tap][row][16B]
  uint8_t a2[8 * 2048];           // local features fp16: [k8 chunk][row][16B]
  uint8_t bkv[8 * 2048];          // in_proj rows 64..191 fp16: [k8 chunk][n][16B]
  __half wq[64 * 64];             // in_proj rows 0..63
  __half wo[64 * 64];             // out_proj
  alignas(16) int8_t w8qp[64 * 128];
  float qp_a[128], qp_b[128];
  float qp_scale[64], qp_bp[64];
  float dq[64], b2[64], a2c[64], c2[64];
  float bin[192], bout[64];
  float wsq[64];                  // scorer weight, query half
  float a0_a[232], a0_b[232];
  float qv[4][64];                // query (fp16 values)
  float qm[4][64];                // MHA query projection (fp16 values)
  float om[4][64];                // attention output (fp16 values)
  uint32_t keys[4][32];
  int sel[4][32];
  uint64_t mbar;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t ord16(__half h) {
  uint32_t b = __half_as_ushort(h);
  if (b == 0x8000u) b = 0;                       // -0 ranks with +0
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

__global__ void __launch_bounds__(128, 2) tail_kernel(const __grid_constant__ TailParams p) {
  extern __shared__ uint8_t smem_raw[];
  TailSmem& s = *reinterpret_cast<TailSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  grid_dep_launch();
  if (warp == 0) tmem_alloc(&s.tmem_base, kTailTmemCols);
  if (tid == 0) {
    mbar_init(&s.mbar, 1);
    fence_mbar_init();
    s.abort_flag = 0;
  }
  // ---- constants -------------------------------------------------------------------
  for (int idx = tid; idx < 5 * 2048; idx += 128) {
    const int pr = idx >> 11, c = (idx >> 10) & 1, n = (idx >> 4) & 63, e = idx & 15;
    const int q = 2 * pr + c;
    s.w2s[idx] = q < 9 ? (uint8_t)p.conv.w8[((q / 3) * 64 + (q % 3) * 16 + e) * 64 + n] : 0;
  }
  for (int idx = tid; idx < 2048 / 16; idx += 128)
    reinterpret_cast<uint4*>(s.a1 + 9 * 2048)[idx] = make_uint4(0, 0, 0, 0);
  for (int idx = tid; idx < 128 * 64 / 8; idx += 128) {
    // bkv[c][n][8 halves] <- in_proj_weight[64 + n][8c .. 8c+8)
    const int n = idx >> 3, c = idx & 7;
    reinterpret_cast<uint4*>(s.bkv)[c * 128 + n] =
        reinterpret_cast<const uint4*>(p.in_w + (64 + n) * 64)[c];
  }
  for (int idx = tid; idx < 64 * 64 / 8; idx += 128) {
    reinterpret_cast<uint4*>(s.wq)[idx] = reinterpret_cast<const uint4*>(p.in_w)[idx];
    reinterpret_cast<uint4*>(s.wo)[idx] = reinterpret_cast<const uint4*>(p.out_w)[idx];
  }
  for (int idx = tid; idx < 64 * 128 / 16; idx += 128)
    reinterpret_cast<uint4*>(s.w8qp)[idx] = reinterpret_cast<const uint4*>(p.qp.w8)[idx];
  grid_dep_wait();                      // outputs of the front kernel are visible from here
  const ActQuant aq = make_act_quant(p.qp, p.act_mode, p.slots, 1);
  for (int k = tid; k < 128; k += 128) {
    s.qp_a[k] = aq.let ? p.qp.alpha[k] : 0.0f;
    s.qp_b[k] = aq.let ? p.qp.beta[k] : 0.0f;
  }
  if (tid < 64) {
    s.qp_scale[tid] = out_scale(p.qp, aq, tid);
    s.qp_bp[tid] = p.qp.b_prime[tid];
    s.dq[tid] = p.conv.dq[tid];
    s.b2[tid] = p.conv.b2f[tid];
    s.a2c[tid] = p.conv.a2[tid];
    s.c2[tid] = p.conv.c2[tid];
    s.bout[tid] = __half2float(p.out_b[tid]);
    s.wsq[tid] = __half2float(p.scorer_w[64 + tid]);
  }
  for (int k = tid; k < 192; k += 128) s.bin[k] = __half2float(p.in_b[k]);
  const bool a0_let = p.a0_alpha != nullptr;
  const int enc_w = 128 + p.prop_dim;
  for (int k = tid; k < enc_w; k += 128) {
    s.a0_a[k] = a0_let ? p.a0_alpha[k] : 0.0f;
    s.a0_b[k] = a0_let ? p.a0_beta[k] : 0.0f;
  }
  const float sb = __half2float(p.scorer_b[0]);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  uint32_t phase = 0;
  float zmax_a0 = 0.0f;
  ActQuant aq_a0{};
  aq_a0.let = a0_let;

  const int64_t ngroups = (p.B + 3) / 4;
  for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x) {
    const int64_t env = g * 4 + warp;
    const bool have = env < p.B;
    const int r = 32 * warp + lane;              // GEMM row of this thread
    if (have) {
      // ---- 1. query projector: W8A8 over cat(gc, pe) ---------------------------------
      const __half* gc = p.enc + env * p.ld_enc + 64;
      const __half* pe = p.pe + env * kD;
      uint32_t qword = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int k = 4 * lane + b;
        const float x = __half2float(k < 64 ? gc[k] : pe[k - 64]);
        qword |= (uint32_t)(aq.quant(x, s.qp_a[k], s.qp_b[k]) & 0xFF) << (8 * b);
      }
      int acc0 = 0, acc1 = 0;
      const int* w0 = reinterpret_cast<const int*>(s.w8qp + (2 * lane) * 128);
      const int* w1 = reinterpret_cast<const int*>(s.w8qp + (2 * lane + 1) * 128);
#pragma unroll
      for (int w = 0; w < 32; ++w) {
        const int qw = (int)__shfl_sync(0xffffffffu, qword, w);
        acc0 = __dp4a(qw, w0[w], acc0);
        acc1 = __dp4a(qw, w1[w], acc1);
      }
      const float q0 = __half2float(qlinear_out(acc0, s.qp_scale[2 * lane], s.qp_bp[2 * lane]));
      const float q1 = __half2float(qlinear_out(acc1, s.qp_scale[2 * lane + 1], s.qp_bp[2 * lane + 1]));
      s.qv[warp][2 * lane] = q0;
      s.qv[warp][2 * lane + 1] = q1;
      // ---- 2. score_query = q @ w_s[:, 64:]^T + b_s (fp16 matmul then add) ----------------
      const float sqp = warp_sum(fmaf(q1, s.wsq[2 * lane + 1], q0 * s.wsq[2 * lane]));
      const float sq = fp16r(__fadd_rn(fp16r(sqp), sb));
      __syncwarp();
      // MHA query projection: q_mha = fp16(fp16(query @ Wq^T) + b_q)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = 2 * lane + h;
        float a = 0.0f;
        const __half2* wr = reinterpret_cast<const __half2*>(s.wq + n * 64);
#pragma unroll
        for (int c2 = 0; c2 < 32; ++c2) {
          const float2 w = __half22float2(wr[c2]);
          a = fmaf(s.qv[warp][2 * c2], w.x, a);
          a = fmaf(s.qv[warp][2 * c2 + 1], w.y, a);
        }
        s.qm[warp][n] = fp16r(__fadd_rn(fp16r(a), s.bin[n]));
      }
      // ---- 3. top-32 over 187 logits, value desc / index asc ------------------------------
      uint32_t key[6];
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        const int i = lane + 32 * j;
        key[j] = 0;
        if (i < kTok) {
          float lg = fp16r(__fadd_rn(__half2float(p.score_local[env * kTok + i]), sq));
          if (p.noise) lg = fp16r(__fadd_rn(lg, p.noise[env * kTok + i]));
          const __half lh = __float2half_rn(lg);
          if (p.topk_logits_out) p.topk_logits_out[env * kTok + i] = lh;
          key[j] = (ord16(lh) << 16) | (uint32_t)(0xFFFF - i);
        }
      }
      uint32_t thr = 0;
#pragma unroll 1
      for (int bit = 31; bit >= 0; --bit) {
        const uint32_t cand = thr | (1u << bit);
        int cnt = 0;
#pragma unroll
        for (int j = 0; j < 6; ++j) cnt += key[j] >= cand ? 1 : 0;
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        if (cnt >= kTopK) thr = cand;
      }
      int base = 0;
      const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        const bool take = key[j] >= thr && key[j] != 0;
        const uint32_t ball = __ballot_sync(0xffffffffu, take);
        if (take) s.keys[warp][base + __popc(ball & lt)] = key[j];
        base += __popc(ball);
      }
      __syncwarp();
      const uint32_t mine = s.keys[warp][lane];
      int rank = 0;
#pragma unroll
      for (int k = 0; k < 32; ++k) rank += s.keys[warp][k] > mine ? 1 : 0;
      s.sel[warp][rank] = 0xFFFF - (int)(mine & 0xFFFFu);
      __syncwarp();
      const int tok = s.sel[warp][lane];
      if (p.topk_idx_out) p.topk_idx_out[env * kTopK + lane] = tok;
      // ---- 4. im2col of the selected token (9 taps of z8, zero outside the grid) ----------
      const int oh = tok / kW2, ow = tok - (tok / kW2) * kW2;
#pragma unroll
      for (int q = 0; q < 9; ++q) {
        const int ih = oh + q / 3 - 1, iw = ow + q % 3 - 1;
        uint8_t* dst = s.a1 + q * 2048 + r * 16;
        if (ih >= 0 && ih < kH2 && iw >= 0 && iw < kW2)
          cp_async16(dst, p.z8 + (env * kTok + ih * kW2 + iw) * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 9; ++q)
        *reinterpret_cast<uint4*>(s.a1 + q * 2048 + r * 16) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
    cp_async_wait_all();
    fence_async_smem();
    __syncthreads();

    // ---- 5. conv2 recompute for the 128 selected rows ------------------------------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ab = smem_u32(s.a1), wb = smem_u32(s.w2s);
      constexpr uint32_t idesc = idesc_i8(128, 64);
#pragma unroll
      for (int pr = 0; pr < 5; ++pr) {
        const uint64_t ad = smem_desc(ab + pr * 2 * 2048, 2048, 128);
        const uint64_t bd = smem_desc(wb + pr * 2048, 1024, 128);
        mma_i8(tmem, ad, bd, idesc, pr > 0 ? 1u : 0u);
      }
      mma_commit(&s.mbar);
    }
    bool ok = mbar_wait_bounded(&s.mbar, phase);
    phase ^= 1;
    if (!ok) s.abort_flag = 1;
    tc_fence_after();
    __syncthreads();
    if (s.abort_flag) break;

    // ---- 6. local features (fp16) -> A operand of the K|V projection ---------------------
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t rr[16];
      tmem_ld16(tmem + lane_base + cb * 16, rr);
      tmem_ld_wait();
      __half h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = cb * 16 + j;
        h[j] = conv2_out((int32_t)rr[j], s.dq[c], s.b2[c], s.a2c[c], s.c2[c]);
      }
      *reinterpret_cast<uint4*>(s.a2 + (2 * cb) * 2048 + r * 16) = *reinterpret_cast<uint4*>(&h[0]);
      *reinterpret_cast<uint4*>(s.a2 + (2 * cb + 1) * 2048 + r * 16) = *reinterpret_cast<uint4*>(&h[8]);
    }
    tc_fence_before();
    fence_async_smem();
    __syncthreads();

    // ---- 7. K|V = local @ in_proj[64:192]^T (fp32 accumulate in TMEM) -------------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ab = smem_u32(s.a2), bb = smem_u32(s.bkv);
      constexpr uint32_t idesc = idesc_f16(128, 128);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = smem_desc(ab + kk * 2 * 2048, 2048, 128);
        const uint64_t bd = smem_desc(bb + kk * 2 * 2048, 2048, 128);
        mma_f16(tmem + 64, ad, bd, idesc, kk > 0 ? 1u : 0u);
      }
      mma_commit(&s.mbar);
    }
    ok = mbar_wait_bounded(&s.mbar, phase);
    phase ^= 1;
    if (!ok) s.abort_flag = 1;
    tc_fence_after();
    __syncthreads();
    if (s.abort_flag) break;

    // ---- 8. attention: thread = (env, token slot) --------------------------------------
    float kf[64], vf[64];
#pragma unroll
    for (int cb = 0; cb < 8; ++cb) {
      uint32_t rr[16];
      tmem_ld16(tmem + lane_base + 64 + cb * 16, rr);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = cb * 16 + j;             // 0..127: K then V
        const float v = fp16r(__fadd_rn(fp16r(__uint_as_float(rr[j])), s.bin[64 + c]));
        if (c < 64) kf[c] = v; else vf[c - 64] = v;
      }
    }
    tc_fence_before();
    float asum = 0.0f;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      float d = 0.0f;
#pragma unroll
      for (int e = 0; e < 4; ++e) d = fmaf(s.qm[warp][4 * h + e], kf[4 * h + e], d);
      const float sc = fp16r(__fmul_rn(fp16r(d), 0.5f));
      const float mx = warp_max(sc);
      const float ex = expf(sc - mx);
      const float sm = warp_sum(ex);
      const float a = fp16r(__fdiv_rn(ex, sm));
      asum += a;
#pragma unroll
      for (int e = 0; e < 4; ++e) vf[4 * h + e] = a * vf[4 * h + e];
    }
    if (have && p.attn_w_out) p.attn_w_out[env * kTopK + lane] = __float2half_rn(asum / 16.0f);
    warp_reduce64(vf, lane);
    {
      const int c0 = reduce64_channel(lane);
      s.om[warp][c0] = fp16r(vf[0]);
      s.om[warp][c0 + 1] = fp16r(vf[1]);
    }
    __syncwarp();
    // ---- 9. foothold = out_proj(o), encoded[:, 0:64] ---------------------------------------
    if (have) {
      float f2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = 2 * lane + h;
        float a = 0.0f;
        const __half2* wr = reinterpret_cast<const __half2*>(s.wo + n * 64);
#pragma unroll
        for (int c2 = 0; c2 < 32; ++c2) {
          const float2 w = __half22float2(wr[c2]);
          a = fmaf(s.om[warp][2 * c2], w.x, a);
          a = fmaf(s.om[warp][2 * c2 + 1], w.y, a);
        }
        f2[h] = fp16r(__fadd_rn(fp16r(a), s.bout[n]));
      }
      __half2 fh = __floats2half2_rn(f2[0], f2[1]);
      reinterpret_cast<__half2*>(p.enc + env * p.ld_enc)[lane] = fh;
      if (p.act_mode == GLAD_ACT_DYNAMIC && p.a0_absmax) {
        // |alpha*encoded + beta| for actor.0's dynamic s_z
        float zm = fmaxf(aq_a0.absz(f2[0], s.a0_a[2 * lane], s.a0_b[2 * lane]),
                         aq_a0.absz(f2[1], s.a0_a[2 * lane + 1], s.a0_b[2 * lane + 1]));
        for (int k = 64 + lane; k < enc_w; k += 32)
          zm = fmaxf(zm, aq_a0.absz(__half2float(p.enc[env * p.ld_enc + k]), s.a0_a[k], s.a0_b[k]));
        zmax_a0 = fmaxf(zmax_a0, zm);
      }
    }
    __syncthreads();
  }

  if (p.act_mode == GLAD_ACT_DYNAMIC && p.a0_absmax) {
    const float m = warp_max(zmax_a0);
    if (lane == 0 && m > 0.0f) atomic_max_nonneg(&p.slots[2], m);
  }
  if (s.abort_flag) {
    mbar_wait_bounded(&s.mbar, phase);
    if (tid == 0) atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrMmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTailTmemCols);
  }
}

size_t tail_smem_bytes() { return sizeof(TailSmem) + 128; }

cudaError_t launch_tail(const TailParams& p, int grid, cudaStream_t st, bool pdl) {
  const size_t smem = tail_smem_bytes();
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)tail_kernel, done);
  if (e != cudaSuccess) return e;
  return launch_k(tail_kernel, dim3(grid), dim3(128), smem, st, pdl, p);
}

}  // namespace glad
