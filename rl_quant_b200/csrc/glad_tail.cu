// Encoder tail, eight environments per CTA (one warp each):
//   query = QuantLinear(cat(gc, proprio_emb))            qrt/encoder_opt.py:78-79
//   score_query, top-32 of score_local + score_query     qrt/encoder_opt.py:82-95
//   local features of the 32 selected tokens             (conv2 recomputed from z8)
//   16-head single-query attention + out projection      qrt/encoder_opt.py:104-119
//   encoded[:, 0:64] = foothold; absmax for actor.0      qrt/encoder_opt.py:122
//
// The 187 local features are never stored: the front kernel keeps z8 (16 bytes
// per token) and this kernel recomputes conv2 for the 32 selected tokens only
// (identical integer arithmetic and epilogue, so identical fp16 values).
// GEMM rows are r = 32*warp + slot (M = 256 = 8 environments x 32 tokens, two
// M=128 tiles: warps 0-3 and 4-7). The per-warp GEMVs read transposed weight
// copies so that a warp's 32 lanes hit 32 different banks.
#include <cuda_runtime.h>

#include "glad_common.cuh"

namespace glad {

constexpr int kTailWarps = 8;                // one warp per environment slot
constexpr int kTailThreads = 32 * kTailWarps;
constexpr int kTailRows = 32 * kTailWarps;   // GEMM rows per CTA
// Environments per group: 7 of the 8 warp slots, so that 4096 environments make 586
// groups = two per resident CTA (2 per SM x 148) with no third wave; slot 7 is idle.
constexpr int kTailEnvs = 7;
constexpr int kTailTmemCols = 256;           // tile t: columns [128t, 128t+128): conv2, then K|V
constexpr int kTailMaxProp = 104;            // proprio columns of an encoded row
// Inputs of one environment, copied one group ahead: the proprio embedding (64 halves),
// then enc[64, 128 + P) (gc and the proprio columns), so that stage half k >= 64 is enc[k].
constexpr int kTailStageBytes = 2 * kD + 2 * (kD + kTailMaxProp);

// The [k pair c][n pair np] weight tables are read by lane np at a fixed c; element
// (c, np) sits at c*32 + (np ^ (c & 15)), so that the set-up's writes (32 consecutive c
// at a fixed np) take 2 shared-memory wavefronts per warp instead of 32.
__device__ __forceinline__ int swz(int c, int np) { return c * 32 + (np ^ (c & 15)); }

struct __align__(128) TailSmem {
  uint8_t w2s[5 * 2048];          // conv2 B operand (same layout as the front kernel)
  // im2col rows of the selected tokens [tap][row][16 B]; after the conv2 MMA the
  // same bytes hold the local features (fp16) [k8 chunk][row][16 B]
  uint8_t a12[10 * kTailRows * 16];
  uint8_t bkv[8 * 2048];          // in_proj rows 64..191 fp16: [k8 chunk][n][16B]
  uint2 wqT[32 * 32];             // in_proj rows 0..63: [k pair][n pair] -> half2 (n even), half2 (n odd) (swz)
  uint2 woT[32 * 32];             // out_proj, same layout
  int2 w8qpT[32 * 32];            // query_projector int8: [k quad][n pair] (swz)
  alignas(16) uint8_t stage[2][kTailWarps][kTailStageBytes];   // [group parity][warp]
  float qp_a[128], qp_b[128];
  float qp_scale[64], qp_bp[64];
  alignas(16) float dq[64];
  alignas(16) float b2[64];
  alignas(16) float a2c[64];
  float4 ck[64];                  // conv2 epilogue constants per channel {dq, b2, a2, c2}
  alignas(16) float c2[64];
  float bin[192], bout[64];
  __half2 binh[64];              // in_proj bias of K (pairs 0-31) and V (32-63) as half2
  __half2 bqh[32], bouth[32];    // in_proj bias of Q and out_proj bias as half2 pairs
  float wsq[64];                  // scorer weight, query half
  float a0_a[232], a0_b[232];
  float qv[kTailWarps][64];        // query (fp16 values)
  float qm[kTailWarps][64];        // MHA query projection (fp16 values)
  float om[kTailWarps][64];        // attention output (fp16 values)
  uint32_t keys[kTailWarps][32];
  int sel[kTailWarps][32];
  uint64_t mbar;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ uint32_t ord16(__half h) {
  uint32_t b = __half_as_ushort(h);
  if (b == 0x8000u) b = 0;                       // -0 ranks with +0
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

__global__ void __launch_bounds__(kTailThreads, 2) tail_kernel(const __grid_constant__ TailParams p) {
  extern __shared__ uint8_t smem_raw[];
  TailSmem& s = *reinterpret_cast<TailSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NT = kTailThreads;

  grid_dep_launch();
  if (warp == 0) tmem_alloc(&s.tmem_base, kTailTmemCols);
  if (tid == 0) {
    mbar_init(&s.mbar, 1);
    fence_mbar_init();
    s.abort_flag = 0;
  }
  // ---- constants: every global read is issued before the first wait. Raw weights go to
  //      scratch (the im2col buffer) and are re-laid shared -> shared afterwards. ----------------
  uint8_t* scratch = s.a12;
  const bool dyn = p.act_mode == GLAD_ACT_DYNAMIC;
  const bool a0_let = p.a0_alpha != nullptr;
  const int enc_w = 128 + p.prop_dim;
  {
    const uint4* w8 = reinterpret_cast<const uint4*>(p.conv.w8);        // [3*64*64] int8
    const uint4* wi = reinterpret_cast<const uint4*>(p.in_w);           // rows 0..63: [64*64] fp16
    const uint4* wo = reinterpret_cast<const uint4*>(p.out_w);          // [64*64] fp16
    const uint4* wq = reinterpret_cast<const uint4*>(p.qp.w8);          // [64*128] int8
    for (int i = tid; i < 768; i += NT) cp_async16(scratch + 16 * i, w8 + i);
    for (int i = tid; i < 512; i += NT) {
      cp_async16(scratch + 12288 + 16 * i, wi + i);
      cp_async16(scratch + 20480 + 16 * i, wo + i);
      cp_async16(scratch + 28672 + 16 * i, wq + i);
    }
    for (int idx = tid; idx < 128 * 64 / 8; idx += NT) {
      // bkv[c][n][8 halves] <- in_proj_weight[64 + n][8c .. 8c+8)
      const int n = idx >> 3, c = idx & 7;
      cp_async16(s.bkv + (c * 128 + n) * 16, p.in_w + (64 + n) * 64 + 8 * c);
    }
    for (int k = tid; k < 128; k += NT) {
      if (p.qp.alpha) {
        cp_async4(&s.qp_a[k], p.qp.alpha + k);
        cp_async4(&s.qp_b[k], p.qp.beta + k);
      } else {
        s.qp_a[k] = 0.0f;
        s.qp_b[k] = 0.0f;
      }
    }
    for (int i = tid; i < 64; i += NT) {
      cp_async4(&s.qp_scale[i], (dyn ? p.qp.s_w : p.qp.dq_scale) + i);   // raw; scaled below
      cp_async4(&s.qp_bp[i], p.qp.b_prime + i);
      cp_async4(&s.dq[i], p.conv.dq + i);
      cp_async4(&s.b2[i], p.conv.b2f + i);
      cp_async4(&s.a2c[i], p.conv.a2 + i);
      cp_async4(&s.c2[i], p.conv.c2 + i);
    }
    for (int k = tid; k < enc_w; k += NT) {
      if (a0_let) {
        cp_async4(&s.a0_a[k], p.a0_alpha + k);
        cp_async4(&s.a0_b[k], p.a0_beta + k);
      } else {
        s.a0_a[k] = 0.0f;
        s.a0_b[k] = 0.0f;
      }
    }
    cp_async_commit();
  }
  // fp16 vectors through registers
  float r_bout = 0.0f, r_wsq = 0.0f;
  if (tid < 64) {
    r_bout = __half2float(p.out_b[tid]);
    r_wsq = __half2float(p.scorer_w[64 + tid]);
  }
  float r_bin = tid < 192 ? __half2float(p.in_b[tid]) : 0.0f;
  const float sb = __half2float(p.scorer_b[0]);
  // the weight tables need nothing of the front kernel: built before the dependency wait
  cp_async_wait_all();
  __syncthreads();
  conv2_b_relayout(s.w2s, scratch, tid, NT);
  for (int idx = tid; idx < 32 * 32; idx += NT) {
    // [k pair c][n pair np]: (W[2np][2c..], W[2np+1][2c..]) as two half2 (int8: two 4-byte
    // words); a warp reads 32 consecutive c of one row pair
    const int c = idx & 31, np = idx >> 5;
    const uint32_t* wi = reinterpret_cast<const uint32_t*>(scratch + 12288);
    const uint32_t* wo = reinterpret_cast<const uint32_t*>(scratch + 20480);
    const int* w8 = reinterpret_cast<const int*>(scratch + 28672);
    const int d = swz(c, np);
    s.wqT[d] = make_uint2(wi[(2 * np) * 32 + c], wi[(2 * np + 1) * 32 + c]);
    s.woT[d] = make_uint2(wo[(2 * np) * 32 + c], wo[(2 * np + 1) * 32 + c]);
    s.w8qpT[d] = make_int2(w8[(2 * np) * 32 + c], w8[(2 * np + 1) * 32 + c]);
  }
  if (tid < 64) {
    s.bout[tid] = r_bout;
    s.wsq[tid] = r_wsq;
    s.ck[tid] = make_float4(s.dq[tid], s.b2[tid], s.a2c[tid], s.c2[tid]);
  }
  if (tid < 192) s.bin[tid] = r_bin;
  if (tid < 64) s.binh[tid] = __halves2half2(p.in_b[64 + 2 * tid], p.in_b[65 + 2 * tid]);
  if (tid < 32) {
    s.bqh[tid] = __halves2half2(p.in_b[2 * tid], p.in_b[2 * tid + 1]);
    s.bouth[tid] = __halves2half2(p.out_b[2 * tid], p.out_b[2 * tid + 1]);
  }
  for (int idx = tid; idx < kTailRows; idx += NT)      // zero filler tap 9 (past the raw weights)
    reinterpret_cast<uint4*>(s.a12 + 9 * kTailRows * 16)[idx] = make_uint4(0, 0, 0, 0);
  const int64_t ngroups = (p.B + kTailEnvs - 1) / kTailEnvs;
  // this warp's inputs of group g -> stage[b]: the proprio embedding row, then enc[64, 128 + P)
  // in 8-byte copies (rows start on 8-byte boundaries; the last copy may take up to three
  // halves of the row's padding, never read)
  auto prefetch = [&](int64_t g, int b) {
    const int64_t e = g * kTailEnvs + warp;
    if (warp >= kTailEnvs || g >= ngroups || e >= p.B) return;
    uint8_t* st = s.stage[b][warp];
    const uint8_t* pe_row = reinterpret_cast<const uint8_t*>(p.pe + e * kD);
    const uint8_t* enc_row = reinterpret_cast<const uint8_t*>(p.enc + e * p.ld_enc + kD);
    const int n_pe = 2 * kD / 8, n_all = n_pe + (2 * (kD + p.prop_dim) + 7) / 8;
    for (int c = lane; c < n_all; c += 32) {
      if (c < n_pe) cp_async8(st + 8 * c, pe_row + 8 * c);
      else cp_async8(st + 8 * c, enc_row + 8 * (c - n_pe));
    }
  };
  grid_dep_wait();                      // outputs of the front kernel are visible from here
  prefetch(blockIdx.x, 0);
  cp_async_commit();
  const ActQuant aq = make_act_quant(p.qp, p.act_mode, p.slots, p.qp_slot);
  if (tid < 64 && dyn) s.qp_scale[tid] = __fmul_rn(s.qp_scale[tid], aq.s);      // s_w * s_z
  const uint64_t g_offset = p.gumbel ? (uint64_t)*p.gumbel_offset : 0ull;
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  const int tile = warp >> 2;
  const uint32_t tcol = tmem + tile * 128 + ((uint32_t)(32 * (warp & 3)) << 16);
  uint32_t phase = 0;
  float zmax_a0 = 0.0f;
  ActQuant aq_a0{};
  aq_a0.let = a0_let;

  int buf = 0;
  for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, buf ^= 1) {
    const int64_t env = g * kTailEnvs + warp;
    const bool have = warp < kTailEnvs && env < p.B;
    const int r = 32 * warp + lane;              // GEMM row of this thread
    cp_async_wait_all();                         // this group's stage: the only copies in flight
    __syncwarp();
    const __half* stg = reinterpret_cast<const __half*>(s.stage[buf][warp]);   // pe | enc[64..]
    float zm_enc = 0.0f;                         // actor.0 absmax over enc[64, 128 + P)
    if (have) {
      // this environment's local scores, loaded first (used after the two GEMVs)
      __half sl[6];
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        const int i = lane + 32 * j;
        sl[j] = i < kTok ? p.score_local[env * kTok + i] : __float2half(0.0f);
      }
      // ---- 1. query projector: W8A8 over cat(gc, pe) (gc = enc[64, 128)) -------------
      uint32_t qword = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int k = 4 * lane + b;
        const float x = __half2float(k < 64 ? stg[64 + k] : stg[k - 64]);
        qword |= (uint32_t)(aq.quant(x, s.qp_a[k], s.qp_b[k]) & 0xFF) << (8 * b);
      }
      if (p.act_mode == GLAD_ACT_DYNAMIC && p.a0_absmax)
        for (int k = 64 + lane; k < enc_w; k += 32)    // |alpha*enc + beta| for actor.0's s_z
          zm_enc = fmaxf(zm_enc, aq_a0.absz(__half2float(stg[k]), s.a0_a[k], s.a0_b[k]));
      int acc0 = 0, acc1 = 0;
#pragma unroll
      for (int w = 0; w < 32; ++w) {
        const int qw = (int)__shfl_sync(0xffffffffu, qword, w);
        const int2 wv = s.w8qpT[swz(w, lane)];
        acc0 = __dp4a(qw, wv.x, acc0);
        acc1 = __dp4a(qw, wv.y, acc1);
      }
      // y = fp16(acc*scale + b') (qlinear_out); |acc| <= 128*128*128 < 2^22
      const float2 q01 = fp16r2(__fadd_rn(__fmul_rn(i2f_small(acc0), s.qp_scale[2 * lane]), s.qp_bp[2 * lane]),
                                __fadd_rn(__fmul_rn(i2f_small(acc1), s.qp_scale[2 * lane + 1]), s.qp_bp[2 * lane + 1]));
      const float q0 = q01.x, q1 = q01.y;
      s.qv[warp][2 * lane] = q0;
      s.qv[warp][2 * lane + 1] = q1;
      if (p.query_out)
        reinterpret_cast<__half2*>(p.query_out + env * kD)[lane] = __floats2half2_rn(q0, q1);
      // ---- 2. score_query = q @ w_s[:, 64:]^T + b_s (fp16 matmul then add) ----------------
      const float sqp = warp_sum(fmaf(q1, s.wsq[2 * lane + 1], q0 * s.wsq[2 * lane]));
      const float sq = fp16r(__fadd_rn(fp16r(sqp), sb));
      __syncwarp();
      // ---- 3. top-32 over 187 logits, value desc / index asc ------------------------------
      // fp16 logit = fp16(score_local + score_query): a half add (the fp32 sum of two fp16
      // values rounds to the same fp16 as the exact sum); the Gumbel term is fp16-valued too
      uint32_t key[6];
      const __half sqh = __float2half_rn(sq);
#pragma unroll
      for (int j = 0; j < 6; ++j) {
        const int i = lane + 32 * j;
        key[j] = 0;
        if (i < kTok) {
          __half lh = __hadd_rn(sl[j], sqh);
          if (p.gumbel) lh = __hadd_rn(lh, __float2half_rn(gumbel16(p.gumbel_seed, g_offset, env, i)));
          else if (p.noise) lh = __float2half_rn(__fadd_rn(__half2float(lh), p.noise[env * kTok + i]));
          if (p.topk_logits_out) p.topk_logits_out[env * kTok + i] = lh;
          key[j] = (ord16(lh) << 16) | (uint32_t)(0xFFFF - i);
        }
      }
      // threshold = the 32nd largest key: first the 32nd largest fp16 value t (radix over
      // the 16 value bits, two bits per step, the three counts of a step packed into one
      // warp reduction: 10 bits each, at most 187), then among the keys of value t the
      // (32 - #greater)-th lowest token index
      uint32_t thr;
      {
        uint32_t t = 0;
#pragma unroll 1
        for (int bb = 30; bb >= 16; bb -= 2) {
          const uint32_t c1 = t | (1u << bb), c2 = t | (2u << bb), c3 = t | (3u << bb);
          uint32_t pk = 0;
#pragma unroll
          for (int j = 0; j < 6; ++j)
            pk += (key[j] >= c1 ? 1u : 0u) + (key[j] >= c2 ? (1u << 10) : 0u) + (key[j] >= c3 ? (1u << 20) : 0u);
          pk = __reduce_add_sync(0xffffffffu, pk);
          const uint32_t n1 = pk & 1023u, n2 = (pk >> 10) & 1023u, n3 = pk >> 20;
          t = n3 >= kTopK ? c3 : n2 >= kTopK ? c2 : n1 >= kTopK ? c1 : t;
        }
        uint32_t gt = 0;
#pragma unroll
        for (int j = 0; j < 6; ++j) gt += key[j] > (t | 0xFFFFu) ? 1u : 0u;   // value above t
        const int need = kTopK - (int)__reduce_add_sync(0xffffffffu, gt);   // >= 1
        int acc = 0;
        thr = t;
#pragma unroll
        for (int j = 0; j < 6; ++j) {
          const uint32_t ball = __ballot_sync(0xffffffffu, key[j] != 0 && (key[j] & 0xFFFF0000u) == t);
          const int c = __popc(ball);
          if (acc < need && acc + c >= need)
            thr = t | (0xFFFFu - (uint32_t)(32 * j + (int)__fns(ball, 0, need - acc)));
          acc += c;
        }
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
        uint8_t* dst = s.a12 + q * (kTailRows * 16) + r * 16;
        if (ih >= 0 && ih < kH2 && iw >= 0 && iw < kW2)
          cp_async16(dst, p.z8 + (env * kTok + ih * kW2 + iw) * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
      // MHA query projection: q_mha = fp16(fp16(query @ Wq^T) + b_q); lane -> n = 2*lane, 2*lane+1
      // (after the gather is issued: the GEMV runs while the z8 rows arrive)
      {
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int c2 = 0; c2 < 32; ++c2) {
          const uint2 wv = s.wqT[swz(c2, lane)];
          const float x0 = s.qv[warp][2 * c2], x1 = s.qv[warp][2 * c2 + 1];
          const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
          const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
          a0 = fmaf(x0, w0.x, a0);
          a0 = fmaf(x1, w0.y, a0);
          a1 = fmaf(x0, w1.x, a1);
          a1 = fmaf(x1, w1.y, a1);
        }
        const float2 qm = __half22float2(__hadd2_rn(__floats2half2_rn(a0, a1), s.bqh[lane]));
        s.qm[warp][2 * lane] = qm.x;
        s.qm[warp][2 * lane + 1] = qm.y;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 9; ++q)
        *reinterpret_cast<uint4*>(s.a12 + q * (kTailRows * 16) + r * 16) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
    cp_async_wait_all();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();

    // the next group's inputs land while this one finishes
    prefetch(g + gridDim.x, buf ^ 1);
    cp_async_commit();

    // ---- 5. conv2 recompute for the 256 selected rows (two M=128 tiles) -------------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ab = smem_u32(s.a12), wb = smem_u32(s.w2s);
      constexpr uint32_t idesc = idesc_i8(128, 64);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int pr = 0; pr < 5; ++pr) {
          const uint64_t ad = smem_desc(ab + pr * 2 * (kTailRows * 16) + t * 2048, kTailRows * 16, 128);
          const uint64_t bd = smem_desc(wb + pr * 2048, 1024, 128);
          mma_i8(tmem + t * 128, ad, bd, idesc, pr > 0 ? 1u : 0u);
        }
      mma_commit(&s.mbar);
    }
    bool ok = mbar_wait_bounded(&s.mbar, phase);
    phase ^= 1;
    if (!ok) s.abort_flag = 1;
    tc_fence_after();
    __syncthreads();
    if (s.abort_flag) break;

    // ---- 6. local features (fp16) -> A operand of the K|V projection (over the im2col bytes)
    // TMEM read in the 16x256b shape: a thread holds rows g, g+8, g+16, g+24 of its warp and
    // channels 2q, 2q+1, 8+2q, 9+2q of each 16-channel chunk, so it loads 4 channels'
    // constants per chunk instead of 16
    {
      const int q = lane & 3, g = lane >> 2;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t ra[8], rb[8];
        tmem_ld16x256b_x2(tcol + cb * 16, ra);
        tmem_ld16x256b_x2(tcol + cb * 16 + (16u << 16), rb);
        tmem_ld_wait();
        const int cc = cb * 16;
        const float4 k0 = s.ck[cc + 2 * q], k1 = s.ck[cc + 2 * q + 1];
        const float4 k2 = s.ck[cc + 8 + 2 * q], k3 = s.ck[cc + 9 + 2 * q];
        uint8_t* chunk = s.a12 + (2 * cb) * (kTailRows * 16) + 4 * q;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t (&v)[8] = hh ? rb : ra;
          const int row = 32 * warp + 16 * hh + g;      // and row + 8
          const __half2 h0 = __floats2half2_rn(conv2_val((int32_t)v[0], k0.x, k0.y, k0.z, k0.w),
                                               conv2_val((int32_t)v[1], k1.x, k1.y, k1.z, k1.w));
          const __half2 h1 = __floats2half2_rn(conv2_val((int32_t)v[2], k0.x, k0.y, k0.z, k0.w),
                                               conv2_val((int32_t)v[3], k1.x, k1.y, k1.z, k1.w));
          const __half2 h2 = __floats2half2_rn(conv2_val((int32_t)v[4], k2.x, k2.y, k2.z, k2.w),
                                               conv2_val((int32_t)v[5], k3.x, k3.y, k3.z, k3.w));
          const __half2 h3 = __floats2half2_rn(conv2_val((int32_t)v[6], k2.x, k2.y, k2.z, k2.w),
                                               conv2_val((int32_t)v[7], k3.x, k3.y, k3.z, k3.w));
          *reinterpret_cast<__half2*>(chunk + row * 16) = h0;
          *reinterpret_cast<__half2*>(chunk + (row + 8) * 16) = h1;
          *reinterpret_cast<__half2*>(chunk + kTailRows * 16 + row * 16) = h2;
          *reinterpret_cast<__half2*>(chunk + kTailRows * 16 + (row + 8) * 16) = h3;
        }
      }
    }
    tc_fence_before();
    fence_async_smem();
    __syncthreads();

    // ---- 7. K|V = local @ in_proj[64:192]^T (fp32 accumulate in TMEM, over conv2's columns)
    if (tid == 0) {
      tc_fence_after();
      const uint32_t ab = smem_u32(s.a12), bb = smem_u32(s.bkv);
      constexpr uint32_t idesc = idesc_f16(128, 128);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = smem_desc(ab + kk * 2 * (kTailRows * 16) + t * 2048, kTailRows * 16, 128);
          const uint64_t bd = smem_desc(bb + kk * 2 * 2048, 2048, 128);
          mma_f16(tmem + t * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
      mma_commit(&s.mbar);
    }
    ok = mbar_wait_bounded(&s.mbar, phase);
    phase ^= 1;
    if (!ok) s.abort_flag = 1;
    tc_fence_after();
    __syncthreads();
    if (s.abort_flag) break;

    // ---- 8. attention: thread = (env, token slot), 16 channels (4 heads) at a time ------------
    float sc[kHeads];
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t rr[16];
      tmem_ld16(tcol + cb * 16, rr);
      tmem_ld_wait();
      float dd[4];
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        float d = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int c = 16 * cb + 4 * hh + e;
          // fp16(fp16(k) + b): one half2 add (the fp32 sum of two fp16 values rounds to the
          // same fp16 as the exact sum, which is what the half add returns)
          const __half2 k0 = __floats2half2_rn(__uint_as_float(rr[4 * hh + e]), __uint_as_float(rr[4 * hh + e + 1]));
          const float2 kv = __half22float2(__hadd2_rn(k0, s.binh[c >> 1]));
          d = fmaf(s.qm[warp][c], kv.x, d);
          d = fmaf(s.qm[warp][c + 1], kv.y, d);
        }
        dd[hh] = d;
      }
#pragma unroll
      for (int hh = 0; hh < 4; hh += 2) {
        // fp16(fp16(d) * 0.5): a half multiply by 0.5 rounds the same exact product
        const float2 s01 = __half22float2(__hmul2_rn(__floats2half2_rn(dd[hh], dd[hh + 1]), __float2half2_rn(0.5f)));
        sc[4 * cb + hh] = s01.x;
        sc[4 * cb + hh + 1] = s01.y;
      }
    }
    // softmax over the 32 tokens of every head: the 16 heads' butterflies interleaved
    float red[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) red[h] = sc[h];
    warp_allreduce16<true>(red, lane);
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      sc[h] = expf(sc[h] - red[h]);
      red[h] = sc[h];
    }
    warp_allreduce16<false>(red, lane);
    float asum = 0.0f;
#pragma unroll
    for (int h = 0; h < kHeads; h += 2) {
      const float2 a = fp16r2(__fdiv_rn(sc[h], red[h]), __fdiv_rn(sc[h + 1], red[h + 1]));
      asum += a.x;
      asum += a.y;
      sc[h] = a.x;
      sc[h + 1] = a.y;
    }
    if (have && p.attn_w_out) p.attn_w_out[env * kTopK + lane] = __float2half_rn(asum / 16.0f);
#pragma unroll
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t rr[16];
      tmem_ld16(tcol + 64 + cb * 16, rr);
      tmem_ld_wait();
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const int c = 16 * cb + j;
        const __half2 v0 = __floats2half2_rn(__uint_as_float(rr[j]), __uint_as_float(rr[j + 1]));
        const float2 vb = __half22float2(__hadd2_rn(v0, s.binh[32 + (c >> 1)]));
        v[j] = sc[4 * cb + (j >> 2)] * vb.x;
        v[j + 1] = sc[4 * cb + (j >> 2)] * vb.y;
      }
      const float o = warp_reduce16(v, lane);    // lanes L, L^16: channel 16*cb + (L & 15)
      if (lane < 16) s.om[warp][16 * cb + lane] = fp16r(o);
    }
    tc_fence_before();
    __syncwarp();
    // ---- 9. foothold = out_proj(o), encoded[:, 0:64] ---------------------------------------
    if (have) {
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
      for (int c2 = 0; c2 < 32; ++c2) {
        const uint2 wv = s.woT[swz(c2, lane)];
        const float x0 = s.om[warp][2 * c2], x1 = s.om[warp][2 * c2 + 1];
        const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
        const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
        a0 = fmaf(x0, w0.x, a0);
        a0 = fmaf(x1, w0.y, a0);
        a1 = fmaf(x0, w1.x, a1);
        a1 = fmaf(x1, w1.y, a1);
      }
      const float2 f01 = __half22float2(__hadd2_rn(__floats2half2_rn(a0, a1), s.bouth[lane]));
      const float f0 = f01.x, f1 = f01.y;
      reinterpret_cast<__half2*>(p.enc + env * p.ld_enc)[lane] = __floats2half2_rn(f0, f1);
      if (p.act_mode == GLAD_ACT_DYNAMIC && p.a0_absmax) {
        // |alpha*encoded + beta| for actor.0's dynamic s_z
        const float zm = fmaxf(aq_a0.absz(f0, s.a0_a[2 * lane], s.a0_b[2 * lane]),
                               aq_a0.absz(f1, s.a0_a[2 * lane + 1], s.a0_b[2 * lane + 1]));
        zmax_a0 = fmaxf(zmax_a0, fmaxf(zm, zm_enc));
      }
    }
    __syncthreads();
  }
  cp_async_wait_all();                           // a prefetch left in flight by an abort

  if (p.act_mode == GLAD_ACT_DYNAMIC && p.a0_absmax) {
    // one atomic per CTA on actor.0's absmax slot
    const float m = warp_max(zmax_a0);
    if (lane == 0) s.qv[warp][0] = m;            // the query rows are free after the last group
    __syncthreads();
    if (tid == 0) {
      float mm = s.qv[0][0];
#pragma unroll
      for (int w = 1; w < kTailWarps; ++w) mm = fmaxf(mm, s.qv[w][0]);
      if (mm > 0.0f) atomic_max_nonneg(&p.slots[2], mm);
    }
  }
  if (p.gumbel && tid == 0) {
    // the last CTA to finish advances the offset for the next call (every CTA has read it)
    __threadfence();
    if (atomicAdd(reinterpret_cast<unsigned int*>(&p.slots[p.done_slot]), 1u) == gridDim.x - 1)
      atomicAdd(p.gumbel_offset, 1ull);
  }
  if (s.abort_flag) {
    mbar_wait_bounded(&s.mbar, phase ^ 1);
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
// two CTAs per SM (228 KB of shared memory, 1 KB of it reserved per CTA)
static_assert(2 * (sizeof(TailSmem) + 128 + 1024) <= 228 * 1024, "tail shared memory");

// Persistent grid: one CTA per group of environments, at most two per SM.
int tail_grid(int64_t B, int sms) {
  const int64_t groups = (B + kTailEnvs - 1) / kTailEnvs;
  return (int)(groups < (int64_t)sms * 2 ? groups : (int64_t)sms * 2);
}

cudaError_t launch_tail(const TailParams& p, int grid, cudaStream_t st, bool pdl) {
  // the staged copies of an encoded row need 8-byte row starts, P <= kTailMaxProp and the
  // row's columns up to the next multiple of 4 inside its stride
  if (p.ld_enc % 4 || p.prop_dim < 0 || p.prop_dim > kTailMaxProp || 128 + ((p.prop_dim + 3) & ~3) > p.ld_enc)
    return cudaErrorInvalidValue;
  const size_t smem = tail_smem_bytes();
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)tail_kernel, done);
  if (e != cudaSuccess) return e;
  return launch_k(tail_kernel, dim3(grid), dim3(kTailThreads), smem, st, pdl, p);
}

}  // namespace glad
