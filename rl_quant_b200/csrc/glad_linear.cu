// W8A8 QuantLinear as a tcgen05 int8 GEMM, plus the small kernels of the
// forward (dynamic absmax) and of the weight refresh (requantisation,
// batched cast-copies).
//
// Reference: qrt/qlinear.py:84-138 (QuantLinear), qrt/qconv.py:247-284
// (QuantCNN.requantize_), qrt/runtime.py:224-271 (sync_weights_from).
#include <cuda_runtime.h>

#include "glad_common.cuh"

namespace glad {

// ---- tcgen05 int8 GEMM --------------------------------------------------------------
// CTA = 128 rows x NT columns, 256 threads. A (activations) is quantised on
// the way into shared memory, B is the layer's int8 weight rows. Both
// K-major, no swizzle:
//   A: [Kp/16 chunks][128 rows][16 B]   (LBO = 2048, SBO = 128)
//   B: [Kp/16 chunks][NT rows][16 B]    (LBO = NT*16, SBO = 128)
// Epilogue: warp w reads TMEM lane quarter (w & 3) and column half (w >> 2).
constexpr int kGemmThreads = 256;

template <int NT>
__global__ void __launch_bounds__(kGemmThreads, 1) qgemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int K = p.L.in_features;
  const int Kp = (K + 31) & ~31;         // K padded to the MMA K-step (zero fill)
  uint8_t* As = base;
  uint8_t* Bs = As + (size_t)Kp * 128;
  float* cscale = reinterpret_cast<float*>(Bs + (size_t)Kp * NT);
  float* cbias = cscale + NT;
  float* calpha = cbias + NT;
  float* cbeta = calpha + NT;
  float* kalpha = cbeta + NT;            // [Kp] this layer's LET
  float* kbeta = kalpha + Kp;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(kbeta + Kp);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t m0 = (int64_t)blockIdx.x * 128;
  const int n0 = blockIdx.y * NT;
  const int N = p.L.out_features;
  const int Np = (N + 7) & ~7;
  grid_dep_launch();
  constexpr uint32_t kCols = NT < 32 ? 32 : NT;

  if (warp == 0) tmem_alloc(tmem_slot, kCols);
  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
    *abort_flag = 0;
  }
  // weights: rows n0..n0+NT of w8 (zero past Np / K)
  const int kc16 = Kp / 16;
  const bool rows16 = (K & 15) == 0;
  for (int idx = tid; idx < NT * kc16; idx += kGemmThreads) {
    const int c = idx / NT, n = idx - c * NT;
    uint8_t* dst = Bs + c * (NT * 16) + n * 16;
    const int8_t* src = p.L.w8 + (int64_t)(n0 + n) * K + c * 16;
    if (n0 + n < Np && c * 16 + 16 <= K && rows16) {
      cp_async16(dst, src);
    } else {
      uint2 lo = make_uint2(0, 0), hi = make_uint2(0, 0);
      if (n0 + n < Np && c * 16 + 8 <= K) lo = *reinterpret_cast<const uint2*>(src);
      if (n0 + n < Np && c * 16 + 16 <= K) hi = *reinterpret_cast<const uint2*>(src + 8);
      *reinterpret_cast<uint4*>(dst) = make_uint4(lo.x, lo.y, hi.x, hi.y);
    }
  }
  cp_async_commit();
  grid_dep_wait();                      // the producer of x and of the absmax slot is done
  const ActQuant aq = make_act_quant(p.L, p.act_mode, p.slots, p.slot);
  for (int j = tid; j < NT; j += kGemmThreads) {
    const int n = n0 + j;
    const bool in = n < N;
    cscale[j] = in ? out_scale(p.L, aq, n) : 0.0f;
    cbias[j] = in ? p.L.b_prime[n] : 0.0f;
    calpha[j] = (in && p.next_let) ? p.next_alpha[n] : 0.0f;
    cbeta[j] = (in && p.next_let) ? p.next_beta[n] : 0.0f;
  }
  for (int k = tid; k < Kp; k += kGemmThreads) {
    kalpha[k] = (aq.let && k < K) ? p.L.alpha[k] : 0.0f;
    kbeta[k] = (aq.let && k < K) ? p.L.beta[k] : 0.0f;
  }
  __syncthreads();
  // activations: quantise 8 elements at a time
  const int k8n = Kp / 8, k8real = K / 8;
  const bool f32in = p.x_dtype == GLAD_DTYPE_F32;
  for (int idx = tid; idx < 128 * k8n; idx += kGemmThreads) {
    const int r = idx / k8n, k8 = idx - r * k8n;
    const int64_t m = m0 + r;
    uint2 out = make_uint2(0, 0);
    if (m < p.M && k8 < k8real) {
      float x[8];
      if (f32in) {
        const float* src = reinterpret_cast<const float*>(p.x) + m * p.ldx + k8 * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = src[e];
      } else {
        const __half* src = reinterpret_cast<const __half*>(p.x) + m * p.ldx + k8 * 8;
        if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
          const uint4 v = *reinterpret_cast<const uint4*>(src);
          const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = __half2float(h[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = __half2float(src[e]);
        }
      }
      uint32_t w[2] = {0, 0};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = k8 * 8 + e;
        w[e >> 2] |= (uint32_t)(aq.quant(x[e], kalpha[k], kbeta[k]) & 0xFF) << (8 * (e & 3));
      }
      out = make_uint2(w[0], w[1]);
    }
    *reinterpret_cast<uint2*>(As + (k8 >> 1) * 2048 + r * 16 + (k8 & 1) * 8) = out;
  }
  cp_async_wait_all();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (tid == 0) {
    const uint32_t ab = smem_u32(As), bb = smem_u32(Bs);
    constexpr uint32_t idesc = idesc_i8(128, NT);
    for (int kc = 0; kc < Kp / 32; ++kc) {
      const uint64_t ad = smem_desc(ab + kc * 2 * 2048, 2048, 128);
      const uint64_t bd = smem_desc(bb + kc * 2 * NT * 16, NT * 16, 128);
      mma_i8(tmem, ad, bd, idesc, kc > 0 ? 1u : 0u);
    }
    mma_commit(mbar);
  }
  const bool ok = mbar_wait_bounded(mbar, 0);
  if (!ok) *abort_flag = 1;
  tc_fence_after();
  __syncthreads();

  float zmax = 0.0f;
  if (!*abort_flag) {
    const int quarter = warp & 3, half = warp >> 2;
    const int64_t m = m0 + 32 * quarter + lane;
    const bool row_ok = m < p.M;
    ActQuant nq{};
    nq.let = p.next_let != 0;
    static_assert(NT % 32 == 0, "N tile must be a multiple of 32");
    constexpr int kHalfCols = NT / 2;
    constexpr int kChunks = kHalfCols / 16;
#pragma unroll 1
    for (int cb = 0; cb < kChunks; ++cb) {
      const int col0 = half * kHalfCols + cb * 16;     // first column of this chunk (tile-local)
      uint32_t rr[16];
      tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + col0, rr);
      tmem_ld_wait();
      __align__(16) __half h[16];
      float f[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int jj = col0 + j;
        f[j] = qlinear_out32((int32_t)rr[j], cscale[jj], cbias[jj]);
        h[j] = __float2half_rn(f[j]);
        if (p.elu) h[j] = elu16(h[j]);
        if (p.next_slot >= 0 && n0 + jj < N)
          zmax = fmaxf(zmax, nq.absz(__half2float(h[j]), calpha[jj], cbeta[jj]));
      }
      if (row_ok) {
        const int nb = n0 + col0;
        if (p.y) {
          __half* dst = p.y + m * p.ldy + nb;
          if (nb + 16 <= N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
            reinterpret_cast<uint4*>(dst)[0] = reinterpret_cast<const uint4*>(h)[0];
            reinterpret_cast<uint4*>(dst)[1] = reinterpret_cast<const uint4*>(h)[1];
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (nb + j < N) dst[j] = h[j];
          }
        }
        if (p.y32) {
          float* dst = p.y32 + m * p.ldy32 + nb;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (nb + j < N) dst[j] = p.y32_round16 ? __half2float(h[j]) : f[j];
        }
      }
    }
  }
  if (p.next_slot >= 0 && p.act_mode == GLAD_ACT_DYNAMIC) {
    const float mm = warp_max(zmax);
    if (lane == 0 && mm > 0.0f) atomic_max_nonneg(&p.slots[p.next_slot], mm);
  }
  if (*abort_flag) {
    mbar_wait_bounded(mbar, 0);
    if (tid == 0 && p.slots)
      atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrMmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

size_t qgemm_smem_bytes(int K, int NT) {
  const size_t Kp = (size_t)((K + 31) & ~31);
  return Kp * 128 + Kp * NT + 4 * NT * sizeof(float) + 2 * Kp * sizeof(float) + 64 + 128;
}

template <int NT>
cudaError_t launch_qgemm(const GemmParams& p, cudaStream_t st, bool pdl) {
  const size_t smem = qgemm_smem_bytes(p.L.in_features, NT);
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)qgemm_kernel<NT>, done);
  if (e != cudaSuccess) return e;
  const int Np = (p.L.out_features + 7) & ~7;
  dim3 grid((unsigned)((p.M + 127) / 128), (unsigned)((Np + NT - 1) / NT));
  return launch_k(qgemm_kernel<NT>, grid, dim3(kGemmThreads), smem, st, pdl, p);
}
template cudaError_t launch_qgemm<128>(const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_qgemm<64>(const GemmParams&, cudaStream_t, bool);
template cudaError_t launch_qgemm<32>(const GemmParams&, cudaStream_t, bool);


// ---- dynamic absmax of alpha*x + beta over [M, K] ---------------------------------------
// `round16`: the input is first rounded to fp16 (the .half() cast in front of
// the compiled actor, qrt/integration.py:206).
__global__ void absmax_kernel(const void* x, int dtype, int64_t M, int64_t ld, int K,
                              const float* alpha, const float* beta, int round16,
                              float* slot, const float* norm_mean, const float* norm_var, float norm_eps) {
  grid_dep_launch();
  ActQuant q{};
  q.let = alpha != nullptr;
  float m = 0.0f;
  // block = 256 threads = 8 rows x 32 lanes; lanes walk the row's K columns
  const int lane = threadIdx.x & 31, rw = threadIdx.x >> 5;
  for (int64_t r0 = (int64_t)blockIdx.x * 8; r0 < M; r0 += (int64_t)gridDim.x * 8) {
    const int64_t r = r0 + rw;
    if (r >= M) continue;
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = lane + 32 * u;
      v[u] = 0.0f;
      if (k < K)
        v[u] = dtype == GLAD_DTYPE_F32 ? reinterpret_cast<const float*>(x)[r * ld + k]
                                       : __half2float(reinterpret_cast<const __half*>(x)[r * ld + k]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = lane + 32 * u;
      if (k < K) {
        if (norm_mean) v[u] = obs_norm(v[u], norm_mean, norm_var, norm_eps, k);
        const float xv = round16 ? fp16r(v[u]) : v[u];
        m = fmaxf(m, q.absz(xv, q.let ? alpha[k] : 0.0f, q.let ? beta[k] : 0.0f));
      }
    }
    for (int k = lane + 128; k < K; k += 32) {     // rows wider than 128
      float xv = dtype == GLAD_DTYPE_F32 ? reinterpret_cast<const float*>(x)[r * ld + k]
                                         : __half2float(reinterpret_cast<const __half*>(x)[r * ld + k]);
      if (norm_mean) xv = obs_norm(xv, norm_mean, norm_var, norm_eps, k);
      if (round16) xv = fp16r(xv);
      m = fmaxf(m, q.absz(xv, q.let ? alpha[k] : 0.0f, q.let ? beta[k] : 0.0f));
    }
  }
  m = warp_max(m);
  if (lane == 0 && m > 0.0f) atomic_max_nonneg(slot, m);
}

cudaError_t launch_absmax(const void* x, int dtype, int64_t M, int64_t ld, int K,
                          const float* alpha, const float* beta, int round16, float* slot,
                          int num_sms, cudaStream_t st, const float* norm_mean, const float* norm_var,
                          float norm_eps) {
  int64_t blocks = (M + 7) / 8;
  if (blocks > 4LL * num_sms) blocks = 4LL * num_sms;
  if (blocks < 1) blocks = 1;
  absmax_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, dtype, M, ld, K, alpha, beta, round16, slot,
                                                  norm_mean, norm_var, norm_eps);
  return cudaGetLastError();
}

// Per-layer scales reported through GladActorAux::act_scales.
struct ScaleArgs {
  const float* s_z[6];
  int let[6];
};
__global__ void act_scales_kernel2(const float* slots, int act_mode, ScaleArgs a, float* out) {
  const int i = threadIdx.x;
  if (i < 6) out[i] = act_mode == GLAD_ACT_DYNAMIC ? dyn_scale(slots[i], a.let[i] != 0) : *a.s_z[i];
}
cudaError_t launch_act_scales(const float* slots, int act_mode, const float* const s_z[6],
                              const int let[6], float* out, cudaStream_t st) {
  ScaleArgs a;
  for (int i = 0; i < 6; ++i) {
    a.s_z[i] = s_z[i];
    a.let[i] = let[i];
  }
  act_scales_kernel2<<<1, 32, 0, st>>>(slots, act_mode, a, out);
  return cudaGetLastError();
}

// ---- QuantLinear.requantize_ (qrt/qlinear.py:84-102) ---------------------------------
// One warp per output row; blockIdx.y = layer.
constexpr int kMaxRequantLayers = 16;
struct RequantTable {
  GladQLinearSrc l[kMaxRequantLayers];
  int n;
};

__device__ __forceinline__ float load_w(const void* p, int dtype, int64_t i) {
  return dtype == GLAD_DTYPE_F32 ? reinterpret_cast<const float*>(p)[i]
                                 : __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__global__ void requant_qlinear_kernel(const __grid_constant__ RequantTable t) {
  const GladQLinearSrc& L = t.l[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * (blockDim.x >> 5) + warp;
  if (n >= L.N) return;
  const int K = L.K;
  float amax = 0.0f, bsum = 0.0f;
  for (int k = lane; k < K; k += 32) {
    float w = load_w(L.weight, L.w_dtype, (int64_t)n * K + k);
    if (L.alpha) w = __fdiv_rn(w, L.alpha[k]);
    amax = fmaxf(amax, fabsf(w));
    if (L.alpha && L.beta) bsum += __fmul_rn(w, L.beta[k]);
  }
  amax = warp_max(amax);
  bsum = warp_sum(bsum);
  const float s_w = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
  for (int k = lane; k < K; k += 32) {
    float w = load_w(L.weight, L.w_dtype, (int64_t)n * K + k);
    if (L.alpha) w = __fdiv_rn(w, L.alpha[k]);
    int q = __float2int_rn(__fdiv_rn(w, s_w));
    q = q < -128 ? -128 : (q > 127 ? 127 : q);
    L.w8[(int64_t)n * K + k] = (int8_t)q;
  }
  if (lane == 0) {
    const float b = L.bias ? load_w(L.bias, L.w_dtype, n) : 0.0f;
    L.dq_scale[n] = __fmul_rn(s_w, *L.s_z);
    L.s_w[n] = s_w;
    L.b_prime[n] = (L.alpha && L.beta) ? __fsub_rn(b, bsum) : b;
  }
}

cudaError_t launch_requant_qlinear(const GladQLinearSrc* layers, int n, cudaStream_t st) {
  RequantTable t;
  t.n = n;
  int maxN = 0;
  for (int i = 0; i < n; ++i) {
    t.l[i] = layers[i];
    if (layers[i].N > maxN) maxN = layers[i].N;
  }
  dim3 grid((unsigned)((maxN + 7) / 8), (unsigned)n);
  requant_qlinear_kernel<<<grid, 256, 0, st>>>(t);
  return cudaGetLastError();
}

// ---- QuantCNN.requantize_ (qrt/qconv.py:247-284), no LET -------------------------------
__global__ void requant_qcnn_kernel(const __grid_constant__ GladQCNNSrc s) {
  const int tid = threadIdx.x;
  const float sz = *s.s_z;
  const int dt = s.dtype;
  const bool h16 = dt == GLAD_DTYPE_F16;
  auto rd = [dt](const void* p, int i) { return load_w(p, dt, i); };
  // BN affine y = a*x + c evaluated in the parameters' dtype, then widened
  // (qrt/qconv.py:252-255).
  auto bn = [&](const void* w, const void* b, const void* mu, const void* var, float eps, int c,
                float& a, float& cc) {
    if (h16) {
      const float den = fp16r(sqrtf(fp16r(__fadd_rn(rd(var, c), eps))));
      a = fp16r(__fdiv_rn(rd(w, c), den));
    } else {
      a = __fdiv_rn(rd(w, c), sqrtf(__fadd_rn(rd(var, c), eps)));
    }
    cc = __fsub_rn(rd(b, c), __fmul_rn(a, rd(mu, c)));
  };
  if (tid < 16) {
    float a1, c1;
    bn(s.bn1_w, s.bn1_b, s.bn1_mean, s.bn1_var, s.eps1, tid, a1, c1);
    if (s.alpha) {                        // LET folded into BN1 (qrt/qconv.py:256-258)
      a1 = __fmul_rn(a1, s.alpha[tid]);
      c1 = __fadd_rn(__fmul_rn(c1, s.alpha[tid]), s.beta ? s.beta[tid] : 0.0f);
    }
    s.qa[tid] = __fdiv_rn(a1, sz);
    s.qc[tid] = __fdiv_rn(c1, sz);
    s.b1f[tid] = rd(s.conv1_b, tid);
  }
  // w1p [128,16]: k = kh*16 + kw*3 + c for kh<5, kw*3+c<15
  for (int idx = tid; idx < 128 * 16; idx += blockDim.x) {
    const int k = idx >> 4, n = idx & 15;
    const int kh = k >> 4, r = k & 15;
    float v = 0.0f;
    if (kh < 5 && r < 15) {
      const int kw = r / 3, c = r % 3;
      v = rd(s.conv1_w, ((n * 3 + c) * 5 + kh) * 5 + kw);
    }
    reinterpret_cast<__half*>(s.w1p)[idx] = __float2half_rn(v);
  }
  if (tid < 64) {
    const int n = tid;
    // conv2_w [64][16][3][3] -> W' = W/alpha per input channel (LET, qconv.py:271-272)
    auto w2 = [&](int c, int kh, int kw) {
      const float w = rd(s.conv2_w, ((n * 16 + c) * 3 + kh) * 3 + kw);
      return s.alpha ? __fdiv_rn(w, s.alpha[c]) : w;
    };
    float amax = 0.0f, bsum = 0.0f;
    for (int c = 0; c < 16; ++c)
      for (int kh = 0; kh < 3; ++kh)
        for (int kw = 0; kw < 3; ++kw) {
          const float w = w2(c, kh, kw);
          amax = fmaxf(amax, fabsf(w));
          if (s.alpha && s.beta) bsum += __fmul_rn(w, s.beta[c]);
        }
    const float s_w = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    // w8[kh][kw*16 + c][n]
    for (int kh = 0; kh < 3; ++kh)
      for (int ks = 0; ks < 64; ++ks) {
        int q = 0;
        if (ks < 48) {
          q = __float2int_rn(__fdiv_rn(w2(ks & 15, kh, ks >> 4), s_w));
          q = q < -128 ? -128 : (q > 127 ? 127 : q);
        }
        s.w8[(kh * 64 + ks) * 64 + n] = (int8_t)q;
      }
    s.dq[n] = __fmul_rn(s_w, sz);
    s.b2f[n] = __fsub_rn(rd(s.conv2_b, n), bsum);   // b' = b - sum W'*beta (qconv.py:280-281)
    float a2, c2;
    bn(s.bn2_w, s.bn2_b, s.bn2_mean, s.bn2_var, s.eps2, n, a2, c2);
    s.a2[n] = a2;
    s.c2[n] = c2;
  }
}

cudaError_t launch_requant_qcnn(const GladQCNNSrc& s, cudaStream_t st) {
  requant_qcnn_kernel<<<1, 256, 0, st>>>(s);
  return cudaGetLastError();
}

// ---- batched cast-copy (qrt/runtime.py:251-253) ----------------------------------------
constexpr int kMaxCast = 96;
struct CastTable {
  GladCastCopy it[kMaxCast];
};
__global__ void cast_copy_kernel(const __grid_constant__ CastTable t) {
  const GladCastCopy& c = t.it[blockIdx.y];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < c.n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = c.src_dtype == GLAD_DTYPE_F32 ? reinterpret_cast<const float*>(c.src)[i]
                                                  : __half2float(reinterpret_cast<const __half*>(c.src)[i]);
    if (c.dst_dtype == GLAD_DTYPE_F32)
      reinterpret_cast<float*>(c.dst)[i] = v;
    else
      reinterpret_cast<__half*>(c.dst)[i] = __float2half_rn(v);
  }
}

cudaError_t launch_cast_copy(const GladCastCopy* items, int n, cudaStream_t st) {
  for (int b = 0; b < n; b += kMaxCast) {
    CastTable t;
    const int cnt = (n - b) < kMaxCast ? (n - b) : kMaxCast;
    int64_t maxn = 1;
    for (int i = 0; i < cnt; ++i) {
      t.it[i] = items[b + i];
      if (items[b + i].n > maxn) maxn = items[b + i].n;
    }
    int64_t blocks = (maxn + 255) / 256;
    if (blocks > 256) blocks = 256;
    cast_copy_kernel<<<dim3((unsigned)blocks, (unsigned)cnt), 256, 0, st>>>(t);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace glad
