// Fused actor MLP: the four W8A8 QuantLinear layers of the actor head
// 224 -> 512 -> 256 -> 128 -> 29 with ELU between them (rsl_rl/networks/mlp.py:
// 59-83, each layer qrt/qlinear.py:111-138) in ONE kernel.
//
// Rows are cut into 128-row tiles. A tile belongs to a cluster of four CTAs
// that split each hidden layer's output columns (512/256/128 -> 128/64/32 per
// CTA); the 29-wide head runs on cluster rank 0. A CTA's epilogue turns its
// accumulator columns into fp16 ELU activations held in registers. With a
// dynamic s_z the absmax of the next layer's input over the WHOLE batch must be
// known before anything can be quantised (qrt/qlinear.py:126-128), so every CTA
// adds its part with an atomic max and all CTAs meet at a grid-wide barrier
// (arrival counter, bounded spin). Each CTA then quantises its columns and
// stores the int8 slice directly into the A operand of all four CTAs of its
// cluster (distributed shared memory). Hidden activations never leave the SM.
//
// The grid barrier needs every CTA resident at once: the host launches this
// kernel only when the device's cluster occupancy admits the whole grid (one
// CTA per SM) and otherwise runs the per-layer GEMM kernels. Spins give up
// after 2 s, set a status bit and let the kernel finish.
#include <cuda_runtime.h>

#include <type_traits>

#include "glad_common.cuh"

namespace glad {

constexpr int kMlpCluster = 4;
constexpr int kMlpThreads = 512;                 // 16 warps: 4 per TMEM lane quarter

// shared memory (bytes)
constexpr int kOffA0 = 0;                        // A of layers 0 and 2: [K/16][128 rows][16 B], K <= 256
constexpr int kOffA1 = kOffA0 + 128 * 256;       // A of layers 1 and 3: K <= 512
constexpr int kOffW0 = kOffA1 + 128 * 512;       // B slices [K/16][rows][16 B]: 128x224
constexpr int kOffW1 = kOffW0 + 128 * 224;       //   64x512
constexpr int kOffW2 = kOffW1 + 64 * 512;        //   32x256
constexpr int kOffW3 = kOffW2 + 32 * 256;        //   32x128 (head, rank 0)
constexpr int kOffH = kOffW3 + 32 * 128;         // fp16 activations [16-col chunk][2][128 rows][8 halves]
constexpr int kOffF = kOffH + 128 * 128 * 2;     // float constants
constexpr int kFInA = 0;                         // [224] LET alpha / beta of layer 0's input
constexpr int kFInB = 224;
constexpr int kFSw = 448;                        // [256] s_w (dynamic) or dq_scale (static), own columns
constexpr int kFBp = 704;                        // [256] b_prime
constexpr int kFNa = 960;                        // [224] LET alpha / beta of the next layer, own columns
constexpr int kFNb = 1184;
constexpr int kFSc = 1408;                       // [256] output scale of the running layer
constexpr int kFCount = 1664;
constexpr int kOffBar = kOffF + kFCount * 4;        // mbarrier, TMEM slot, abort flag
constexpr int kOffRed = kOffBar + 64;                // per-warp maxima [16]
constexpr int kMlpSmem = kOffRed + 64;
// Each layer's K is split over kMlpChains partial accumulators issued by warps 0-3 in
// parallel (an MMA issue costs ~140 cycles per warp); the int32 partial sums are added
// exactly in the epilogue. Chain c occupies TMEM columns [c*N, (c+1)*N); every layer
// has at least four 32-wide K steps, so every chain is written.
constexpr int kMlpChains = 4;
constexpr uint32_t kMlpTmemCols = 512;
static_assert(kMlpSmem + 128 <= 227 * 1024, "shared memory");

// per-layer shape: K, own output columns, column base into the per-column tables
__host__ __device__ constexpr int mlp_k(int l) { return l == 0 ? 224 : l == 1 ? 512 : l == 2 ? 256 : 128; }
__host__ __device__ constexpr int mlp_n(int l) { return l == 0 ? 512 : l == 1 ? 256 : l == 2 ? 128 : kActions; }
__host__ __device__ constexpr int mlp_nj(int l) { return l == 0 ? 128 : l == 1 ? 64 : 32; }
__host__ __device__ constexpr int mlp_cb(int l) { return l == 0 ? 0 : l == 1 ? 128 : l == 2 ? 192 : 224; }
__host__ __device__ constexpr int mlp_abuf(int l) { return (l & 1) ? kOffA1 : kOffA0; }
__host__ __device__ constexpr int mlp_wbuf(int l) {
  return l == 0 ? kOffW0 : l == 1 ? kOffW1 : l == 2 ? kOffW2 : kOffW3;
}

struct MlpParams {
  GladQLinear L[4];
  int act_mode;
  const __half* x;         // encoded [M, ldx] fp16
  int64_t M, ldx;
  float* mean;             // [M, ldm] = float(fp16(head output))
  int64_t ldm;
  float* slots;            // absmax slots 2..5, status, barrier counters
  uint32_t barrier_extra;  // arrivals the grid barriers wait for beyond the grid (0; tests only)
  uint64_t barrier_limit_ns;   // spin limit of the grid barriers
};

// Failure-path test hook (glad_debug_mlp_barrier): process-wide, read at launch.
static uint32_t g_mlp_barrier_extra = 0;
static uint64_t g_mlp_barrier_limit_ns = 0;
constexpr uint64_t kMlpBarrierLimitNs = 2000000000ull;

// Rows [n0, n0+ROWS) of a row-major int8 [*, K] weight -> [K/16][ROWS][16 B] (compile-time
// shapes: the index split is a shift).
template <int K, int ROWS>
__device__ __forceinline__ void mlp_load_w(uint8_t* dst, const int8_t* w8, int n0, int tid) {
  constexpr int n16 = ROWS * (K / 16);
#pragma unroll 1
  for (int idx = tid; idx < n16; idx += kMlpThreads) {
    const int c = idx / ROWS, n = idx % ROWS;
    cp_async16(dst + idx * 16, w8 + (int64_t)(n0 + n) * K + c * 16);
  }
}

// 16 fp16 values -> 16 int8 (one uint4) with per-column LET constants. For the dynamic
// LET scale (the common case) the fast quotient of all 16 values is rounded first and
// the exact path of ActQuant::qbits runs only when one of them lies near a rounding
// boundary (one test per 16 values instead of one branch per value).
__device__ __forceinline__ uint4 mlp_quant16(const uint4 v0, const uint4 v1, const ActQuant& aq,
                                             const float* a, const float* b) {
  const uint32_t h[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  float x[16], al[16], be[16];
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    const float4 a4 = *reinterpret_cast<const float4*>(a + j);
    const float4 b4 = *reinterpret_cast<const float4*>(b + j);
    const float2 x01 = __half22float2(*reinterpret_cast<const __half2*>(&h[j >> 1]));
    const float2 x23 = __half22float2(*reinterpret_cast<const __half2*>(&h[(j >> 1) + 1]));
    x[j] = x01.x, x[j + 1] = x01.y, x[j + 2] = x23.x, x[j + 3] = x23.y;
    al[j] = a4.x, al[j + 1] = a4.y, al[j + 2] = a4.z, al[j + 3] = a4.w;
    be[j] = b4.x, be[j + 1] = b4.y, be[j + 2] = b4.z, be[j + 3] = b4.w;
  }
  uint32_t q[16];
  bool near = true;
  if (aq.let && aq.dyn) {
    constexpr float kMagic = 12582912.0f;
    near = false;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float z = __fadd_rn(__fmul_rn(x[j], al[j]), be[j]);
      const float t = fminf(fmaxf(__fmul_rn(z, aq.rcp), -128.0f), 127.0f);
      const float u = __fadd_rn(t, kMagic);
      near |= fabsf(__fsub_rn(t, __fsub_rn(u, kMagic))) >= 0.4999f;
      q[j] = __float_as_uint(u);
    }
  }
  if (near) {
#pragma unroll
    for (int j = 0; j < 16; ++j) q[j] = aq.qbits(x[j], al[j], be[j]);
  }
  // low bytes of q -> four words (byte permutes instead of masks and shifts)
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    w[j] = __byte_perm(__byte_perm(q[4 * j], q[4 * j + 1], 0x0040), __byte_perm(q[4 * j + 2], q[4 * j + 3], 0x0040),
                       0x5410);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void mlp_mma(uint8_t* sm, uint32_t tmem, uint64_t* mbar, uint32_t& phase,
                                        int* abort_flag, bool& mma_timeout, int abuf, int wbuf, int K,
                                        uint32_t idesc, int nj) {
  const int w = threadIdx.x >> 5;
  if (w < kMlpChains) {
    // chain w: K steps w, w + 4, ... into columns [w*nj, (w+1)*nj), from one elected lane
    tc_fence_after();
    const uint32_t ab = smem_u32(sm + abuf), bb = smem_u32(sm + wbuf);
    for (int kc = w; kc < K / 32; kc += kMlpChains) {
      const uint64_t ad = smem_desc(ab + kc * 2 * 2048, 2048, 128);
      const uint64_t bd = smem_desc(bb + kc * 2 * nj * 16, nj * 16, 128);
      mma_i8_warp(tmem + (uint32_t)(w * nj), ad, bd, idesc, kc >= kMlpChains ? 1u : 0u);
    }
    mma_commit_warp(mbar);
  }
  if (!mbar_wait_bounded(mbar, phase)) {
    *abort_flag = 1;
    mma_timeout = true;
  }
  phase ^= 1;
  tc_fence_after();
  __syncthreads();
}

// 16 accumulator columns at `taddr`: the sum of the kMlpChains partial chains (int32,
// exact), chain c at column offset c * nj; all chains' loads are in flight before one wait.
template <int W>
__device__ __forceinline__ void mlp_ld_acc(uint32_t taddr, int nj, uint32_t (&r)[W]) {
  static_assert(W == 8 || W == 16, "8 or 16 columns");
  uint32_t t[kMlpChains - 1][W];
  if constexpr (W == 16) {
    tmem_ld16(taddr, r);
#pragma unroll
    for (int c = 1; c < kMlpChains; ++c) tmem_ld16(taddr + (uint32_t)(c * nj), t[c - 1]);
  } else {
    tmem_ld8(taddr, r);
#pragma unroll
    for (int c = 1; c < kMlpChains; ++c) tmem_ld8(taddr + (uint32_t)(c * nj), t[c - 1]);
  }
  tmem_ld_wait();
#pragma unroll
  for (int c = 1; c < kMlpChains; ++c)
#pragma unroll
    for (int j = 0; j < W; ++j) r[j] += t[c - 1][j];
}

// 16 int32 accumulators -> fp32, exactly: through the mantissa of 1.5*2^23 (two ALU
// operations) when every |acc| < 2^22, which the OR of the offset values shows, else
// by the conversion instruction.
template <int W>
__device__ __forceinline__ void mlp_acc_f32(const uint32_t (&r)[W], float (&a)[W]) {
  uint32_t span = 0;
#pragma unroll
  for (int j = 0; j < W; ++j) span |= r[j] + (1u << 22);
  if (span < (1u << 23)) {
#pragma unroll
    for (int j = 0; j < W; ++j) a[j] = i2f_small((int32_t)r[j]);
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j) a[j] = (float)(int32_t)r[j];
  }
}

// ELU of two fp16 values (each computed in fp32 and rounded to fp16, as elu16).
__device__ __forceinline__ __half2 elu16x2(__half2 h) {
  const float2 x = __half22float2(h);
  return __floats2half2_rn(x.x > 0.0f ? x.x : expm1f(x.x), x.y > 0.0f ? x.y : expm1f(x.y));
}

// Grid-wide barrier on counter `ctr` (one arrival per CTA), folded with the batch
// absmax: the CTA's warps leave their maxima in `red`, thread 0 adds one atomic max
// to `slot`, arrives with a release add and spins with acquire loads. The spin gives
// up after limit_ns (2 s; status bit, abort flag); an aborted CTA still arrives.
__device__ __forceinline__ void mlp_grid_barrier(int* abort_flag, float* red, float* slot, uint32_t* ctr,
                                                 uint32_t expected, uint32_t* status, uint64_t limit_ns) {
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < kMlpThreads / 32; ++w) m = fmaxf(m, red[w]);
    if (m > 0.0f) atomic_max_nonneg(slot, m);
    red_release_add(ctr, 1u);
    if (!*abort_flag) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_gpu(ctr) < expected) {
        if (global_timer_ns() - t0 > limit_ns) {
          *abort_flag = 1;
          atomicOr(status, kDevErrBarrierTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kMlpThreads, 1) mlp_kernel(const __grid_constant__ MlpParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  float* F = reinterpret_cast<float*>(sm + kOffF);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(sm + kOffBar + 12);
  float* red = reinterpret_cast<float*>(sm + kOffRed);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, part = warp >> 2;   // TMEM lane quarter, column-chunk phase
  const int row = 32 * quarter + lane;              // tile row of this thread in the epilogues
  const uint32_t rank = cluster_ctarank();
  const int64_t m0 = (int64_t)(blockIdx.x / kMlpCluster) * 128;
  const int64_t m = m0 + row;
  const bool row_ok = m < p.M;
  const bool dyn = p.act_mode == GLAD_ACT_DYNAMIC;
  uint32_t* status = reinterpret_cast<uint32_t*>(&p.slots[kSlotStatus]);
  uint32_t phase = 0;
  bool mma_timeout = false;

  if (warp == 0) tmem_alloc(tmem_slot, kMlpTmemCols);
  if (tid == 0) {
    mbar_init(mbar, kMlpChains);
    fence_mbar_init();
    *abort_flag = 0;
  }

  // per-column constants, copied asynchronously with the weights
  for (int k = tid; k < 224; k += kMlpThreads) {
    if (p.L[0].alpha) {
      cp_async4(&F[kFInA + k], p.L[0].alpha + k);
      cp_async4(&F[kFInB + k], p.L[0].beta + k);
    } else {
      F[kFInA + k] = 0.0f;
      F[kFInB + k] = 0.0f;
    }
  }
  for (int l = 0; l < 4; ++l) {
    const GladQLinear& L = p.L[l];
    const int nj = mlp_nj(l), n0 = l < 3 ? (int)rank * nj : 0;
    for (int j = tid; j < nj; j += kMlpThreads) {
      const int n = n0 + j;
      if (n < mlp_n(l)) {
        cp_async4(&F[kFSw + mlp_cb(l) + j], (dyn ? L.s_w : L.dq_scale) + n);
        cp_async4(&F[kFBp + mlp_cb(l) + j], L.b_prime + n);
      } else {
        F[kFSw + mlp_cb(l) + j] = 0.0f;
        F[kFBp + mlp_cb(l) + j] = 0.0f;
      }
      if (l < 3) {
        const GladQLinear& Ln = p.L[l + 1];
        if (Ln.alpha) {
          cp_async4(&F[kFNa + mlp_cb(l) + j], Ln.alpha + n);
          cp_async4(&F[kFNb + mlp_cb(l) + j], Ln.beta + n);
        } else {
          F[kFNa + mlp_cb(l) + j] = 0.0f;
          F[kFNb + mlp_cb(l) + j] = 0.0f;
        }
      }
    }
  }
  cp_async_commit();
  // weight slices of all four layers, in flight while the input is quantised; layer 0's
  // are a group of their own, so its MMA waits for those alone
  mlp_load_w<224, 128>(sm + kOffW0, p.L[0].w8, (int)rank * 128, tid);
  cp_async_commit();
  mlp_load_w<512, 64>(sm + kOffW1, p.L[1].w8, (int)rank * 64, tid);
  mlp_load_w<256, 32>(sm + kOffW2, p.L[2].w8, (int)rank * 32, tid);
  if (rank == 0) mlp_load_w<128, 32>(sm + kOffW3, p.L[3].w8, 0, tid);
  cp_async_commit();
  grid_dep_wait();                      // encoded rows and slot 2 of the preceding kernel
  // this thread's item of the layer-0 input (rank j quantises tile rows [32j, 32j+32), 14
  // chunks of 16 columns each; warp k takes chunk k of the 32 rows, so that its constants are
  // one broadcast and its stores fill consecutive rows), loaded before the waits below so
  // that its latency overlaps them
  static_assert(32 * 14 <= kMlpThreads, "one input item per thread");
  const int in_rr = 32 * (int)rank + lane, in_kc = warp;
  const bool in_ok = tid < 32 * 14 && m0 + in_rr < p.M;
  uint4 in0 = make_uint4(0, 0, 0, 0), in1 = in0;
  if (in_ok) {
    const uint4* src = reinterpret_cast<const uint4*>(p.x + (m0 + in_rr) * p.ldx + in_kc * 16);
    in0 = src[0];
    in1 = src[1];
  }
  ActQuant aq = make_act_quant(p.L[0], p.act_mode, p.slots, 2);   // input of the running layer
  cp_async_wait_group<2>();             // constants landed; the weights may still be in flight
  __syncthreads();
  tc_fence_before();
  cluster_sync_all();                            // every CTA of the cluster runs before DSMEM stores
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;

  // ---- layer 0 input: rank j quantises tile rows [32j, 32j+32) for the whole cluster ------
  if (tid < 32 * 14) {
    uint4 q = make_uint4(0, 0, 0, 0);
    if (in_ok) q = mlp_quant16(in0, in1, aq, &F[kFInA + in_kc * 16], &F[kFInB + in_kc * 16]);
    const uint32_t off = smem_u32(sm + kOffA0) + in_kc * 2048 + in_rr * 16;
#pragma unroll
    for (int r = 0; r < kMlpCluster; ++r) st_cluster_v4(mapa_shared(off, r), q);
  }
  cp_async_wait_group<1>();             // layer 0's weight slice (the later layers' may still land)
  fence_async_smem();
  fence_async_cluster();
  cluster_sync_all();

  // ---- hidden layers: MMA, epilogue to fp16 ELU (shared memory), absmax, grid barrier,
  //      quantise own columns into every cluster CTA's next A operand --------------------------
  uint4* H = reinterpret_cast<uint4*>(sm + kOffH);
#pragma unroll 1
  for (int l = 0; l < 3; ++l) {
    const int NJ = mlp_nj(l), CB = mlp_cb(l), nch = NJ / 16;
    for (int j = tid; j < NJ; j += kMlpThreads)
      F[kFSc + CB + j] = dyn ? __fmul_rn(F[kFSw + CB + j], aq.s) : F[kFSw + CB + j];
    if (!*abort_flag)
      mlp_mma(sm, tmem, mbar, phase, abort_flag, mma_timeout, mlp_abuf(l), mlp_wbuf(l), mlp_k(l),
              l == 0 ? idesc_i8(128, 128) : l == 1 ? idesc_i8(128, 64) : idesc_i8(128, 32), NJ);
    const GladQLinear& Ln = p.L[l + 1];
    const bool nlet = Ln.alpha != nullptr;
    const bool want_max = dyn && row_ok;
    float zmax = 0.0f;
    if (!*abort_flag) {
#pragma unroll 1
      // work units of 16 columns; a layer with only two 16-column chunks (actor.4) is cut
      // into 8-column halves so that all four warps of each lane quarter take part
      auto unit = [&](auto wc, int c0) {
        constexpr int W = decltype(wc)::value;
        uint32_t r[W];
        mlp_ld_acc<W>(tmem + lane_base + c0, NJ, r);
        float a[W];
        mlp_acc_f32<W>(r, a);
        uint32_t h[W / 2];
#pragma unroll
        for (int j = 0; j < W; j += 4) {
          const int c = CB + c0 + j;
          const float4 sc = *reinterpret_cast<const float4*>(&F[kFSc + c]);
          const float4 bp = *reinterpret_cast<const float4*>(&F[kFBp + c]);
          // y = fp16(acc*scale + b') (qlinear_out32), then ELU in fp32 rounded to fp16
          const __half2 p01 = elu16x2(__floats2half2_rn(__fadd_rn(__fmul_rn(a[j], sc.x), bp.x),
                                                        __fadd_rn(__fmul_rn(a[j + 1], sc.y), bp.y)));
          const __half2 p23 = elu16x2(__floats2half2_rn(__fadd_rn(__fmul_rn(a[j + 2], sc.z), bp.z),
                                                        __fadd_rn(__fmul_rn(a[j + 3], sc.w), bp.w)));
          h[j >> 1] = *reinterpret_cast<const uint32_t*>(&p01);
          h[(j >> 1) + 1] = *reinterpret_cast<const uint32_t*>(&p23);
          if (want_max) {
            const float2 f01 = __half22float2(p01), f23 = __half22float2(p23);
            if (nlet) {
              const float4 na = *reinterpret_cast<const float4*>(&F[kFNa + c]);
              const float4 nb = *reinterpret_cast<const float4*>(&F[kFNb + c]);
              zmax = fmaxf(zmax, fabsf(__fadd_rn(__fmul_rn(f01.x, na.x), nb.x)));
              zmax = fmaxf(zmax, fabsf(__fadd_rn(__fmul_rn(f01.y, na.y), nb.y)));
              zmax = fmaxf(zmax, fabsf(__fadd_rn(__fmul_rn(f23.x, na.z), nb.z)));
              zmax = fmaxf(zmax, fabsf(__fadd_rn(__fmul_rn(f23.y, na.w), nb.w)));
            } else {
              zmax = fmaxf(fmaxf(zmax, fmaxf(fabsf(f01.x), fabsf(f01.y))), fmaxf(fabsf(f23.x), fabsf(f23.y)));
            }
          }
        }
        // H: [16-column chunk][8-column half][128 rows][8 halves]; c0 / 8 indexes the halves
#pragma unroll
        for (int u = 0; u < W / 8; ++u)
          H[(c0 / 8 + u) * 128 + row] = make_uint4(h[4 * u], h[4 * u + 1], h[4 * u + 2], h[4 * u + 3]);
      };
      if (nch >= 4) {
#pragma unroll 1
        for (int ch = part; ch < nch; ch += 4) unit(std::integral_constant<int, 16>{}, ch * 16);
      } else {
#pragma unroll 1
        for (int u8 = part; u8 < 2 * nch; u8 += 4) unit(std::integral_constant<int, 8>{}, u8 * 8);
      }
    }
    tc_fence_before();
    if (dyn) {
      zmax = warp_max(zmax);
      if (lane == 0) red[warp] = zmax;
      mlp_grid_barrier(abort_flag, red, &p.slots[3 + l],
                       reinterpret_cast<uint32_t*>(&p.slots[kSlotMlpBarrier + l]), gridDim.x + p.barrier_extra, status,
                       p.barrier_limit_ns);
      aq.let = nlet;
      aq.dyn = true;
      aq.s = dyn_scale(ld_relaxed_gpu(&p.slots[3 + l]), nlet);
      aq.rcp = __fdiv_rn(1.0f, aq.s);
      aq.inv = 0.0f;
    } else {
      __syncthreads();
      aq = make_act_quant(Ln, GLAD_ACT_STATIC, p.slots, 0);
    }
    if (!*abort_flag) {
      const uint32_t abase = smem_u32(sm + mlp_abuf(l + 1));
      const int kc0 = (int)rank * nch;             // first K chunk of the next layer owned here
#pragma unroll 1
      for (int it = tid; it < nch * 128; it += kMlpThreads) {
        const int ch = it >> 7, rr = it & 127;
        const uint4 q = mlp_quant16(H[(ch * 2) * 128 + rr], H[(ch * 2 + 1) * 128 + rr], aq,
                                    &F[kFNa + CB + ch * 16], &F[kFNb + CB + ch * 16]);
        const uint32_t off = abase + (kc0 + ch) * 2048 + rr * 16;
#pragma unroll
        for (int r = 0; r < kMlpCluster; ++r) st_cluster_v4(mapa_shared(off, r), q);
      }
    }
    if (l == 0) {                          // the later layers' weight slices, before layer 1's MMA
      cp_async_wait_all();
      fence_async_smem();
    }
    fence_async_cluster();
    cluster_sync_all();
  }

  // ---- head (rank 0): 128 x 32 (29 real) outputs, mean = float(fp16(y)) (qrt/integration.py:206)
  if (rank == 0 && !*abort_flag) {
    constexpr int CB = mlp_cb(3);
    if (tid < 32) F[kFSc + CB + tid] = dyn ? __fmul_rn(F[kFSw + CB + tid], aq.s) : F[kFSw + CB + tid];
    mlp_mma(sm, tmem, mbar, phase, abort_flag, mma_timeout, mlp_abuf(3), mlp_wbuf(3), 128,
            idesc_i8(128, 32), 32);
    // staged in layer 2's A operand (dead: its MMA completed, no remote stores follow)
    // and written row-contiguous by all threads
    float* stage = reinterpret_cast<float*>(sm + kOffA0);   // [128 rows][33]
    const bool ok = !*abort_flag;                            // uniform after mlp_mma's barrier
    if (ok && part < 2) {
      const int col0 = part * 16;
      uint32_t r[16];
      mlp_ld_acc(tmem + lane_base + col0, 32, r);
      float a[16];
      mlp_acc_f32(r, a);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = col0 + j;
        if (n < kActions)
          stage[row * 33 + n] =
              __half2float(__float2half_rn(__fadd_rn(__fmul_rn(a[j], F[kFSc + CB + n]), F[kFBp + CB + n])));
      }
    }
    __syncthreads();
    if (ok) {
      const int rows = (int)(p.M - m0 < 128 ? p.M - m0 : 128);
      for (int i = tid; i < rows * kActions; i += kMlpThreads) {
        const int rr = i / kActions, c = i - rr * kActions;
        p.mean[(m0 + rr) * p.ldm + c] = stage[rr * 33 + c];
      }
    }
  }

  // ---- teardown ----------------------------------------------------------------------------
  if (mma_timeout) {
    mbar_wait_bounded(mbar, phase ^ 1);          // the MMA still in flight gets one more bounded wait
    atomicOr(status, kDevErrMmaTimeout);
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kMlpTmemCols);
  }
}

// Largest number of 4-CTA clusters of this kernel resident at once (cached per device).
static int mlp_max_clusters(cudaStream_t st) {
  static int cached[64];
  static bool have[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (have[dev]) return cached[dev];
  static bool done[64] = {false};
  if (allow_max_smem((const void*)mlp_kernel, done) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kMlpCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(kMlpCluster);
  cfg.blockDim = dim3(kMlpThreads);
  cfg.dynamicSmemBytes = kMlpSmem + 128;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (const void*)mlp_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cached[dev] = n;
  have[dev] = true;
  return n;
}

// Number of 128-row tiles the fused MLP can take in one launch (0: not usable).
int mlp_max_tiles(int act_mode, cudaStream_t st) {
  const int n = mlp_max_clusters(st);
  if (n <= 0) return 0;
  return act_mode == GLAD_ACT_DYNAMIC ? n : (1 << 30);
}

cudaError_t launch_mlp(const GladQLinear (&L)[4], int act_mode, const __half* x, int64_t M, int64_t ldx,
                       float* mean, int64_t ldm, float* slots, cudaStream_t st, bool pdl) {
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)mlp_kernel, done);
  if (e != cudaSuccess) return e;
  MlpParams p{};
  for (int i = 0; i < 4; ++i) p.L[i] = L[i];
  p.act_mode = act_mode;
  p.x = x;
  p.M = M;
  p.ldx = ldx;
  p.mean = mean;
  p.ldm = ldm;
  p.slots = slots;
  p.barrier_extra = g_mlp_barrier_extra;
  p.barrier_limit_ns = g_mlp_barrier_limit_ns ? g_mlp_barrier_limit_ns : kMlpBarrierLimitNs;
  const int tiles = (int)((M + 127) / 128);
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kMlpCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(tiles * kMlpCluster));
  cfg.blockDim = dim3(kMlpThreads);
  cfg.dynamicSmemBytes = kMlpSmem + 128;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, mlp_kernel, p);
}

}  // namespace glad

namespace glad {
int set_last_error(int code, const char* msg);   // glad_abi.cu
}

extern "C" int glad_debug_mlp_barrier(uint32_t extra_arrivals, uint64_t limit_ns) {
  if (extra_arrivals > 1024) return glad::set_last_error(GLAD_ERR_INVALID_ARG, "extra_arrivals above 1024");
  glad::g_mlp_barrier_extra = extra_arrivals;
  glad::g_mlp_barrier_limit_ns = limit_ns;
  return GLAD_OK;
}
