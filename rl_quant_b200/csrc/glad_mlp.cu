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

#include "glad_common.cuh"

namespace glad {

constexpr int kMlpCluster = 4;
constexpr int kMlpThreads = 256;
constexpr int kSlotBarrier = 16;                 // slots[16..18]: grid-barrier arrival counters

// shared memory (bytes)
constexpr int kOffA0 = 0;                        // A of layers 0 and 2: [K/16][128 rows][16 B], K <= 256
constexpr int kOffA1 = kOffA0 + 128 * 256;       // A of layers 1 and 3: K <= 512
constexpr int kOffW0 = kOffA1 + 128 * 512;       // B slices [K/16][rows][16 B]: 128x224
constexpr int kOffW1 = kOffW0 + 128 * 224;       //   64x512
constexpr int kOffW2 = kOffW1 + 64 * 512;        //   32x256
constexpr int kOffW3 = kOffW2 + 32 * 256;        //   32x128 (head, rank 0)
constexpr int kOffF = kOffW3 + 32 * 128;         // float constants
constexpr int kFInA = 0;                         // [224] LET alpha / beta of layer 0's input
constexpr int kFInB = 224;
constexpr int kFSc = 448;                        // [256] s_w (dynamic) or dq_scale (static) per own column
constexpr int kFBp = 704;                        // [256] b_prime
constexpr int kFNa = 960;                        // [224] LET alpha / beta of the next layer, own columns
constexpr int kFNb = 1184;
constexpr int kFCount = 1408;
constexpr int kOffBar = kOffF + kFCount * 4;
constexpr int kMlpSmem = kOffBar + 64;
constexpr uint32_t kMlpTmemCols = 128;

// per-layer shape: K, own output columns, column base into the kFSc/kFBp/kFNa tables
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
};

// Rows [n0, n0+rows) of a row-major int8 [*, K] weight -> [K/16][rows][16 B].
__device__ __forceinline__ void mlp_load_w(uint8_t* dst, const int8_t* w8, int K, int n0, int rows,
                                           int tid) {
  const int n16 = rows * (K / 16);
  for (int idx = tid; idx < n16; idx += kMlpThreads) {
    const int c = idx / rows, n = idx - c * rows;
    cp_async16(dst + c * rows * 16 + n * 16, w8 + (int64_t)(n0 + n) * K + c * 16);
  }
}

// 16 fp16 values (two uint4) -> 16 int8 (one uint4) with per-column LET constants.
__device__ __forceinline__ uint4 mlp_quant16(const uint32_t (&h)[8], const ActQuant& aq, const float* a,
                                             const float* b) {
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const __half2 h2 = *reinterpret_cast<const __half2*>(&h[j >> 1]);
    const float x = (j & 1) ? __high2float(h2) : __low2float(h2);
    const int q = aq.quant(x, a[j], b[j]);
    w[j >> 2] |= (uint32_t)(q & 0xFF) << (8 * (j & 3));
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

struct MlpCtx {
  uint8_t* sm;
  float* F;
  uint64_t* mbar;
  int* abort_flag;
  uint32_t tmem;
  uint32_t rank;
  int tid, warp, lane, quarter, half, row;
  int64_t m;
  bool row_ok, dyn;
  bool mma_timeout;        // this thread's last MMA wait ran out (the MMA may still be in flight)
  uint32_t phase;
};

__device__ __forceinline__ void mlp_mma(MlpCtx& c, int abuf, int wbuf, int K, uint32_t idesc, int nj) {
  if (c.tid == 0) {
    tc_fence_after();
    const uint32_t ab = smem_u32(c.sm + abuf), bb = smem_u32(c.sm + wbuf);
    for (int kc = 0; kc < K / 32; ++kc) {
      const uint64_t ad = smem_desc(ab + kc * 2 * 2048, 2048, 128);
      const uint64_t bd = smem_desc(bb + kc * 2 * nj * 16, nj * 16, 128);
      mma_i8(c.tmem, ad, bd, idesc, kc > 0 ? 1u : 0u);
    }
    mma_commit(c.mbar);
  }
  if (!mbar_wait_bounded(c.mbar, c.phase)) {
    *c.abort_flag = 1;
    c.mma_timeout = true;
  }
  c.phase ^= 1;
  tc_fence_after();
  __syncthreads();
}

// Grid-wide barrier on counter `ctr` (one arrival per CTA). The spin gives up
// after 2 s (status bit, abort flag); an aborted CTA still arrives.
__device__ __forceinline__ void mlp_grid_barrier(MlpCtx& c, uint32_t* ctr, uint32_t expected,
                                                 uint32_t* status) {
  __syncthreads();
  if (c.tid == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    if (!*c.abort_flag) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_gpu(ctr) < expected) {
        if (global_timer_ns() - t0 > 2000000000ull) {
          *c.abort_flag = 1;
          atomicOr(status, kDevErrBarrierTimeout);
          break;
        }
        __nanosleep(100);
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// Hidden layer l: MMA, epilogue (scale, bias, fp16, ELU), dynamic absmax of the
// next layer's input, grid barrier, quantise own columns into every cluster
// CTA's next A operand.
template <int l>
__device__ __forceinline__ void mlp_hidden(MlpCtx& c, const MlpParams& p, const ActQuant& aq,
                                           ActQuant& aqn, uint32_t* status) {
  constexpr int K = mlp_k(l), NJ = mlp_nj(l), CB = mlp_cb(l);
  constexpr int kChunks = NJ / 32;               // 16-column chunks per thread (two column halves)
  const bool run = !*c.abort_flag;
  if (run) mlp_mma(c, mlp_abuf(l), mlp_wbuf(l), K, idesc_i8(128, NJ), NJ);
  const bool ok = !*c.abort_flag;
  const GladQLinear& Ln = p.L[l + 1];
  const bool nlet = Ln.alpha != nullptr;
  uint32_t hv[kChunks][8];
  float zmax = 0.0f;
  if (ok) {
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int col0 = c.half * (NJ / 2) + ch * 16;
      uint32_t r[16];
      tmem_ld16(c.tmem + ((uint32_t)(32 * c.quarter) << 16) + col0, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        __half h2v[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int lc = col0 + j + e;
          const float sw = c.F[kFSc + CB + lc];
          const float sc = c.dyn ? __fmul_rn(sw, aq.s) : sw;
          const __half h = elu16(__float2half_rn(qlinear_out32((int32_t)r[j + e], sc, c.F[kFBp + CB + lc])));
          h2v[e] = h;
          if (c.dyn && c.row_ok) {
            const float x = __half2float(h);
            zmax = fmaxf(zmax, nlet ? fabsf(__fadd_rn(__fmul_rn(x, c.F[kFNa + CB + lc]), c.F[kFNb + CB + lc]))
                                    : fabsf(x));
          }
        }
        __half2 pk = __halves2half2(h2v[0], h2v[1]);
        hv[ch][j >> 1] = *reinterpret_cast<uint32_t*>(&pk);
      }
    }
  }
  tc_fence_before();
  if (c.dyn) {
    zmax = warp_max(zmax);
    if (c.lane == 0 && zmax > 0.0f) atomic_max_nonneg(&p.slots[3 + l], zmax);
    mlp_grid_barrier(c, reinterpret_cast<uint32_t*>(&p.slots[kSlotBarrier + l]), gridDim.x, status);
    aqn.let = nlet;
    aqn.dyn = true;
    aqn.s = dyn_scale(ld_relaxed_gpu(&p.slots[3 + l]), nlet);
    aqn.rcp = __fdiv_rn(1.0f, aqn.s);
    aqn.inv = 0.0f;
  } else {
    aqn = make_act_quant(Ln, GLAD_ACT_STATIC, p.slots, 0);
  }
  if (!*c.abort_flag) {
    const uint32_t abase = smem_u32(c.sm + mlp_abuf(l + 1));
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int col0 = c.half * (NJ / 2) + ch * 16;
      const uint4 q = mlp_quant16(hv[ch], aqn, &c.F[kFNa + CB + col0], &c.F[kFNb + CB + col0]);
      const int kchunk = ((int)c.rank * NJ + col0) >> 4;     // K chunk of the next layer
      const uint32_t off = abase + kchunk * 2048 + c.row * 16;
#pragma unroll
      for (int r = 0; r < kMlpCluster; ++r) st_cluster_v4(mapa_shared(off, r), q);
    }
  }
  fence_async_cluster();
  cluster_sync_all();
}

__global__ void __launch_bounds__(kMlpThreads, 1) mlp_kernel(const __grid_constant__ MlpParams p) {
  extern __shared__ uint8_t smem_raw[];
  MlpCtx c;
  c.sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  c.F = reinterpret_cast<float*>(c.sm + kOffF);
  c.mbar = reinterpret_cast<uint64_t*>(c.sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(c.sm + kOffBar + 8);
  c.abort_flag = reinterpret_cast<int*>(c.sm + kOffBar + 12);
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  c.quarter = c.warp & 3;
  c.half = c.warp >> 2;
  c.row = 32 * c.quarter + c.lane;
  c.rank = cluster_ctarank();
  const int64_t m0 = (int64_t)(blockIdx.x / kMlpCluster) * 128;
  c.m = m0 + c.row;
  c.row_ok = c.m < p.M;
  c.dyn = p.act_mode == GLAD_ACT_DYNAMIC;
  c.phase = 0;
  c.mma_timeout = false;
  uint32_t* status = reinterpret_cast<uint32_t*>(&p.slots[kSlotStatus]);
  const int tid = c.tid;

  if (c.warp == 0) tmem_alloc(tmem_slot, kMlpTmemCols);
  if (tid == 0) {
    mbar_init(c.mbar, 1);
    fence_mbar_init();
    *c.abort_flag = 0;
  }
  // weight slices of all four layers, in flight while the input is quantised
  mlp_load_w(c.sm + kOffW0, p.L[0].w8, 224, (int)c.rank * 128, 128, tid);
  mlp_load_w(c.sm + kOffW1, p.L[1].w8, 512, (int)c.rank * 64, 64, tid);
  mlp_load_w(c.sm + kOffW2, p.L[2].w8, 256, (int)c.rank * 32, 32, tid);
  if (c.rank == 0) mlp_load_w(c.sm + kOffW3, p.L[3].w8, 128, 0, 32, tid);
  cp_async_commit();

  const ActQuant aq0 = make_act_quant(p.L[0], p.act_mode, p.slots, 2);
  for (int k = tid; k < 224; k += kMlpThreads) {
    c.F[kFInA + k] = aq0.let ? p.L[0].alpha[k] : 0.0f;
    c.F[kFInB + k] = aq0.let ? p.L[0].beta[k] : 0.0f;
  }
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const GladQLinear& L = p.L[l];
    const int nj = mlp_nj(l), n0 = l < 3 ? (int)c.rank * nj : 0;
    for (int j = tid; j < nj; j += kMlpThreads) {
      const int n = n0 + j;
      const bool in = n < mlp_n(l);
      c.F[kFSc + mlp_cb(l) + j] = in ? (c.dyn ? L.s_w[n] : L.dq_scale[n]) : 0.0f;
      c.F[kFBp + mlp_cb(l) + j] = in ? L.b_prime[n] : 0.0f;
      if (l < 3) {
        const GladQLinear& Ln = p.L[l + 1];
        c.F[kFNa + mlp_cb(l) + j] = Ln.alpha ? Ln.alpha[n] : 0.0f;
        c.F[kFNb + mlp_cb(l) + j] = Ln.alpha ? Ln.beta[n] : 0.0f;
      }
    }
  }
  __syncthreads();
  tc_fence_before();
  cluster_sync_all();                            // every CTA of the cluster runs before DSMEM stores
  tc_fence_after();
  c.tmem = *tmem_slot;

  // ---- layer 0 input: rank j quantises tile rows [32j, 32j+32) for the whole cluster ------
  {
    const uint32_t abase = smem_u32(c.sm + kOffA0);
    for (int it = tid; it < 32 * 14; it += kMlpThreads) {
      const int rr = 32 * (int)c.rank + it / 14, kc = it % 14;
      const int64_t mm = m0 + rr;
      uint4 q = make_uint4(0, 0, 0, 0);
      if (mm < p.M) {
        const uint4* src = reinterpret_cast<const uint4*>(p.x + mm * p.ldx + kc * 16);
        const uint4 v0 = src[0], v1 = src[1];
        const uint32_t h[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        q = mlp_quant16(h, aq0, &c.F[kFInA + kc * 16], &c.F[kFInB + kc * 16]);
      }
      const uint32_t off = abase + kc * 2048 + rr * 16;
#pragma unroll
      for (int r = 0; r < kMlpCluster; ++r) st_cluster_v4(mapa_shared(off, r), q);
    }
  }
  cp_async_wait_all();
  fence_async_smem();
  fence_async_cluster();
  cluster_sync_all();

  ActQuant aq1, aq2, aq3;
  mlp_hidden<0>(c, p, aq0, aq1, status);
  mlp_hidden<1>(c, p, aq1, aq2, status);
  mlp_hidden<2>(c, p, aq2, aq3, status);

  // ---- head (rank 0): 128 x 32 (29 real) outputs, mean = float(fp16(y)) (qrt/integration.py:206)
  if (c.rank == 0 && !*c.abort_flag) {
    mlp_mma(c, mlp_abuf(3), mlp_wbuf(3), 128, idesc_i8(128, 32), 32);
    if (!*c.abort_flag) {
      const int col0 = c.half * 16;
      uint32_t r[16];
      tmem_ld16(c.tmem + ((uint32_t)(32 * c.quarter) << 16) + col0, r);
      tmem_ld_wait();
      if (c.row_ok) {
        float* dst = p.mean + c.m * p.ldm;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = col0 + j;
          if (n < kActions) {
            const float sw = c.F[kFSc + mlp_cb(3) + n];
            const float sc = c.dyn ? __fmul_rn(sw, aq3.s) : sw;
            dst[n] = __half2float(qlinear_out((int32_t)r[j], sc, c.F[kFBp + mlp_cb(3) + n]));
          }
        }
      }
    }
  }

  // ---- teardown ----------------------------------------------------------------------------
  if (c.mma_timeout) {
    mbar_wait_bounded(c.mbar, c.phase ^ 1);      // the MMA still in flight gets one more bounded wait
    atomicOr(status, kDevErrMmaTimeout);
  }
  tc_fence_before();
  cluster_sync_all();
  if (c.warp == 0) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kMlpTmemCols);
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
                       float* mean, int64_t ldm, float* slots, cudaStream_t st) {
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
  const int tiles = (int)((M + 127) / 128);
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kMlpCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(tiles * kMlpCluster));
  cfg.blockDim = dim3(kMlpThreads);
  cfg.dynamicSmemBytes = kMlpSmem + 128;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mlp_kernel, p);
}

}  // namespace glad
