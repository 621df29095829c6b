// MLP heads with fp16 activations, one cluster kernel per call:
//   * W4A16 actor MLP 224 -> 512 -> 256 -> 128 -> 29 with int4 weights (symmetric,
//     one fp16 scale per 64 consecutive inputs of a row). The reference names
//     INT4 only as future work (README.md:259); the format is this library's own:
//     W'[n,k] = fp16(q[n,k] * s[n, k/64]), q in [-8, 7].
//   * the fp16 critic MLP (128+P) -> 512 -> 256 -> 128 -> 1 of qrt full mode
//     (qrt/integration.py:42-43 leaves the critic unquantised).
// Each layer computes y = fp16(x @ W^T + b) with fp32 accumulation; hidden layers
// apply ELU in fp16; the head returns float(fp16(y)).
//
// One cluster of four CTAs per 128-row tile, as the INT8 fused MLP: CTA r owns
// output columns [r*NJ, (r+1)*NJ) of each hidden layer (NJ = 128/64/32) and the
// head (<= 32 outputs) runs on rank 0. A CTA builds its slice of the fp16 B operand
// in shared memory (int4: dequantised from a packed slice prefetched by cp.async
// while the previous layer runs; fp16: copied), issues kind::f16 tcgen05 MMAs, and
// stores its fp16 ELU columns into the A operand of all four CTAs (distributed
// shared memory). There is no batch-wide reduction, so any batch size launches.
#include <cuda_runtime.h>

#include "glad_common.cuh"

namespace glad {

constexpr int kW4Cluster = 4;
constexpr int kW4Threads = 256;
constexpr int kW4Group = 64;

// shared memory (bytes)
constexpr int kW4OffA = 0;                          // fp16 A: [K/8 chunks][128 rows][16 B], K <= 512
constexpr int kW4OffB = kW4OffA + 64 * 2048;        // fp16 B: [K/8 chunks][NJ rows][16 B] <= 64 KB
constexpr int kW4OffP = kW4OffB + 64 * 1024;        // packed int4 slice of one layer <= 16 KB
constexpr int kW4OffS = kW4OffP + 16 * 1024;        // its fp16 scales <= 1 KB
constexpr int kW4OffBias = kW4OffS + 1024;          // fp32 bias of the CTA's columns, 4 layers [256]
constexpr int kW4OffBar = kW4OffBias + 256 * 4;
constexpr int kW4Smem = kW4OffBar + 64;
static_assert(kW4Smem + 128 <= 227 * 1024, "shared memory");

__host__ __device__ constexpr int w4_nj(int l) { return l == 0 ? 128 : l == 1 ? 64 : 32; }
__host__ __device__ constexpr int w4_cb(int l) { return l == 0 ? 0 : l == 1 ? 128 : l == 2 ? 192 : 224; }
__host__ __device__ constexpr int w4_groups(int K) { return (K + kW4Group - 1) / kW4Group; }
__host__ __device__ constexpr int round16(int K) { return (K + 15) & ~15; }

struct HalfLayer {
  const void* w;           // int4: packed [N, K/2]; fp16: [N, K] row-major
  const __half* scales;    // int4 only: [N, ceil(K/64)]
  const __half* bias;      // [N] or null
  int K, N;
};

struct HalfMlpParams {
  HalfLayer L[4];          // hidden widths 512 / 256 / 128; head N <= 32; L[0].K <= 256
  const __half* x;         // [M, ldx] fp16
  int64_t M, ldx;
  float* out;              // [M, ldo] = float(fp16(head output))
  int64_t ldo;
  unsigned int* status;    // device status word or null
};

// 8 halves [8c, 8c+8) of row `row` (K columns, stride ld) -> 16 bytes of shared
// memory: one 16-byte copy when whole and aligned, else element loads, zero past K.
__device__ __forceinline__ void half_chunk(uint8_t* dst, const __half* row, int c, int K, bool vec_ok) {
  if (vec_ok && 8 * c + 8 <= K) {
    cp_async16(dst, row + 8 * c);
  } else {
    __align__(16) __half v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 8 * c + e < K ? row[8 * c + e] : __float2half(0.0f);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
  }
}

// Packed rows [n0, n0+rows) of an int4 layer and their scales -> P / S.
__device__ __forceinline__ void w4_fetch(uint8_t* P, uint8_t* S, const HalfLayer& L, int n0, int rows, int tid) {
  const int K = L.K, kb = K / 2, G = w4_groups(K);
  const uint8_t* pk = reinterpret_cast<const uint8_t*>(L.w);
  const int live = max(0, min(rows, L.N - n0));      // rows past N are zero (head padding)
  const int nbytes = live * kb;
  for (int i = tid; i < nbytes / 16; i += kW4Threads)
    cp_async16(P + 16 * i, pk + (int64_t)n0 * kb + 16 * i);
  for (int i = tid; i < (rows * kb - nbytes) / 16; i += kW4Threads)
    *reinterpret_cast<uint4*>(P + nbytes + 16 * i) = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < rows * G; i += kW4Threads) {
    const int r = i / G;
    reinterpret_cast<__half*>(S)[i] = r < live ? L.scales[(int64_t)(n0 + r) * G + (i - r * G)] : __float2half(0.0f);
  }
}

// P / S (rows x K) -> fp16 B operand [Kp/8][rows][16 B]: W' = fp16(q * s).
__device__ __forceinline__ void w4_dequant(uint8_t* B, const uint8_t* P, const uint8_t* S, int K, int rows,
                                           int tid) {
  const int kb = K / 2, G = w4_groups(K);
  for (int idx = tid; idx < rows * (K / 8); idx += kW4Threads) {
    const int c = idx / rows, n = idx - c * rows;     // lanes walk rows: 16-byte stores, 4-byte loads
    const uint32_t w = *reinterpret_cast<const uint32_t*>(P + n * kb + 4 * c);
    const float s = __half2float(reinterpret_cast<const __half*>(S)[n * G + (8 * c) / kW4Group]);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int lo = (int)((w >> (8 * j)) & 0xF), hi = (int)((w >> (8 * j + 4)) & 0xF);
      const float a = (float)(lo >= 8 ? lo - 16 : lo) * s, b = (float)(hi >= 8 ? hi - 16 : hi) * s;
      const __half2 h = __floats2half2_rn(a, b);
      o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(B + c * rows * 16 + n * 16) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int idx = tid; idx < rows * (round16(K) / 8 - K / 8); idx += kW4Threads)   // K padding chunk
    *reinterpret_cast<uint4*>(B + (K / 8) * rows * 16 + idx * 16) = make_uint4(0, 0, 0, 0);
}

// fp16 weight rows [n0, n0+rows) -> B operand [Kp/8][rows][16 B] (cp.async where aligned).
__device__ __forceinline__ void f16_fetch_b(uint8_t* B, const HalfLayer& L, int n0, int rows, int tid) {
  const int K = L.K, Kp8 = round16(K) / 8;
  const __half* w = reinterpret_cast<const __half*>(L.w);
  const bool vec_ok = (K % 8) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  for (int idx = tid; idx < rows * Kp8; idx += kW4Threads) {
    const int c = idx / rows, n = idx - c * rows;
    uint8_t* dst = B + c * rows * 16 + n * 16;
    if (n0 + n < L.N) half_chunk(dst, w + (int64_t)(n0 + n) * K, c, K, vec_ok);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

template <bool W4>
__global__ void __launch_bounds__(kW4Threads, 1) halfmlp_kernel(const __grid_constant__ HalfMlpParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* A = sm + kW4OffA;
  uint8_t* Bw = sm + kW4OffB;
  uint8_t* P = sm + kW4OffP;
  uint8_t* S = sm + kW4OffS;
  float* bias = reinterpret_cast<float*>(sm + kW4OffBias);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + kW4OffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kW4OffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(sm + kW4OffBar + 12);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int row = 32 * quarter + lane;
  const uint32_t rank = cluster_ctarank();
  const int64_t m0 = (int64_t)(blockIdx.x / kW4Cluster) * 128;
  const int64_t m = m0 + row;
  const bool row_ok = m < p.M;
  uint32_t phase = 0;
  bool mma_timeout = false;

  if (warp == 0) tmem_alloc(tmem_slot, 128);
  if (tid == 0) {
    mbar_init(mbar, 1);
    fence_mbar_init();
    *abort_flag = 0;
  }
  // weights of layer 0 (int4: packed slice; fp16: the B operand itself) and biases
  if (W4) w4_fetch(P, S, p.L[0], (int)rank * 128, 128, tid);
  else f16_fetch_b(Bw, p.L[0], (int)rank * 128, 128, tid);
  for (int l = 0; l < 4; ++l) {
    const int nj = l < 3 ? w4_nj(l) : 32, n0 = l < 3 ? (int)rank * nj : 0;
    for (int j = tid; j < nj; j += kW4Threads) {
      const int n = n0 + j;
      bias[w4_cb(l) + j] = (n < p.L[l].N && p.L[l].bias) ? __half2float(p.L[l].bias[n]) : 0.0f;
    }
  }
  // layer-0 input rows (fp16, K-major chunks, zero past K and past M)
  grid_dep_wait();
  {
    const int K0 = p.L[0].K, c8 = round16(K0) / 8;
    const bool vec_ok = (K0 % 8) == 0 && (p.ldx % 8) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    for (int idx = tid; idx < 128 * c8; idx += kW4Threads) {
      const int r = idx / c8, c = idx - r * c8;
      uint8_t* dst = A + c * 2048 + r * 16;
      if (m0 + r < p.M) half_chunk(dst, p.x + (m0 + r) * p.ldx, c, K0, vec_ok);
      else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  tc_fence_before();
  cluster_sync_all();                               // every CTA runs before the first DSMEM store
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;

#pragma unroll 1
  for (int l = 0; l < 4; ++l) {
    const bool head = l == 3;
    if (head && rank != 0) break;                   // uniform per CTA
    const int K = p.L[l].K, Kp = round16(K), NJ = head ? 32 : w4_nj(l);
    // ---- this layer's fp16 B operand ------------------------------------------------------
    if (W4) {
      w4_dequant(Bw, P, S, K, NJ, tid);
    } else if (l > 0) {
      f16_fetch_b(Bw, p.L[l], head ? 0 : (int)rank * NJ, NJ, tid);
      cp_async_commit();
      cp_async_wait_all();
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // int4: prefetch the next layer's packed slice while this layer runs
    if (W4 && l < 3) {
      const int nn = l + 1;
      if (nn < 3) w4_fetch(P, S, p.L[nn], (int)rank * w4_nj(nn), w4_nj(nn), tid);
      else if (rank == 0) w4_fetch(P, S, p.L[3], 0, 32, tid);
      cp_async_commit();
    }
    // ---- MMA ----------------------------------------------------------------------------------
    if (!*abort_flag) {
      if (tid == 0) {
        tc_fence_after();
        const uint32_t ab = smem_u32(A), bb = smem_u32(Bw);
        const uint32_t idesc = NJ == 128 ? idesc_f16(128, 128) : NJ == 64 ? idesc_f16(128, 64) : idesc_f16(128, 32);
        for (int kc = 0; kc < Kp / 16; ++kc) {
          const uint64_t ad = smem_desc(ab + kc * 2 * 2048, 2048, 128);
          const uint64_t bd = smem_desc(bb + kc * 2 * NJ * 16, NJ * 16, 128);
          mma_f16(tmem, ad, bd, idesc, kc > 0 ? 1u : 0u);
        }
        mma_commit(mbar);
      }
      if (!mbar_wait_bounded(mbar, phase)) {
        *abort_flag = 1;
        mma_timeout = true;
      }
      phase ^= 1;
    }
    tc_fence_after();
    __syncthreads();
    if (head) {
      // ---- head: out = float(fp16(y)) (qrt/integration.py:206) ------------------------------
      if (!*abort_flag) {
        const int col0 = half * 16;
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + col0, r);
        tmem_ld_wait();
        if (row_ok) {
          float* dst = p.out + m * p.ldo;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = col0 + j;
            if (n < p.L[3].N)
              dst[n] = __half2float(__float2half_rn(__fadd_rn(__uint_as_float(r[j]), bias[w4_cb(3) + n])));
          }
        }
      }
      break;
    }
    // every CTA of the cluster has finished reading its A before any CTA overwrites it
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    // ---- epilogue: bias, fp16, ELU -> the next layer's A in all four CTAs ----------------------
    if (!*abort_flag) {
      const uint32_t abase = smem_u32(A);
#pragma unroll 1
      for (int ch = half; ch < NJ / 16; ch += 2) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + ch * 16, r);
        tmem_ld_wait();
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int c = w4_cb(l) + ch * 16 + j;
          const __half y0 = elu16(__float2half_rn(__fadd_rn(__uint_as_float(r[j]), bias[c])));
          const __half y1 = elu16(__float2half_rn(__fadd_rn(__uint_as_float(r[j + 1]), bias[c + 1])));
          const __half2 pk = __halves2half2(y0, y1);
          h[j >> 1] = *reinterpret_cast<const uint32_t*>(&pk);
        }
        const int kchunk = ((int)rank * NJ + ch * 16) >> 3;   // 8-column K chunk of the next layer
        const uint32_t o0 = abase + kchunk * 2048 + row * 16;
        const uint4 v0 = make_uint4(h[0], h[1], h[2], h[3]), v1 = make_uint4(h[4], h[5], h[6], h[7]);
#pragma unroll
        for (int q = 0; q < kW4Cluster; ++q) {
          st_cluster_v4(mapa_shared(o0, q), v0);
          st_cluster_v4(mapa_shared(o0 + 2048, q), v1);
        }
      }
    }
    tc_fence_before();
    cp_async_wait_all();                            // int4: the prefetched slice of the next layer
    fence_async_cluster();
    cluster_sync_all();
    tc_fence_after();
  }

  // ---- teardown ----------------------------------------------------------------------------
  cp_async_wait_all();
  if (mma_timeout) {
    mbar_wait_bounded(mbar, phase ^ 1);
    if (p.status) atomicOr(p.status, kDevErrMmaTimeout);
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

template <bool W4>
static cudaError_t launch_halfmlp(const HalfMlpParams& p, cudaStream_t st, bool pdl) {
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)halfmlp_kernel<W4>, done);
  if (e != cudaSuccess) return e;
  const int64_t tiles = (p.M + 127) / 128;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kW4Cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(tiles * kW4Cluster));
  cfg.blockDim = dim3(kW4Threads);
  cfg.dynamicSmemBytes = kW4Smem + 128;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, halfmlp_kernel<W4>, p);
}

cudaError_t launch_w4mlp(const GladW4Linear (&L)[4], const __half* x, int64_t M, int64_t ldx, float* mean,
                         int64_t ldm, unsigned int* status, cudaStream_t st, bool pdl) {
  HalfMlpParams p{};
  for (int i = 0; i < 4; ++i)
    p.L[i] = HalfLayer{L[i].packed, reinterpret_cast<const __half*>(L[i].scales),
                       reinterpret_cast<const __half*>(L[i].bias), L[i].in_features, L[i].out_features};
  p.x = x;
  p.M = M;
  p.ldx = ldx;
  p.out = mean;
  p.ldo = ldm;
  p.status = status;
  return launch_halfmlp<true>(p, st, pdl);
}

// The fp16 critic MLP: layers {weight [N,K] fp16, bias}, K0 = L[0].in_features <= 256.
cudaError_t launch_f16mlp(const GladLinear16 (&L)[4], const __half* x, int64_t M, int64_t ldx, float* value,
                          int64_t ldv, unsigned int* status, cudaStream_t st, bool pdl) {
  HalfMlpParams p{};
  for (int i = 0; i < 4; ++i)
    p.L[i] = HalfLayer{L[i].weight, nullptr, reinterpret_cast<const __half*>(L[i].bias), L[i].in_features,
                       L[i].out_features};
  p.x = x;
  p.M = M;
  p.ldx = ldx;
  p.out = value;
  p.ldo = ldv;
  p.status = status;
  return launch_halfmlp<false>(p, st, pdl);
}

}  // namespace glad
