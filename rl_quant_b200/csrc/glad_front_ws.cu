// Encoder front of the fused actor forward, warp-specialised.
//
// One persistent CTA per SM runs the per-environment chain of the front --
// observation row -> conv1 (fp16 tcgen05) -> z8 -> conv2 (int8 tcgen05) -> fp16
// local features -> GPS/scorer logits GEMM -> softmax -> pooling GEMM -> gc -- for
// the environments blockIdx.x, blockIdx.x + gridDim.x, ... Every stage has its own
// warps and every buffer between two stages is double-buffered, so up to six
// environments are in flight: while the conv2 epilogue of environment i runs, the
// conv1 epilogue of i+1, the conversion of i+2 and the softmax of i-1 run on other
// warps. Stages hand buffers over through mbarriers (a producer's arrival or an
// MMA commit marks "full", the consumer's arrival "empty"); no CTA-wide barrier
// is taken inside the loop.
//
//   warp 0      observation rows -> stage ring (one bulk copy per row body)
//   warps 1-2   conv1 MMAs (tile 0 / tile 1)           warp 3  conv2 MMAs
//   warp 4      logits MMAs                            warp 5  pooling MMAs
//   warps 6-7   stage -> fp16 conv1 planes
//   warps 8-11  conv1 epilogue: TMEM -> z8 -> conv2 strip and z8 (global)
//   warps 12-19 conv2 epilogue: TMEM -> fp16 local-feature tiles
//   warps 20-27 two groups of four; group g takes the environments i = g, g+2, ...:
//               per step the logits -> softmax -> pooling weights of i and the pooled
//               gc of i-2 (whose pooling MMAs ran meanwhile); group 0 first computes
//               the int8 proprio embedding of all the CTA's environments (one batched
//               GEMM after the proprio-absmax grid barrier)
//
// The operand layouts, descriptors and epilogue arithmetic are those of the
// pipelined front kernel (front_layout.cuh, glad_front.cu): identical integers and
// roundings. Reference: qrt/qconv.py:54-163, qrt/encoder_opt.py:41-77,
// qrt/qlinear.py:111-138.
#include <cuda_runtime.h>

#include <cstddef>

#include "front_layout.cuh"

namespace glad {

namespace ws {
constexpr int kWarps = 28;
constexpr int kThreads = kWarps * 32;
constexpr int kLoad = 0, kMma1 = 1, kMma2 = 3, kMmaLg = 4, kMmaPl = 5;
constexpr int kCvt = 6, kCvtWarps = 2, kCvtThreads = 32 * kCvtWarps;   // warps 6-7
constexpr int kNLocal = 3;                    // local-feature tiles in flight
constexpr int kEpi1 = 8;                      // warps 8-11
constexpr int kEpi2 = 12;                     // warps 12-19
constexpr int kSoft = 20;                     // warps 20-27: two groups of four, alternate environments
constexpr int kBarSoft = 2;                   // named barriers 2 and 3: one per softmax group
// TMEM columns (512 allocated): conv2 [0,256) buffer b at 128b, tile t at +64t; conv1
// [256,320) buffer b at +32b, tile t at +16t; logits [320,384) likewise; pooling
// [384,448) buffer b at +32b, K half h at +16h; batched proprio embedding [448,512)
constexpr uint32_t kColC2 = 0, kColC1 = 256, kColLg = 320, kColPl = 384, kColPe = 448;
constexpr uint32_t kTmemCols = 512;
constexpr int kLocalBytes = 2 * 8 * 128 * 16;     // fp16 local tile [tile][8-channel chunk][128 rows][16 B]
constexpr int kPeABytes = 8 * 2048;               // proprio A tile [16-byte K chunk][128 rows][16 B], K <= 128
}  // namespace ws

struct __align__(128) WsSmem {
  alignas(128) uint8_t local16[ws::kNLocal][ws::kLocalBytes];
  alignas(128) uint8_t pe_a[ws::kPeABytes];   // also the raw conv weights during the set-up
  alignas(128) uint8_t bpool[2][16 * 16 * 16];
  alignas(128) uint8_t blog[8 * 16 * 16];
  alignas(128) uint8_t stage[2][kStageBytes];
  alignas(128) uint8_t planes[2][kPlanesBytes];
  alignas(128) uint8_t strip[2][kStripBytes];
  alignas(128) uint8_t w1s[kW1sBytes];
  alignas(128) uint8_t w2s[kW2sBytes];
  alignas(128) uint8_t pe_w[8 * 64 * 16];     // int8 embedding weights as B: [K chunk][64 n][16 B]
  alignas(16) float b1[16];
  alignas(16) float qa[16];
  alignas(16) float qc[16];
  alignas(16) float dq[64];
  alignas(16) float b2[64];
  alignas(16) float a2[64];
  alignas(16) float c2[64];
  float4 ck[64];                              // conv2 epilogue constants per channel {dq, b2, a2, c2}
  float pe_la[kMaxProp], pe_lb[kMaxProp];     // proprio embedding LET alpha / beta
  float pe_scale[64], pe_bp[64];
  float qp_a[128], qp_b[128];                 // query projector LET (absmax of its input)
  float poolv[2][128];                        // [softmax group]
  float red[2][12];                           // [softmax group]: maxima [0,4), sums of tile 0 [4,8), tile 1 [8,12)
  float wmax[ws::kWarps];
  uint64_t c1_adesc[2][16];                   // [planes buffer][tile*8 + K-step]
  uint64_t c1_bdesc[8];
  uint64_t c2_adesc[2][10];                   // [strip buffer][tile*5 + K-step]
  uint64_t c2_bdesc[5];
  uint64_t lg_adesc[ws::kNLocal][2][4];       // [local buffer][tile][K-step]
  uint64_t lg_bdesc[4];
  uint64_t pl_adesc[ws::kNLocal][8];          // [local buffer][K-step]
  uint64_t pl_bdesc[2][8];                    // [pooling-weight buffer][K-step]
  uint64_t stage_full[2], stage_empty[2], planes_full[2], c1_full[2], c1_empty[2], strip_full[2];
  uint64_t c2_full[2], c2_empty[2], lg_full[2], lg_empty[2], pw_full[2];
  uint64_t local_full[ws::kNLocal], local_empty[ws::kNLocal];   // [local buffer]
  uint64_t pool_full[2], pool_empty[2], pe_done;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kWsSmemBytes = sizeof(WsSmem) + 128;   // + in-kernel alignment
static_assert(kWsSmemBytes <= 227 * 1024, "front_ws shared memory");

__device__ __forceinline__ bool ws_aborted(const WsSmem& s) {
  return *reinterpret_cast<const volatile int*>(&s.abort) != 0;
}

// Bounded wait on phase `parity` of `bar` that also gives up as soon as another
// role has aborted (so no role outlives a failure by more than one limit).
__device__ __noinline__ bool ws_wait(WsSmem& s, uint64_t* bar, uint32_t parity, float* slots) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(&s.abort)) return false;
    if (global_timer_ns() - t0 > 2000000000ull) {
      *reinterpret_cast<volatile int*>(&s.abort) = 1;
      atomicOr(reinterpret_cast<unsigned int*>(&slots[kSlotStatus]), kDevErrMmaTimeout);
      return false;
    }
  }
}

// ws_wait by every lane of a warp, with a warp-uniform result (an MMA issue from an
// elected lane and the warp-collective TMEM loads need the whole warp).
__device__ __forceinline__ bool warp_wait(WsSmem& s, uint64_t* bar, uint32_t parity, float* slots) {
  return __all_sync(0xffffffffu, ws_wait(s, bar, parity, slots));
}

__global__ void __launch_bounds__(ws::kThreads, 1) front_ws_kernel(const __grid_constant__ FrontParams p) {
  extern __shared__ uint8_t smem_raw[];
  WsSmem& s = *reinterpret_cast<WsSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3;
  const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
  constexpr int NT = ws::kThreads;
  grid_dep_launch();

  const int P = p.prop_dim;
  const int esz = p.in_dtype == GLAD_DTYPE_F32 ? 4 : 2;
  const int row_elems = P + kMap;
  const bool dyn = p.act_mode == GLAD_ACT_DYNAMIC;
  const int G = gridDim.x;
  const int n_env = blockIdx.x < p.B ? (int)((p.B - 1 - (int64_t)blockIdx.x) / G) + 1 : 0;
  auto env_of = [&](int i) { return (int64_t)blockIdx.x + (int64_t)i * G; };
  // warp 0: row of environment i -> stage[i & 1]; lane 0 bulk-copies the 16-byte aligned
  // body, lanes 1-6 the ragged head and tail words (4-byte rows; each of the six arrives
  // once its copies have landed, so stage_full expects 7 arrivals and the body's bytes)
  auto issue_row = [&](int i) {
    const int b = i & 1;
    const RowStage r = row_stage(p.in, env_of(i), p.ld, esz, row_elems, s.stage[b]);
    if (lane == 0) {
      const uint32_t n = r.body_hi - r.body_lo;
      mbar_arrive_expect_tx(&s.stage_full[b], n);
      if (n) bulk_copy_g2s(r.stage + r.body_lo, r.src + r.body_lo, n, &s.stage_full[b]);
    } else if (lane <= 6) {
      const int j = lane - 1;
      const int nh = (int)(r.body_lo - r.lo) >> 2, nt = (int)(r.hi - r.body_hi) >> 2;   // <= 3 each
      if (j < 3 && j < nh) cp_async4(r.stage + r.lo + 4 * j, r.src + r.lo + 4 * j);
      if (j >= 3 && j - 3 < nt) cp_async4(r.stage + r.body_hi + 4 * (j - 3), r.src + r.body_hi + 4 * (j - 3));
      cp_async_mbar_arrive_noinc(&s.stage_full[b]);
    }
  };

  // ---- one-time set-up ---------------------------------------------------------------------
  if (warp == 0) tmem_alloc(&s.tmem_base, ws::kTmemCols);
  if (tid == 0) {
    uint64_t* full2[] = {s.stage_full, s.c1_full, s.c1_empty, s.strip_full, s.c2_full, s.c2_empty,
                         s.lg_full, s.lg_empty, s.pw_full, s.pool_full, s.pool_empty,
                         s.stage_empty, s.planes_full};
    const uint32_t cnt[] = {7, 2, 4, 4, 1, 8, 1, 4, 4, 1, 4, ws::kCvtWarps, ws::kCvtWarps};
    for (int k = 0; k < 13; ++k)
      for (int b = 0; b < 2; ++b) mbar_init(&full2[k][b], cnt[k]);
    for (int b = 0; b < ws::kNLocal; ++b) {
      mbar_init(&s.local_full[b], 8);              // the eight conv2-epilogue warps
      mbar_init(&s.local_empty[b], 1);             // the pooling MMAs' commit
    }
    mbar_init(&s.pe_done, 1);
    fence_mbar_init();
    s.abort = 0;
  }
  if (warp == 0) {                      // the first two rows are in flight during the rest of the set-up
    __syncwarp();
    for (int i = 0; i < 2 && i < n_env; ++i) issue_row(i);
  }
  uint8_t* scratch = s.pe_a;            // raw conv weights until the derived operands exist
#pragma unroll 1
  for (int i = tid; i < 3 * 64 * 64 / 16; i += NT)
    cp_async16(scratch + 16 * i, reinterpret_cast<const uint4*>(p.conv.w8) + i);
#pragma unroll 1
  for (int i = tid; i < 128 * 16 * 2 / 16; i += NT)
    cp_async16(scratch + 12288 + 16 * i, reinterpret_cast<const uint4*>(p.conv.w1p) + i);
  if (tid < 16) {
    cp_async4(&s.b1[tid], p.conv.b1f + tid);
    cp_async4(&s.qa[tid], p.conv.qa + tid);
    cp_async4(&s.qc[tid], p.conv.qc + tid);
  }
  if (tid < 64) {
    cp_async4(&s.dq[tid], p.conv.dq + tid);
    cp_async4(&s.b2[tid], p.conv.b2f + tid);
    cp_async4(&s.a2[tid], p.conv.a2 + tid);
    cp_async4(&s.c2[tid], p.conv.c2 + tid);
    cp_async4(&s.pe_scale[tid], (dyn ? p.pe.s_w : p.pe.dq_scale) + tid);   // raw; scaled by s_z later
    cp_async4(&s.pe_bp[tid], p.pe.b_prime + tid);
  }
  // int8 embedding weights as the B operand: [16-byte K chunk][64 n][16 B], K zero-padded
  // to a multiple of 32 (P % 4 == 0, w8 16-byte aligned)
  const int pe_kc = ((P + 31) >> 5) * 2;
#pragma unroll 1
  for (int idx = tid; idx < pe_kc * kD * 4; idx += NT) {
    const int c = idx / (kD * 4), n = (idx >> 2) % kD, t4 = idx & 3;
    const int k = c * 16 + 4 * t4;
    uint8_t* dst = s.pe_w + c * 1024 + n * 16 + 4 * t4;
    if (k < P) cp_async4(dst, p.pe.w8 + (size_t)n * P + k);
    else *reinterpret_cast<uint32_t*>(dst) = 0u;
  }
  for (int k = tid; k < P; k += NT) {
    if (p.pe.alpha) {
      cp_async4(&s.pe_la[k], p.pe.alpha + k);
      cp_async4(&s.pe_lb[k], p.pe.beta + k);
    } else {
      s.pe_la[k] = 0.0f;
      s.pe_lb[k] = 0.0f;
    }
  }
  if (tid < 128) {
    if (p.qp.alpha) {
      cp_async4(&s.qp_a[tid], p.qp.alpha + tid);
      cp_async4(&s.qp_b[tid], p.qp.beta + tid);
    } else {
      s.qp_a[tid] = 0.0f;
      s.qp_b[tid] = 0.0f;
    }
  }
  cp_async_commit();
  // zero: conv halos (planes, strips), the local tiles (rows past the grid stay zero and
  // finite for the pooling GEMM), the pooling / logits B operands (unused columns)
  {
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll 1
    for (int i = tid; i < 2 * kPlanesBytes / 16; i += NT) reinterpret_cast<uint4*>(&s.planes[0][0])[i] = z;
#pragma unroll 1
    for (int i = tid; i < 2 * kStripBytes / 16; i += NT) reinterpret_cast<uint4*>(&s.strip[0][0])[i] = z;
#pragma unroll 1
    for (int i = tid; i < ws::kNLocal * ws::kLocalBytes / 16; i += NT)
      reinterpret_cast<uint4*>(&s.local16[0][0])[i] = z;
#pragma unroll 1
    for (int i = tid; i < 2 * 16 * 16 * 16 / 16; i += NT) reinterpret_cast<uint4*>(&s.bpool[0][0])[i] = z;
#pragma unroll 1
    for (int i = tid; i < 8 * 16 * 16 / 16; i += NT) reinterpret_cast<uint4*>(s.blog)[i] = z;
  }
  // dynamic int8 proprio embedding: this CTA's part of the batch absmax of
  // |alpha*fp16(x) + beta| over the proprio columns (qrt/qlinear.py:124-128)
  const bool grid_absmax = dyn && p.pe_absmax;
  if (grid_absmax) {
    float m = 0.0f;
    for (int i = warp; i < n_env; i += ws::kWarps) {
      const int64_t row = env_of(i);
#pragma unroll 4
      for (int k = lane; k < P; k += 32) {
        const float x = esz == 4 ? reinterpret_cast<const float*>(p.in)[row * p.ld + k]
                                 : __half2float(reinterpret_cast<const __half*>(p.in)[row * p.ld + k]);
        const float xr = fp16r(x);
        m = fmaxf(m, p.pe.alpha ? fabsf(__fadd_rn(__fmul_rn(xr, p.pe.alpha[k]), p.pe.beta[k])) : fabsf(xr));
      }
    }
    m = warp_max(m);
    if (lane == 0) s.wmax[warp] = m;
  }
  const __half lgw = tid < 2 * kD ? (tid < kD ? p.gps_w[tid] : p.scorer_w[tid - kD]) : __float2half(0.0f);
  const float gb = __half2float(p.gps_b[0]);
  grid_dep_wait();                      // workspace slots written by a preceding kernel are visible
  cp_async_wait_all();
  __syncthreads();
  if (grid_absmax && tid == 0) {
    // publish this CTA's maximum and arrive; the embedding warps wait before the first use
    float m = s.wmax[0];
#pragma unroll 1
    for (int w = 1; w < ws::kWarps; ++w) m = fmaxf(m, s.wmax[w]);
    if (m > 0.0f) atomic_max_nonneg(&p.slots[0], m);
    red_release_add(reinterpret_cast<uint32_t*>(&p.slots[kSlotFrontBarrier]), 1u);
  }
  // ---- derived operands ---------------------------------------------------------------------
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
    if (tid < 64) s.ck[tid] = make_float4(s.dq[tid], s.b2[tid], s.a2[tid], s.c2[tid]);
    if (tid < 2 * kD) {                  // logits B: row 0 = GPS weight, row 1 = scorer (local half)
      const int n = tid >> 6, c = (tid & 63) >> 3, e = tid & 7;
      reinterpret_cast<__half*>(s.blog)[(c * 16 + n) * 8 + e] = lgw;
    }
    // every MMA descriptor of the loop, one per thread
    if (tid < 32) {
      const int bb = tid >> 4, t = (tid >> 3) & 1, pr = tid & 7;
      const uint32_t c0 = conv1_chunk_off(2 * pr), c1 = conv1_chunk_off(2 * pr + 1);
      s.c1_adesc[bb][t * 8 + pr] = smem_desc(smem_u32(s.planes[bb]) + c0 + t * 128 * 16, c1 - c0, 128);
    } else if (tid < 40) {
      const int pr = tid - 32;
      s.c1_bdesc[pr] = smem_desc(smem_u32(s.w1s) + pr * 512, 256, 128);
    } else if (tid < 60) {
      const int bb = (tid - 40) / 10, t = ((tid - 40) % 10) / 5, pr = (tid - 40) % 5;
      const int o0 = conv2_tap_off(2 * pr), o1 = conv2_tap_off(2 * pr + 1);
      s.c2_adesc[bb][t * 5 + pr] = smem_desc(smem_u32(s.strip[bb]) + (t * 128 + o0) * 16, (o1 - o0) * 16, 128);
    } else if (tid < 65) {
      const int pr = tid - 60;
      s.c2_bdesc[pr] = smem_desc(smem_u32(s.w2s) + pr * 2048, 1024, 128);
    } else if (tid < 65 + 8 * ws::kNLocal) {
      // logits: A = local tile t, K-major (8-channel chunks 2048 B apart, 8-row groups 128 B)
      const int bb = (tid - 65) >> 3, t = ((tid - 65) >> 2) & 1, kk = (tid - 65) & 3;
      s.lg_adesc[bb][t][kk] = smem_desc(smem_u32(s.local16[bb]) + t * 16384 + kk * 2 * 2048, 2048, 128);
    } else if (tid < 69 + 8 * ws::kNLocal) {
      const int kk = tid - 65 - 8 * ws::kNLocal;
      s.lg_bdesc[kk] = smem_desc(smem_u32(s.blog) + kk * 2 * 256, 256, 128);
    } else if (tid < 69 + 16 * ws::kNLocal) {
      // pooling: A = the local tile read M-major (M = tile*64 + channel: 8-channel blocks
      // 2048 B apart; K = row: 8-row blocks 128 B apart), B = softmax weights, K-major
      const int x = tid - 69 - 8 * ws::kNLocal, bb = x >> 3, kk = x & 7;
      s.pl_adesc[bb][kk] = smem_desc(smem_u32(s.local16[bb]) + kk * 256, 128, 2048);
    } else if (tid < 85 + 16 * ws::kNLocal) {
      const int x = tid - 69 - 16 * ws::kNLocal, bb = x >> 3, kk = x & 7;
      s.pl_bdesc[bb][kk] = smem_desc(smem_u32(s.bpool[bb]) + kk * 2 * 256, 256, 128);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == ws::kLoad) {
    // ---- observation rows -> stage ring ----------------------------------------------------
    int last = n_env < 2 ? n_env - 1 : 1;
    for (int i = 2; i < n_env; ++i) {
      if (!warp_wait(s, &s.stage_empty[i & 1], ((i >> 1) - 1) & 1, p.slots)) break;
      issue_row(i);
      last = i;
    }
    if (ws_aborted(s))                   // copies still in flight land before the CTA exits
      for (int i = last > 0 ? last - 1 : 0; i <= last; ++i)
        mbar_wait_bounded(&s.stage_full[i & 1], (i >> 1) & 1);
  } else if (warp == ws::kMma1 || warp == ws::kMma1 + 1) {
    // ---- conv1 MMAs: tile t by warp 1 + t ----------------------------------------------------
    const int t = warp - ws::kMma1;
    constexpr uint32_t idesc = idesc_f16(128, 16);
    int issued = -1;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1;
      if (!warp_wait(s, &s.planes_full[b], k & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.c1_empty[b], (k - 1) & 1, p.slots)) break;
      tc_fence_after();
#pragma unroll
      for (int pr = 0; pr < 8; ++pr)
        mma_f16_warp(tmem + ws::kColC1 + 32 * b + 16 * t, s.c1_adesc[b][t * 8 + pr], s.c1_bdesc[pr], idesc,
                     pr > 0 ? 1u : 0u);
      mma_commit_warp(&s.c1_full[b]);
      issued = i;
    }
    if (ws_aborted(s) && issued >= 0) mbar_wait_bounded(&s.c1_full[issued & 1], (issued >> 1) & 1);
  } else if (warp == ws::kMma2) {
    // ---- conv2 MMAs (both tiles) --------------------------------------------------------------
    constexpr uint32_t idesc = idesc_i8(128, 64);
    int issued = -1;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1;
      if (!warp_wait(s, &s.strip_full[b], k & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.c2_empty[b], (k - 1) & 1, p.slots)) break;
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int pr = 0; pr < 5; ++pr)
          mma_i8_warp(tmem + ws::kColC2 + 128 * b + 64 * t, s.c2_adesc[b][t * 5 + pr], s.c2_bdesc[pr], idesc,
                      pr > 0 ? 1u : 0u);
      mma_commit_warp(&s.c2_full[b]);
      issued = i;
    }
    if (ws_aborted(s) && issued >= 0) mbar_wait_bounded(&s.c2_full[issued & 1], (issued >> 1) & 1);
  } else if (warp == ws::kMmaLg) {
    // ---- logits MMAs: [gps, scorer-local] = local @ [w_g; w_s]^T per tile -----------------------
    constexpr uint32_t idesc = idesc_f16(128, 16);
    int issued = -1;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1, lb = i % ws::kNLocal;
      if (!warp_wait(s, &s.local_full[lb], (i / ws::kNLocal) & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.lg_empty[b], (k - 1) & 1, p.slots)) break;
      tc_fence_after();
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_warp(tmem + ws::kColLg + 32 * b + 16 * t, s.lg_adesc[lb][t][kk], s.lg_bdesc[kk], idesc,
                       kk > 0 ? 1u : 0u);
      mma_commit_warp(&s.lg_full[b]);
      issued = i;
    }
    if (ws_aborted(s) && issued >= 0) mbar_wait_bounded(&s.lg_full[issued & 1], (issued >> 1) & 1);
  } else if (warp == ws::kMmaPl) {
    // ---- pooling MMAs: gc partials = local^T @ softmax weights ----------------------------------
    constexpr uint32_t idesc = idesc_f16_amajor_m(128, 16);
    int issued = -1;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1, lb = i % ws::kNLocal;
      if (!warp_wait(s, &s.pw_full[b], k & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.pool_empty[b], (k - 1) & 1, p.slots)) break;
      tc_fence_after();
      // rows 0-63 and 64-127 of each tile into two accumulators (columns +0 / +16), added
      // afterwards: the summation order of the pipelined front, so both give identical gc
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_warp(tmem + ws::kColPl + 32 * b + 16 * h, s.pl_adesc[lb][4 * h + kk], s.pl_bdesc[b][4 * h + kk],
                       idesc, kk > 0 ? 1u : 0u);
      mma_commit_warp(&s.pool_full[b]);
      mma_commit_warp(&s.local_empty[lb]);    // the last reader of local tile lb is done
      issued = i;
    }
    if (ws_aborted(s) && issued >= 0) mbar_wait_bounded(&s.pool_full[issued & 1], (issued >> 1) & 1);
  } else if (warp < ws::kEpi1) {
    // ---- stage -> fp16 conv1 planes ------------------------------------------------------------
    const int ct = tid - ws::kCvt * 32;
    const uint32_t nbytes = (uint32_t)row_elems * esz;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1;
      if (!warp_wait(s, &s.stage_full[b], k & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.c1_full[b], (k - 1) & 1, p.slots)) break;   // planes[b] free
      const RowStage r = row_stage(p.in, env_of(i), p.ld, esz, row_elems, s.stage[b]);
      uint8_t* pl = s.planes[b];
      if (esz == 4 && r.lo == 0 && r.hi == nbytes) {
        // the whole fp32 row is in shared memory
        const float* st = reinterpret_cast<const float*>(r.stage) + P;
#pragma unroll 1
        for (int px = ct; px < kH1 * kW1; px += ws::kCvtThreads) {
          const int ih = px / kW1, iw = px - ih * kW1;
          const int pi = ih & 1, rr = ((ih - pi) >> 1) + 1;
          const __half2 h01 = __floats2half2_rn(st[3 * px], st[3 * px + 1]);
          const __half2 h2z = __floats2half2_rn(st[3 * px + 2], 0.0f);
          *reinterpret_cast<uint2*>(pl + pi * kPlaneBytes + rr * kRowBytes + (iw + 2) * 8) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h2z));
        }
      } else {
        // fp16 rows (or rows off 4-byte alignment): bytes outside the staged range come
        // from global memory
#pragma unroll 1
        for (int px = ct; px < kH1 * kW1; px += ws::kCvtThreads) {
          const int ih = px / kW1, iw = px - ih * kW1;
          const int pi = ih & 1, rr = ((ih - pi) >> 1) + 1;
          const int c0 = P + 3 * px;
          float v0, v1, v2;
          if (esz == 4) {
            v0 = row_elem<4>(r, c0);
            v1 = row_elem<4>(r, c0 + 1);
            v2 = row_elem<4>(r, c0 + 2);
          } else {
            v0 = row_elem<2>(r, c0);
            v1 = row_elem<2>(r, c0 + 1);
            v2 = row_elem<2>(r, c0 + 2);
          }
          const __half2 h01 = __floats2half2_rn(v0, v1);
          const __half2 h2z = __floats2half2_rn(v2, 0.0f);
          *reinterpret_cast<uint2*>(pl + pi * kPlaneBytes + rr * kRowBytes + (iw + 2) * 8) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h2z));
        }
      }
      fence_async_smem();               // planes -> tensor core; stage reads before the next bulk copy
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.planes_full[b]);
        mbar_arrive(&s.stage_empty[b]);
      }
    }
  } else if (warp < ws::kEpi2) {
    // ---- conv1 epilogue: TMEM -> z8 -> conv2 strip (and z8 for the tail) ------------------------
    const bool live1 = 128 + 32 * quarter < 11 * 19;          // tile-1 rows of this warp in the grid
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1;
      if (!warp_wait(s, &s.c1_full[b], k & 1, p.slots)) break;
      if (i >= 2 && !warp_wait(s, &s.c2_full[b], (k - 1) & 1, p.slots)) break;   // strip[b] free
      tc_fence_after();
      const int64_t e = env_of(i);
      uint8_t* strip = s.strip[b];
      const int nt = live1 ? 2 : 1;
#pragma unroll 1
      for (int t = 0; t < nt; ++t) {
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + ws::kColC1 + 32 * b + 16 * t, r);
        tmem_ld_wait();
        if (t == nt - 1) {                 // the accumulators are read: conv1 of i+2 may start
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.c1_empty[b]);
        }
        const int m = 128 * t + 32 * quarter + lane;
        const int oh = m / 19, ow = m - oh * 19;
        if (oh < kH2 && ow < kW2) {
          uint32_t pk[4];
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const float4 b4 = *reinterpret_cast<const float4*>(&s.b1[4 * w4]);
            const float4 qa4 = *reinterpret_cast<const float4*>(&s.qa[4 * w4]);
            const float4 qc4 = *reinterpret_cast<const float4*>(&s.qc[4 * w4]);
            const uint32_t q0 = conv1_qbits(__uint_as_float(r[4 * w4 + 0]), b4.x, qa4.x, qc4.x);
            const uint32_t q1 = conv1_qbits(__uint_as_float(r[4 * w4 + 1]), b4.y, qa4.y, qc4.y);
            const uint32_t q2 = conv1_qbits(__uint_as_float(r[4 * w4 + 2]), b4.z, qa4.z, qc4.z);
            const uint32_t q3 = conv1_qbits(__uint_as_float(r[4 * w4 + 3]), b4.w, qa4.w, qc4.w);
            pk[w4] = __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
          }
          const uint4 v = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(strip + ((oh + 1) * kStripCols + ow + 1) * 16) = v;
          reinterpret_cast<uint4*>(p.z8_out)[e * kTok + oh * kW2 + ow] = v;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.strip_full[b]);
    }
  } else if (warp < ws::kSoft) {
    // ---- conv2 epilogue: TMEM -> fp16 local features (operand of the logits and pooling GEMMs) --
    // TMEM is read in the 16x256b shape: per 16-channel chunk a thread holds 4 rows x 4
    // channels (rows g, g+8, g+16, g+24 of the warp's quarter; channels 2q, 2q+1, 8+2q,
    // 9+2q), so it loads the constants of 4 channels instead of 16 broadcast loads (the
    // shared-memory pipe bounds this kernel); each warp store covers 8 rows x 16 bytes.
    const int c0 = 32 * ((warp - ws::kEpi2) >> 2);
    const int q = lane & 3, g = lane >> 2;
    const bool live1 = 128 + 32 * quarter < 11 * kStripCols;
    for (int i = 0; i < n_env; ++i) {
      const int b = i & 1, k = i >> 1;
      if (!warp_wait(s, &s.c2_full[b], k & 1, p.slots)) break;
      const int lb = i % ws::kNLocal;
      if (i >= ws::kNLocal && !warp_wait(s, &s.local_empty[lb], (i / ws::kNLocal - 1) & 1, p.slots))
        break;                                                  // local tile lb free
      tc_fence_after();
      const int64_t e = env_of(i);
      const int nt = live1 ? 2 : 1;
      // per 16-channel chunk its constants are loaded once and serve both tiles
#pragma unroll 1
      for (int hc = 0; hc < 2; ++hc) {
        const int cc = c0 + 16 * hc;
        const float4 k0 = s.ck[cc + 2 * q], k1 = s.ck[cc + 2 * q + 1];
        const float4 k2 = s.ck[cc + 8 + 2 * q], k3 = s.ck[cc + 9 + 2 * q];
#pragma unroll 1
        for (int t = 0; t < nt; ++t) {
          uint32_t ra[8], rb[8];
          const uint32_t ta = tmem + lane_base + ws::kColC2 + 128 * b + 64 * t + cc;
          tmem_ld16x256b_x2(ta, ra);                  // rows g, g+8 of the quarter
          tmem_ld16x256b_x2(ta + (16u << 16), rb);    // rows 16+g, 24+g
          tmem_ld_wait();
          if (hc == 1 && t == nt - 1) {      // the accumulators are read: conv2 of i+2 may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.c2_empty[b]);
          }
          uint8_t* tile = s.local16[lb] + 16384 * t + (cc >> 3) * 2048 + 4 * q;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t (&r)[8] = hh ? rb : ra;
            const int row = 32 * quarter + 16 * hh + g;   // and row + 8
            const __half2 h0 = __floats2half2_rn(conv2_val((int32_t)r[0], k0.x, k0.y, k0.z, k0.w),
                                                 conv2_val((int32_t)r[1], k1.x, k1.y, k1.z, k1.w));
            const __half2 h1 = __floats2half2_rn(conv2_val((int32_t)r[2], k0.x, k0.y, k0.z, k0.w),
                                                 conv2_val((int32_t)r[3], k1.x, k1.y, k1.z, k1.w));
            const __half2 h2 = __floats2half2_rn(conv2_val((int32_t)r[4], k2.x, k2.y, k2.z, k2.w),
                                                 conv2_val((int32_t)r[5], k3.x, k3.y, k3.z, k3.w));
            const __half2 h3 = __floats2half2_rn(conv2_val((int32_t)r[6], k2.x, k2.y, k2.z, k2.w),
                                                 conv2_val((int32_t)r[7], k3.x, k3.y, k3.z, k3.w));
            *reinterpret_cast<__half2*>(tile + row * 16) = h0;
            *reinterpret_cast<__half2*>(tile + (row + 8) * 16) = h1;
            *reinterpret_cast<__half2*>(tile + 2048 + row * 16) = h2;
            *reinterpret_cast<__half2*>(tile + 2048 + (row + 8) * 16) = h3;
            if (p.feat_out) {
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int m = 128 * t + row + 8 * j;
                const int oh = m / kStripCols, ow = m - oh * kStripCols;
                if (oh < kH2 && ow < kW2) {
                  __half2* dst = reinterpret_cast<__half2*>(p.feat_out + (e * kTok + oh * kW2 + ow) * kD + cc + 2 * q);
                  dst[0] = j ? h1 : h0;
                  dst[4] = j ? h3 : h2;
                }
              }
            }
          }
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.local_full[lb]);
    }
  } else {
    // ---- proprio embedding, then softmax / pooled gc per environment ---------------------------
    const int sid = (tid - ws::kSoft * 32) & 127;             // 32 * quarter + lane within the group
    const int wg = (warp - ws::kSoft) >> 2;
    const int sbar = ws::kBarSoft + wg;
    float zmax_qp = 0.0f;
    ActQuant aq_qp{};
    aq_qp.let = p.qp.alpha != nullptr;
    bool fail = false;
    if (wg == 0) {
      // (1) the batch scale of the embedding's input
      ActQuant aq_pe{};
      if (grid_absmax) {
        bool ok = true;
        if (sid == 0) {                   // every CTA has added its part (bounded spin, 2 s)
          const uint32_t* ctr = reinterpret_cast<const uint32_t*>(&p.slots[kSlotFrontBarrier]);
          const uint64_t t0 = global_timer_ns();
          while (ld_acquire_gpu(ctr) < (uint32_t)G) {
            if (global_timer_ns() - t0 > 2000000000ull) {
              ok = false;
              *reinterpret_cast<volatile int*>(&s.abort) = 1;
              atomicOr(reinterpret_cast<unsigned int*>(&p.slots[kSlotStatus]), kDevErrBarrierTimeout);
              break;
            }
          }
        }
        fail = named_bar_or(sbar, 128, !ok);
        aq_pe.let = p.pe.alpha != nullptr;
        aq_pe.dyn = true;
        aq_pe.s = dyn_scale(ld_relaxed_gpu(&p.slots[0]), aq_pe.let);
        aq_pe.rcp = __fdiv_rn(1.0f, aq_pe.s);
        aq_pe.inv = 0.0f;
      } else {
        aq_pe = make_act_quant(p.pe, p.act_mode, p.slots, 0);
      }
      if (dyn && sid < kD) s.pe_scale[sid] = __fmul_rn(s.pe_scale[sid], aq_pe.s);   // s_w * s_z
      named_bar_sync(sbar, 128);
      // (2) the int8 embedding of all this CTA's environments in batches of 128 rows: the
      // quantised rows are the A operand, w8 the B operand, the int32 products land in TMEM
      // columns [448, 512); the fp16 proprio goes to `enc`
      const int pe_q = pe_kc * 4;                                // 4-value items per row
      uint32_t ph_pe = 0;
      for (int j0 = 0; j0 < n_env && !fail; j0 += 128) {
        const int nb = n_env - j0 < 128 ? n_env - j0 : 128;
        for (int item = sid; item < nb * pe_q; item += 128) {
          const int r = item / pe_q, k0 = 4 * (item - r * pe_q);
          const int64_t e = env_of(j0 + r);
          auto ld = [&](int kk) -> __half {
            if (kk >= P) return __float2half(0.0f);
            return esz == 4 ? __float2half_rn(reinterpret_cast<const float*>(p.in)[e * p.ld + kk])
                            : reinterpret_cast<const __half*>(p.in)[e * p.ld + kk];
          };
          const __half h0 = ld(k0), h1 = ld(k0 + 1), h2 = ld(k0 + 2), h3 = ld(k0 + 3);
          auto qz = [&](__half h, int kk) {
            return kk < P ? ((uint32_t)aq_pe.quant(__half2float(h), s.pe_la[kk], s.pe_lb[kk]) & 0xFFu) : 0u;
          };
          *reinterpret_cast<uint32_t*>(s.pe_a + (k0 >> 4) * 2048 + r * 16 + (k0 & 15)) =
              qz(h0, k0) | (qz(h1, k0 + 1) << 8) | (qz(h2, k0 + 2) << 16) | (qz(h3, k0 + 3) << 24);
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
        named_bar_sync(sbar, 128);
        if (warp == ws::kSoft) {
          tc_fence_after();
          constexpr uint32_t idesc = idesc_i8(128, 64);
          for (int kk = 0; kk < pe_kc / 2; ++kk)
            mma_i8_warp(tmem + ws::kColPe, smem_desc(smem_u32(s.pe_a) + kk * 4096, 2048, 128),
                        smem_desc(smem_u32(s.pe_w) + kk * 2048, 1024, 128), idesc, kk > 0 ? 1u : 0u);
          mma_commit_warp(&s.pe_done);
        }
        const bool ok = ws_wait(s, &s.pe_done, ph_pe, p.slots);
        ph_pe ^= 1;
        if (named_bar_or(sbar, 128, !ok)) {
          fail = true;
          break;
        }
        tc_fence_after();
        if (32 * quarter < nb) {
          const int r = 32 * quarter + lane;
          const int64_t e = env_of(j0 + r);
  #pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t acc[16];
            tmem_ld16(tmem + lane_base + ws::kColPe + 16 * c, acc);
            tmem_ld_wait();
            if (r < nb) {
              uint32_t hw[8];
  #pragma unroll
              for (int t = 0; t < 16; t += 2) {
                const int n = 16 * c + t;
                const __half y0 = qlinear_out((int32_t)acc[t], s.pe_scale[n], s.pe_bp[n]);
                const __half y1 = qlinear_out((int32_t)acc[t + 1], s.pe_scale[n + 1], s.pe_bp[n + 1]);
                if (dyn) {
                  zmax_qp = fmaxf(zmax_qp, aq_qp.absz(__half2float(y0), s.qp_a[kD + n], s.qp_b[kD + n]));
                  zmax_qp = fmaxf(zmax_qp, aq_qp.absz(__half2float(y1), s.qp_a[kD + n + 1], s.qp_b[kD + n + 1]));
                }
                const __half2 h2 = __halves2half2(y0, y1);
                hw[t >> 1] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.pe_out + e * kD + 16 * c);
              dst[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
              dst[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            }
          }
        }
        tc_fence_before();
        named_bar_sync(sbar, 128);   // the A tile and the TMEM columns serve the next batch
      }
    }
    // (3) per step i: logits -> softmax -> pooling weights of environment i, then the pooled
    //     gc of environment i-2 (its pooling MMAs ran while the softmax of i was computed)
    const int ri = sid;                                       // row of tile 0; tile 1 row 128 + ri
    const bool live1 = 128 + 32 * quarter < 11 * kStripCols;
    const int oh0 = ri / kStripCols, ow0 = ri - oh0 * kStripCols;
    const int m1 = 128 + ri, oh1 = m1 / kStripCols, ow1 = m1 - oh1 * kStripCols;
    const int tok0 = oh0 < kH2 && ow0 < kW2 ? oh0 * kW2 + ow0 : -1;
    const int tok1 = oh1 < kH2 && ow1 < kW2 ? oh1 * kW2 + ow1 : -1;
    for (int i = wg; i < n_env + 2 && !fail; i += 2) {
      if (i < n_env) {
        const int b = i & 1, k = i >> 1;
        const int64_t e = env_of(i);
        const bool ok = ws_wait(s, &s.lg_full[b], k & 1, p.slots);
        if (named_bar_or(sbar, 128, !ok)) break;
        tc_fence_after();
        uint32_t la0, la1, lb0 = 0, lb1 = 0;
        tmem_ld2(tmem + lane_base + ws::kColLg + 32 * b, la0, la1);
        if (live1) tmem_ld2(tmem + lane_base + ws::kColLg + 32 * b + 16, lb0, lb1);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.lg_empty[b]);
        // logits (qrt/encoder_opt.py:69-73) and the softmax over the 187 tokens (:75)
        float g0 = -INFINITY, g1 = -INFINITY;
        if (tok0 >= 0) {
          g0 = fp16r(__fadd_rn(fp16r(__uint_as_float(la0)), gb));
          p.score_local[e * kTok + tok0] = __float2half_rn(__uint_as_float(la1));
        }
        if (tok1 >= 0) {
          g1 = fp16r(__fadd_rn(fp16r(__uint_as_float(lb0)), gb));
          p.score_local[e * kTok + tok1] = __float2half_rn(__uint_as_float(lb1));
        }
        float mx = warp_max(fmaxf(g0, g1));
        if (lane == 0) s.red[wg][quarter] = mx;
        named_bar_sync(sbar, 128);
        mx = fmaxf(fmaxf(s.red[wg][0], s.red[wg][1]), fmaxf(s.red[wg][2], s.red[wg][3]));
        const float ex0 = tok0 < 0 ? 0.0f : expf(g0 - mx);
        const float ex1 = tok1 < 0 ? 0.0f : expf(g1 - mx);
        // the pipelined front's order: one warp sum per (tile, quarter), then those sums in
        // sequence (tile 0 quarters 0-3, tile 1 quarters 0-2; tile 1's last quarter is past
        // the grid), so both fronts give the same weights
        const float s0 = warp_sum(ex0), s1 = warp_sum(ex1);
        if (lane == 0) {
          s.red[wg][4 + quarter] = s0;
          s.red[wg][8 + quarter] = s1;
        }
        named_bar_sync(sbar, 128);
        float sm = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) sm += s.red[wg][4 + q];
#pragma unroll
        for (int q = 0; q < 3; ++q) sm += s.red[wg][8 + q];
        // pooling B: column n = tile, K = row within the tile
        const __half w0 = __float2half_rn(__fdiv_rn(ex0, sm)), w1 = __float2half_rn(__fdiv_rn(ex1, sm));
        __half* bp = reinterpret_cast<__half*>(s.bpool[b] + (ri >> 3) * 256);
        bp[ri & 7] = tok0 < 0 ? __float2half(0.0f) : w0;
        bp[8 + (ri & 7)] = tok1 < 0 ? __float2half(0.0f) : w1;
        if (p.gc_w_out) {
          if (tok0 >= 0) p.gc_w_out[e * kTok + tok0] = w0;
          if (tok1 >= 0) p.gc_w_out[e * kTok + tok1] = w1;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.pw_full[b]);
      }
      if (i >= 2 && i - 2 < n_env) {
        // pooled global context gc = sum_i w_i local_i (qrt/encoder_opt.py:76-77) of j = i-2:
        // row tile*64 + c of the pooling accumulator, column `tile`
        const int j = i - 2, b = j & 1, k = j >> 1;
        const int64_t e = env_of(j);
        const bool ok = ws_wait(s, &s.pool_full[b], k & 1, p.slots);
        if (named_bar_or(sbar, 128, !ok)) break;
        tc_fence_after();
        uint32_t d0, d1, f0, f1;
        tmem_ld2(tmem + lane_base + ws::kColPl + 32 * b, d0, d1);
        tmem_ld2(tmem + lane_base + ws::kColPl + 32 * b + 16, f0, f1);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.pool_empty[b]);
        s.poolv[wg][sid] = __fadd_rn(__uint_as_float(sid < 64 ? d0 : d1), __uint_as_float(sid < 64 ? f0 : f1));
        named_bar_sync(sbar, 128);
        if (sid < kD) {
          const __half gh = __float2half_rn(s.poolv[wg][sid] + s.poolv[wg][64 + sid]);
          p.enc[e * p.ld_enc + 64 + sid] = gh;
          if (dyn) zmax_qp = fmaxf(zmax_qp, aq_qp.absz(__half2float(gh), s.qp_a[sid], s.qp_b[sid]));
        }
      }
    }
    // one atomic per CTA on the query projector's absmax slot
    if (dyn) {
      const float m = warp_max(zmax_qp);
      named_bar_sync(sbar, 128);
      if (lane == 0) s.red[wg][quarter] = m;
      named_bar_sync(sbar, 128);
      if (sid == 0) {
        const float mm = fmaxf(fmaxf(s.red[wg][0], s.red[wg][1]), fmaxf(s.red[wg][2], s.red[wg][3]));
        if (mm > 0.0f) atomic_max_nonneg(&p.slots[1], mm);
      }
    }
  }

  // ---- teardown ----------------------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, ws::kTmemCols);
  }
}

// Whether the warp-specialised front can run on the current device (one CTA per SM
// resident, which its proprio-absmax grid barrier needs), cached per device.
bool front_ws_usable() {
  static int cached[64];
  static bool have[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (have[dev]) return cached[dev] > 0;
  static bool done[64] = {false};
  int n = 0;
  if (allow_max_smem((const void*)front_ws_kernel, done) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, front_ws_kernel, ws::kThreads, kWsSmemBytes) !=
          cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cached[dev] = n;
  have[dev] = true;
  return n > 0;
}

cudaError_t launch_front_ws(const FrontParams& p, int grid, cudaStream_t st, bool pdl) {
  static bool done[64] = {false};
  cudaError_t e = allow_max_smem((const void*)front_ws_kernel, done);
  if (e != cudaSuccess) return e;
  return launch_k(front_ws_kernel, dim3(grid), dim3(ws::kThreads), kWsSmemBytes, st, pdl, p);
}

}  // namespace glad
