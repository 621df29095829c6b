// Shared-memory layouts and row staging of the encoder-front kernels (the
// pipelined kernel of glad_front.cu and the warp-specialised kernel of
// glad_front_ws.cu).
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
#pragma once
#include "glad_common.cuh"

namespace glad {

constexpr int kRowBytes = 304;                  // 38 slots x 8 bytes
constexpr int kPlaneRows = 16;
constexpr int kPlaneBytes = kPlaneRows * kRowBytes;   // 4864
constexpr int kPlanesBytes = 2 * kPlaneBytes;          // 9728
constexpr int kW1sBytes = 8 * 512;                     // 8 MMA K-steps x (2 chunks x 16 n x 16 B)
constexpr int kStripCols = 18;
constexpr int kStripBytes = 4736;                      // >= (255 + 2*18 + 2 + 1 + 1) * 16
constexpr int kW2sBytes = 5 * 2048;                    // 5 K-steps x (2 chunks x 64 n x 16 B)
constexpr int kStageBytes = 8864;                      // (128 + 2079) * 4 rounded up + 16
constexpr int kMaxProp = 104;                          // proprio width limit of the fused front mode

// K-chunk q (0..15) of the conv1 GEMM: byte offset inside the planes for GEMM row 0.
__device__ __forceinline__ uint32_t conv1_chunk_off(int q) {
  if (q >= 15) return conv1_chunk_off(14) + 16;        // zero-weight filler chunk
  const int kh = q / 3, j = q % 3;
  return (kh & 1) * kPlaneBytes + (kh >> 1) * kRowBytes + j * 16;
}
// Tap q (0..9) of the conv2 GEMM: position offset of GEMM row 0 in the strip.
__device__ __forceinline__ int conv2_tap_off(int q) {
  if (q >= 9) return 2 * kStripCols + 2 + 1;           // zero-weight filler tap
  return (q / 3) * kStripCols + (q % 3);
}

// One observation row staged in shared memory: the 16-byte aligned body
// arrives by cp.async (16 B), the 4-byte words before and after it by 4-byte
// cp.async; row byte j sits at stage[j] for j in [lo, hi). A row that is not
// 4-byte aligned (fp16 rows at an odd element offset) stages only its body and
// reads the ragged ends from global memory.
struct RowStage {
  const uint8_t* src;    // first byte of the row in global memory
  uint32_t lo, hi;       // staged byte range of the row
  uint32_t body_lo;      // 16-byte aligned body [body_lo, body_hi)
  uint32_t body_hi;
  uint8_t* stage;        // shared copy, indexed by row byte
};

__device__ __forceinline__ RowStage row_stage(const void* base, int64_t row, int64_t ld,
                                              int esz, int nelem, uint8_t* stage) {
  RowStage r;
  r.src = reinterpret_cast<const uint8_t*>(base) + row * ld * esz;
  const uintptr_t a = reinterpret_cast<uintptr_t>(r.src);
  const uint32_t nbytes = (uint32_t)nelem * esz;
  r.stage = stage + (a & 15);                          // same alignment as the source
  const uintptr_t lo16 = (a + 15) & ~uintptr_t(15);
  const uintptr_t hi16 = (a + nbytes) & ~uintptr_t(15);
  r.body_lo = (uint32_t)(lo16 - a);
  r.body_hi = hi16 > lo16 ? (uint32_t)(hi16 - a) : r.body_lo;
  if (nbytes >= 32 && (a & 3) == 0) {
    r.lo = 0;
    r.hi = nbytes & ~3u;
  } else {
    r.lo = r.body_lo;
    r.hi = r.body_hi;
  }
  return r;
}

__device__ __forceinline__ void row_issue(const RowStage& r, int tid, int nthr) {
  const uint32_t n16 = (r.body_hi - r.body_lo) >> 4;
  for (uint32_t i = tid; i < n16; i += nthr)
    cp_async16(r.stage + r.body_lo + i * 16, r.src + r.body_lo + i * 16);
  const int nh = (int)(r.body_lo - r.lo) >> 2, nt = (int)(r.hi - r.body_hi) >> 2;   // <= 3 each
  if (tid < nh) cp_async4(r.stage + r.lo + 4 * tid, r.src + r.lo + 4 * tid);
  else if (tid < nh + nt) cp_async4(r.stage + r.body_hi + 4 * (tid - nh), r.src + r.body_hi + 4 * (tid - nh));
}

// The same with the 16-byte body as ONE bulk copy by thread 0, whose completion
// (a phase of `bar`) the consumers wait for; the ragged head and tail words still go
// by 4-byte cp.async (consumers also wait for their cp.async groups).
__device__ __forceinline__ void row_issue_bulk(const RowStage& r, uint64_t* bar, int tid) {
  const uint32_t n = r.body_hi - r.body_lo;
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, n);
    if (n) bulk_copy_g2s(r.stage + r.body_lo, r.src + r.body_lo, n, bar);
  }
  const int nh = (int)(r.body_lo - r.lo) >> 2, nt = (int)(r.hi - r.body_hi) >> 2;   // <= 3 each
  if (tid >= 1 && tid <= nh) cp_async4(r.stage + r.lo + 4 * (tid - 1), r.src + r.lo + 4 * (tid - 1));
  else if (tid > nh && tid <= nh + nt)
    cp_async4(r.stage + r.body_hi + 4 * (tid - 1 - nh), r.src + r.body_hi + 4 * (tid - 1 - nh));
}

template <int ESZ>
__device__ __forceinline__ float row_elem(const RowStage& r, int i) {
  const uint32_t b = (uint32_t)i * ESZ;
  const uint8_t* p = (b >= r.lo && b < r.hi) ? r.stage + b : r.src + b;
  if (ESZ == 4) return *reinterpret_cast<const float*>(p);
  return __half2float(*reinterpret_cast<const __half*>(p));
}

}  // namespace glad
