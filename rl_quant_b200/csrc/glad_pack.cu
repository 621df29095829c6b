// Packing of the inference copy's tensors into one contiguous device blob, so that the
// per-iteration weight hand-over is a single collective (qrt/runtime.py:224-271 refreshes
// one copy; across GPUs the refreshed copy is broadcast from one rank).
//
// Layout: item i at offset[i], the first 256-byte boundary at or after the end of item
// i-1 (item 0 at 0); the blob is the sum rounded up to 256 bytes. Packing and unpacking
// are one launch each: a byte copy per item (16-byte vectors where source, destination
// and size allow), up to kPackPerLaunch items per launch.
#include <cuda_runtime.h>

#include <cstdio>

#include "../../include/glad_b200.h"

namespace glad {
int set_last_error(int code, const char* msg);   // glad_abi.cu
}

namespace {

constexpr int kPackPerLaunch = 128;          // 3 KB of copy table per launch
constexpr size_t kPackAlign = 256;

struct PackCopy {
  const unsigned char* src;
  unsigned char* dst;
  size_t nbytes;
};
struct PackTable {
  PackCopy it[kPackPerLaunch];
};

__global__ void pack_copy_kernel(const __grid_constant__ PackTable t) {
  const PackCopy& c = t.it[blockIdx.y];
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(c.src) | reinterpret_cast<uintptr_t>(c.dst)) & 15) == 0;
  size_t done = 0;
  if (vec) {
    const size_t n16 = c.nbytes / 16;
    for (size_t i = i0; i < n16; i += stride)
      reinterpret_cast<uint4*>(c.dst)[i] = reinterpret_cast<const uint4*>(c.src)[i];
    done = n16 * 16;
  }
  for (size_t i = done + i0; i < c.nbytes; i += stride) c.dst[i] = c.src[i];
}

// Copy every item to (pack) or from (unpack) its place in the blob, in launches of up
// to kPackPerLaunch items (the copy table travels in the kernel parameters).
cudaError_t launch_pack(const GladPackItem* items, int n, unsigned char* blob, bool pack, cudaStream_t st) {
  for (int b = 0; b < n; b += kPackPerLaunch) {
    PackTable t;
    const int cnt = n - b < kPackPerLaunch ? n - b : kPackPerLaunch;
    size_t maxn = 16;
    for (int i = 0; i < cnt; ++i) {
      const GladPackItem& it = items[b + i];
      unsigned char* place = blob + it.offset;
      unsigned char* tensor = static_cast<unsigned char*>(it.tensor);
      t.it[i] = pack ? PackCopy{tensor, place, it.nbytes} : PackCopy{place, tensor, it.nbytes};
      if (it.nbytes > maxn) maxn = it.nbytes;
    }
    size_t blocks = (maxn / 16 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 64) blocks = 64;
    pack_copy_kernel<<<dim3((unsigned)blocks, (unsigned)cnt), 256, 0, st>>>(t);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int check_items(const GladPackItem* items, int n, size_t blob_bytes, const char* who) {
  char msg[160];
  if (n < 0 || (n > 0 && !items)) {
    snprintf(msg, sizeof(msg), "%s: items must be set and n >= 0", who);
    return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
  }
  for (int i = 0; i < n; ++i) {
    if (items[i].nbytes && !items[i].tensor) {
      snprintf(msg, sizeof(msg), "%s: item %d has no tensor", who, i);
      return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
    }
    if (items[i].offset % kPackAlign || items[i].offset + items[i].nbytes > blob_bytes) {
      snprintf(msg, sizeof(msg), "%s: item %d (offset %zu, %zu bytes) outside the %zu-byte blob or off the "
               "256-byte layout (glad_pack_layout)", who, i, items[i].offset, items[i].nbytes, blob_bytes);
      return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
    }
  }
  return GLAD_OK;
}

}  // namespace

extern "C" {

size_t glad_pack_layout(GladPackItem* items, int n) {
  if (n <= 0 || !items) return kPackAlign;
  size_t off = 0;
  for (int i = 0; i < n; ++i) {
    items[i].offset = off;
    off += (items[i].nbytes + kPackAlign - 1) / kPackAlign * kPackAlign;
  }
  return off > 0 ? off : kPackAlign;
}

static int pack_call(const GladPackItem* items, int n, unsigned char* blob, size_t blob_bytes, bool pack,
                     void* stream, const char* who) {
  int rc = check_items(items, n, blob_bytes, who);
  if (rc) return rc;
  if (n == 0) return GLAD_OK;
  char msg[160];
  if (!blob) {
    snprintf(msg, sizeof(msg), "%s: blob is NULL", who);
    return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
  }
  const cudaError_t e = launch_pack(items, n, blob, pack, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof(msg), "%s: %s", who, cudaGetErrorString(e));
    return glad::set_last_error(GLAD_ERR_CUDA, msg);
  }
  return GLAD_OK;
}

int glad_pack_weights(const GladPackItem* items, int n, void* blob, size_t blob_bytes, void* stream) {
  return pack_call(items, n, static_cast<unsigned char*>(blob), blob_bytes, true, stream, "glad_pack_weights");
}

int glad_unpack_weights(const GladPackItem* items, int n, const void* blob, size_t blob_bytes, void* stream) {
  return pack_call(items, n, const_cast<unsigned char*>(static_cast<const unsigned char*>(blob)), blob_bytes, false,
                   stream, "glad_unpack_weights");
}

}  // extern "C"
