// glad_actor_forward_noalloc: the fused actor forward for callers that must
// not allocate device memory.
//
// Who needs it: a host runtime that owns every device allocation through its
// own pool (a simulator or an inference server that forbids plugins from
// calling cudaMalloc, or that cannot tolerate the implicit synchronisation
// and fragmentation a cudaMalloc/cudaFree pair brings into a running rollout
// loop) cannot hand this library a workspace of its own. This entry point
// uses a scratch array that the library owns instead.
//
// The scratch is a file-scope __device__ array sized for at most
// GLAD_NOALLOC_MAX_B environments; every GPU that loads the library holds it
// (about 11.2 MiB) until the process exits. Host code cannot use the array's
// name as a device address, so the first call on each device (with that
// device current) resolves the address with cudaGetSymbolAddress; make that
// first call before any stream capture. All calls share the one array and
// find the previous call's contents in it: the per-call reductions are
// cleared at the start of every call, and calls that overlap on the GPU
// (two streams, or two host threads) race on the array, so serialise them.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "glad_common.cuh"

namespace {

// Same carve-up as glad_actor_workspace_size(GLAD_NOALLOC_MAX_B): slots,
// z8, score_local, proprio embedding, encoded, h1, h2, h3 (256-byte aligned).
constexpr size_t up256c(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kNoAllocBytes =
    up256c(glad::kSlotsBytes) + up256c((size_t)GLAD_NOALLOC_MAX_B * glad::kTok * 16) +
    up256c((size_t)GLAD_NOALLOC_MAX_B * glad::kTok * 2) + up256c((size_t)GLAD_NOALLOC_MAX_B * glad::kD * 2) +
    up256c((size_t)GLAD_NOALLOC_MAX_B * glad::kEnc * 2) + up256c((size_t)GLAD_NOALLOC_MAX_B * 512 * 2) +
    up256c((size_t)GLAD_NOALLOC_MAX_B * 256 * 2) + up256c((size_t)GLAD_NOALLOC_MAX_B * 128 * 2);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

}  // namespace

namespace glad {
int set_last_error(int code, const char* msg);   // glad_abi.cu
}

namespace {

// The array's device address on the current device, resolved once per device with
// that device current. The first resolution may load the module on the device,
// which a capturing stream does not allow, so it is refused during capture.
// The cached address assumes the device's primary context lives until exit
// (cudaDeviceReset is not supported together with this entry point).
int scratch_address(void** out, cudaStream_t stream, const char* who) {
  char msg[256];
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    snprintf(msg, sizeof(msg), "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
    return glad::set_last_error(GLAD_ERR_CUDA, msg);
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
      snprintf(msg, sizeof(msg),
               "%s: the first call on device %d must come before any stream capture (it resolves the "
               "static scratch's device address)", who, dev);
      return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      snprintf(msg, sizeof(msg), "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
      return glad::set_last_error(GLAD_ERR_CUDA, msg);
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return GLAD_OK;
}

}  // namespace

extern "C" {

int glad_actor_forward_noalloc(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                               int64_t ld_obs, int act_mode, const float* topk_noise, float* mean_out,
                               const GladActorAux* aux, void* stream) {
  char msg[256];
  if (B < 0 || B > GLAD_NOALLOC_MAX_B) {
    snprintf(msg, sizeof(msg),
             "glad_actor_forward_noalloc: B=%lld outside [0, %d] (the static scratch holds at most "
             "GLAD_NOALLOC_MAX_B environments; use glad_actor_forward with a workspace for more)",
             (long long)B, GLAD_NOALLOC_MAX_B);
    return glad::set_last_error(GLAD_ERR_INVALID_ARG, msg);
  }
  if (glad_actor_workspace_size(GLAD_NOALLOC_MAX_B) > kNoAllocBytes)
    return glad::set_last_error(GLAD_ERR_WORKSPACE,
                                "glad_actor_forward_noalloc: static scratch smaller than the workspace layout");
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch, (cudaStream_t)stream, "glad_actor_forward_noalloc");
  if (rc) return rc;
  return glad_actor_forward(w, obs, obs_dtype, B, ld_obs, act_mode, topk_noise, mean_out, aux, scratch,
                            kNoAllocBytes, stream);
}

int glad_actor_noalloc_status(uint32_t* status, void* stream) {
  if (!status) return glad::set_last_error(GLAD_ERR_INVALID_ARG, "glad_actor_noalloc_status: status is NULL");
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch, (cudaStream_t)stream, "glad_actor_noalloc_status");
  if (rc) return rc;
  return glad_workspace_status(scratch, status, stream);
}

}  // extern "C"
