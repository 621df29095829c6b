// C-ABI entry points (include/glad_b200.h): argument checks, workspace
// carve-up and launch order. No allocation happens here; every buffer is the
// caller's.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "glad_common.cuh"

namespace glad {
size_t front_smem_bytes();
template <int MODE>
cudaError_t launch_front(const FrontParams& p, int grid, cudaStream_t st, bool pdl = false);
size_t tail_smem_bytes();
cudaError_t launch_tail(const TailParams& p, int grid, cudaStream_t st, bool pdl = false);
int tail_grid(int64_t B, int sms);
int front_fused_blocks_per_sm();
bool front_ws_usable();
cudaError_t launch_front_ws(const FrontParams& p, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_chain(const FrontParams& p, int grid, cudaStream_t st);
cudaError_t launch_w4mlp(const GladW4Linear (&L)[4], const __half* x, int64_t M, int64_t ldx, float* mean,
                         int64_t ldm, unsigned int* status, cudaStream_t st, bool pdl);
cudaError_t launch_f16mlp(const GladLinear16 (&L)[4], const __half* x, int64_t M, int64_t ldx, float* value,
                          int64_t ldv, unsigned int* status, cudaStream_t st, bool pdl);
template <int NT>
cudaError_t launch_qgemm(const GemmParams& p, cudaStream_t st, bool pdl = false);
size_t qgemm_smem_bytes(int K, int NT);
cudaError_t launch_absmax(const void* x, int dtype, int64_t M, int64_t ld, int K,
                          const float* alpha, const float* beta, int round16, float* slot,
                          int num_sms, cudaStream_t st, const float* norm_mean = nullptr,
                          const float* norm_var = nullptr, float norm_eps = 0.0f);
cudaError_t launch_act_scales(const float* slots, int act_mode, const float* const s_z[6],
                              const int let[6], float* out, cudaStream_t st);
cudaError_t launch_requant_qlinear(const GladQLinearSrc* layers, int n, cudaStream_t st);
cudaError_t launch_requant_qcnn(const GladQCNNSrc& s, cudaStream_t st);
cudaError_t launch_cast_copy(const GladCastCopy* items, int n, cudaStream_t st);
int mlp_max_tiles(int act_mode, cudaStream_t st);
cudaError_t launch_ppo_epilogue(const PpoParams& p, cudaStream_t st, bool pdl);
cudaError_t launch_mlp(const GladQLinear (&L)[4], int act_mode, const __half* x, int64_t M, int64_t ldx,
                       float* mean, int64_t ldm, float* slots, cudaStream_t st, bool pdl = false);
}  // namespace glad

using namespace glad;

namespace {

thread_local char g_err[512] = "";
thread_local cudaEvent_t g_stage_ev[16];
thread_local int g_stage_n = 0;

// Record stage event `i` (if diagnostics are on) on `st`.
void stage_mark(int i, cudaStream_t st) {
  if (i < g_stage_n) cudaEventRecord(g_stage_ev[i], st);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GLAD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define GLAD_CHECK_CUDA(expr, what)              \
  do {                                           \
    cudaError_t e_ = (expr);                     \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

struct DeviceInfo {
  int sms = 0;
  int major = 0;
};

// Per-device properties, queried once per device.
int device_info(DeviceInfo* out) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool have[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(GLAD_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!have[dev]) {
    DeviceInfo d;
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(CC major)");
    cache[dev] = d;
    have[dev] = true;
  }
  if (cache[dev].major != 10)
    return fail(GLAD_ERR_UNSUPPORTED, "device %d is sm_%d0; this library is built for sm_100a",
                dev, cache[dev].major);
  *out = cache[dev];
  return GLAD_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_conv(const GladConvWeights* w, bool c1, bool c2) {
  if (!w) return fail(GLAD_ERR_INVALID_ARG, "conv weights are NULL");
  if (c1 && (!w->w1p || !w->b1f || !w->qa || !w->qc))
    return fail(GLAD_ERR_INVALID_ARG, "conv1 buffers (w1p, b1f, qa, qc) must be set");
  if (c2 && (!w->w8 || !w->dq || !w->b2f || !w->a2 || !w->c2))
    return fail(GLAD_ERR_INVALID_ARG, "conv2 buffers (w8, dq, b2f, a2, c2) must be set");
  if ((c1 && !aligned(w->w1p, 16)) || (c2 && !aligned(w->w8, 16)))
    return fail(GLAD_ERR_INVALID_ARG, "conv weights w1p / w8 must be 16-byte aligned");
  return GLAD_OK;
}

// `gemm`: the layer runs through the tcgen05 GEMM (in_features % 8 == 0,
// qrt/qlinear.py:52-53); otherwise it is the front kernel's dp4a embedding
// (in_features % 4 == 0, <= 128).
// Observation normaliser of a group of `width` columns (mean NULL: none).
int check_norm(const GladObsNorm& n, int width, int obs_dtype) {
  if (!n.mean) return GLAD_OK;
  if (!n.var) return fail(GLAD_ERR_INVALID_ARG, "obs_norm: mean set but var NULL");
  if (n.n != width) return fail(GLAD_ERR_INVALID_ARG, "obs_norm covers %d columns, the group has %d", n.n, width);
  if (obs_dtype != GLAD_DTYPE_F32)
    return fail(GLAD_ERR_INVALID_ARG, "obs_norm needs f32 observations (it runs before the fp16 cast)");
  if (!(n.eps >= 0.0f) || !aligned(n.mean, 4) || !aligned(n.var, 4))
    return fail(GLAD_ERR_INVALID_ARG, "obs_norm: eps must be >= 0 and mean/var 4-byte aligned");
  return GLAD_OK;
}

int check_ql(const GladQLinear* L, const char* name, int K, int N, bool gemm = true) {
  if (!L->w8 || !L->dq_scale || !L->s_w || !L->b_prime || !L->s_z || !L->inv_sz)
    return fail(GLAD_ERR_INVALID_ARG, "%s: QuantLinear buffers must be set", name);
  if ((L->alpha == nullptr) != (L->beta == nullptr))
    return fail(GLAD_ERR_INVALID_ARG, "%s: alpha and beta must both be set or both NULL", name);
  if (K > 0 && L->in_features != K)
    return fail(GLAD_ERR_INVALID_ARG, "%s: in_features %d, expected %d", name, L->in_features, K);
  if (N > 0 && L->out_features != N)
    return fail(GLAD_ERR_INVALID_ARG, "%s: out_features %d, expected %d", name, L->out_features, N);
  if (gemm && (L->in_features <= 0 || L->in_features % 8 != 0 || L->in_features > 1024))
    return fail(GLAD_ERR_INVALID_ARG, "%s: in_features %d must be a multiple of 8 in [8, 1024]",
                name, L->in_features);
  if (!gemm && (L->in_features <= 0 || L->in_features % 4 != 0 || L->in_features > 128))
    return fail(GLAD_ERR_INVALID_ARG, "%s: in_features %d must be a multiple of 4 in [4, 128]",
                name, L->in_features);
  if (L->out_features <= 0) return fail(GLAD_ERR_INVALID_ARG, "%s: out_features must be > 0", name);
  if (!aligned(L->w8, 16))
    return fail(GLAD_ERR_INVALID_ARG, "%s: w8 must be 16-byte aligned", name);
  return GLAD_OK;
}

int front_grid(int64_t B, const DeviceInfo& d, int per_sm) {
  int64_t g = (int64_t)d.sms * per_sm;
  return (int)(B < g ? B : g);
}

// Per-call reset of the slot block (everything but the sticky status word) as a
// one-CTA kernel rather than a memset node: it lets the next kernel launch at once
// (programmatic dependent launch), so the front kernel's set-up (weights, first rows,
// TMEM, mbarriers) overlaps it; the front reads no slot before griddepcontrol.wait.
__global__ void slots_clear_kernel(float* slots) {
  grid_dep_launch();
  if (threadIdx.x < kSlotStatus) slots[threadIdx.x] = 0.0f;
}
static_assert(kSlotStatus <= 64, "one thread per cleared slot");
cudaError_t clear_slots(float* slots, cudaStream_t st) {
  slots_clear_kernel<<<1, 64, 0, st>>>(slots);
  return cudaGetLastError();
}

// Fused-forward workspace layout.
struct ActorWs {
  float* slots;
  int8_t* z8;
  __half* score_local;
  __half* pe;
  __half* enc;
  __half* h1;
  __half* h2;
  __half* h3;
  size_t bytes;
};

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// The warp-specialised front (one CTA per SM) serves the actor forward without an
// observation normaliser and outside the shared-scan actor + critic call; both fronts
// give identical results. GLAD_FRONT_WS=0 selects the pipelined front kernel.
bool use_front_ws(bool dual, bool norm) {
  if (dual || norm) return false;
  const char* env = getenv("GLAD_FRONT_WS");
  if (env && env[0] == '0') return false;
  return front_ws_usable();
}

bool use_fused_mlp(int64_t B, int act_mode, cudaStream_t st) {
  const char* env = getenv("GLAD_MLP_FUSED");
  if (env && env[0] == '0') return false;
  return (B + 127) / 128 <= (int64_t)mlp_max_tiles(act_mode, st);
}

ActorWs actor_ws(void* base, int64_t B, int enc_width = kEnc) {
  ActorWs w;
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += up256(n);
    return r;
  };
  w.slots = reinterpret_cast<float*>(take(kSlotsBytes));
  w.z8 = reinterpret_cast<int8_t*>(take((size_t)B * kTok * 16));
  w.score_local = reinterpret_cast<__half*>(take((size_t)B * kTok * 2));
  w.pe = reinterpret_cast<__half*>(take((size_t)B * kD * 2));
  w.enc = reinterpret_cast<__half*>(take((size_t)B * enc_width * 2));
  w.h1 = reinterpret_cast<__half*>(take((size_t)B * 512 * 2));
  w.h2 = reinterpret_cast<__half*>(take((size_t)B * 256 * 2));
  w.h3 = reinterpret_cast<__half*>(take((size_t)B * 128 * 2));
  w.bytes = off;
  return w;
}

}  // namespace

namespace glad {
// Error reporting for entry points defined in other translation units.
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace glad

extern "C" {

const char* glad_last_error(void) { return g_err; }

int glad_abi_version(void) { return 102; }

int glad_conv1_fused_q(const void* x_nhwc, int64_t B, const GladConvWeights* w, int8_t* z8_out,
                       void* stream) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (B == 0) return GLAD_OK;
  if (!x_nhwc || !z8_out) return fail(GLAD_ERR_INVALID_ARG, "x_nhwc and z8_out must be set");
  if (!aligned(x_nhwc, 4) || !aligned(z8_out, 16))
    return fail(GLAD_ERR_INVALID_ARG, "x_nhwc must be 4-byte and z8_out 16-byte aligned");
  int rc = check_conv(w, true, false);
  if (rc) return rc;
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  FrontParams p{};
  p.in = x_nhwc;
  p.ld = kMap;
  p.in_dtype = GLAD_DTYPE_F16;
  p.B = B;
  p.conv = *w;
  p.z8_out = z8_out;
  GLAD_CHECK_CUDA(launch_front<kModeConv1>(p, front_grid(B, d, 2), (cudaStream_t)stream),
                  "conv1 launch");
  return GLAD_OK;
}

int glad_conv2_int8_fused(const int8_t* z8, int64_t B, const GladConvWeights* w, void* feat_out,
                          int32_t* acc_out, void* stream) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (B == 0) return GLAD_OK;
  if (!z8 || !feat_out) return fail(GLAD_ERR_INVALID_ARG, "z8 and feat_out must be set");
  if (!aligned(z8, 16) || !aligned(feat_out, 16) || (acc_out && !aligned(acc_out, 16)))
    return fail(GLAD_ERR_INVALID_ARG, "z8, feat_out and acc_out must be 16-byte aligned");
  int rc = check_conv(w, false, true);
  if (rc) return rc;
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  FrontParams p{};
  p.in = z8;
  p.ld = kTok * 16;
  p.in_dtype = GLAD_DTYPE_F16;
  p.B = B;
  p.conv = *w;
  p.feat_out = reinterpret_cast<__half*>(feat_out);
  p.acc_out = acc_out;
  GLAD_CHECK_CUDA(launch_front<kModeConv2>(p, front_grid(B, d, 2), (cudaStream_t)stream),
                  "conv2 launch");
  return GLAD_OK;
}

int glad_conv_chain(const void* x_nhwc, int64_t B, const GladConvWeights* w, void* feat_out,
                    int8_t* z8_out, void* stream) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (B == 0) return GLAD_OK;
  if (!x_nhwc || !feat_out) return fail(GLAD_ERR_INVALID_ARG, "x_nhwc and feat_out must be set");
  if (!aligned(x_nhwc, 4) || !aligned(feat_out, 16) || (z8_out && !aligned(z8_out, 16)))
    return fail(GLAD_ERR_INVALID_ARG, "x_nhwc 4-byte, feat_out/z8_out 16-byte alignment required");
  int rc = check_conv(w, true, true);
  if (rc) return rc;
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  FrontParams p{};
  p.in = x_nhwc;
  p.ld = kMap;
  p.in_dtype = GLAD_DTYPE_F16;
  p.B = B;
  p.conv = *w;
  p.feat_out = reinterpret_cast<__half*>(feat_out);
  p.z8_out = z8_out;
  GLAD_CHECK_CUDA(launch_chain(p, front_grid(B, d, 2), (cudaStream_t)stream), "conv chain launch");
  return GLAD_OK;
}

size_t glad_qlinear_workspace_size(void) { return kSlotsBytes; }

int glad_qlinear_forward(const GladQLinear* L, int act_mode, const void* x, int x_dtype, int64_t M,
                         int64_t ldx, void* y, int64_t ldy, float* s_z_out, void* workspace,
                         size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  if (!L) return fail(GLAD_ERR_INVALID_ARG, "layer is NULL");
  int rc = check_ql(L, "qlinear", 0, 0);
  if (rc) return rc;
  if (act_mode != GLAD_ACT_STATIC && act_mode != GLAD_ACT_DYNAMIC)
    return fail(GLAD_ERR_INVALID_ARG, "unknown act_mode %d", act_mode);
  if (x_dtype != GLAD_DTYPE_F16 && x_dtype != GLAD_DTYPE_F32)
    return fail(GLAD_ERR_INVALID_ARG, "unknown x dtype %d", x_dtype);
  if (M < 0) return fail(GLAD_ERR_INVALID_ARG, "M must be >= 0");
  if (M == 0) return GLAD_OK;
  if (!x || !y) return fail(GLAD_ERR_INVALID_ARG, "x and y must be set");
  if (ldx < L->in_features || ldy < L->out_features)
    return fail(GLAD_ERR_INVALID_ARG, "row strides smaller than the row length");
  if (!workspace || workspace_bytes < kSlotsBytes)
    return fail(GLAD_ERR_WORKSPACE, "workspace of %zu bytes required", (size_t)kSlotsBytes);
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  float* slots = reinterpret_cast<float*>(workspace);
  GLAD_CHECK_CUDA(cudaMemsetAsync(slots, 0, kSlotsClearBytes, st), "workspace reset");
  if (act_mode == GLAD_ACT_DYNAMIC)
    GLAD_CHECK_CUDA(launch_absmax(x, x_dtype, M, ldx, L->in_features, L->alpha, L->beta, 0,
                                  &slots[0], d.sms, st),
                    "absmax launch");
  GemmParams p{};
  p.L = *L;
  p.act_mode = act_mode;
  p.slot = 0;
  p.x = x;
  p.x_dtype = x_dtype;
  p.M = M;
  p.ldx = ldx;
  if (x_dtype == GLAD_DTYPE_F16) {
    p.y = reinterpret_cast<__half*>(y);
    p.ldy = ldy;
  } else {
    p.y32 = reinterpret_cast<float*>(y);
    p.ldy32 = ldy;
  }
  p.next_slot = -1;
  p.slots = slots;
  const int N = L->out_features;
  cudaError_t le;
  if (N >= 512 && qgemm_smem_bytes(L->in_features, 128) <= 200 * 1024)
    le = launch_qgemm<128>(p, st);
  else if (N >= 256 && qgemm_smem_bytes(L->in_features, 64) <= 200 * 1024)
    le = launch_qgemm<64>(p, st);
  else
    le = launch_qgemm<32>(p, st);
  GLAD_CHECK_CUDA(le, "qlinear launch");
  if (s_z_out) {
    const float* sz[6] = {L->s_z, L->s_z, L->s_z, L->s_z, L->s_z, L->s_z};
    const int let[6] = {L->alpha != nullptr, 0, 0, 0, 0, 0};
    GLAD_CHECK_CUDA(launch_act_scales(slots, act_mode, sz, let, s_z_out, st), "scale launch");
  }
  return GLAD_OK;
}

size_t glad_actor_workspace_size(int64_t B) { return actor_ws(nullptr, B < 0 ? 0 : B).bytes; }

constexpr int kCriticEnc = 232;   // encoded row stride of the critic (128 + P <= 232)

namespace {
// Fused actor + critic: the critic head's inputs and outputs (eval mode).
struct DualArgs {
  const GladCriticWeights* wc;
  const void* critic_obs;
  int64_t ld_c;
  float* value_out;
  __half* pe_c;          // [B, 64]
  __half* enc_c;         // [B, 232]
};
struct GumbelArgs {
  uint64_t seed;
  unsigned long long* offset;
};
int actor_forward_impl(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                       int64_t ld_obs, int act_mode, const float* topk_noise, const GumbelArgs* gumbel,
                       float* mean_out, const GladActorAux* aux, void* workspace,
                       size_t workspace_bytes, void* stream, const DualArgs* dual = nullptr);
}  // namespace

int glad_actor_forward(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                       int64_t ld_obs, int act_mode, const float* topk_noise, float* mean_out,
                       const GladActorAux* aux, void* workspace, size_t workspace_bytes,
                       void* stream) {
  g_err[0] = 0;
  return actor_forward_impl(w, obs, obs_dtype, B, ld_obs, act_mode, topk_noise, nullptr, mean_out, aux,
                            workspace, workspace_bytes, stream);
}

int glad_actor_forward_train(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                             int64_t ld_obs, int act_mode, uint64_t gumbel_seed,
                             unsigned long long* gumbel_offset, float* mean_out, const GladActorAux* aux,
                             void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  if (!gumbel_offset) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset (device word) must be set");
  if (!aligned(gumbel_offset, 8)) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset must be 8-byte aligned");
  const GumbelArgs g{gumbel_seed, gumbel_offset};
  return actor_forward_impl(w, obs, obs_dtype, B, ld_obs, act_mode, nullptr, &g, mean_out, aux, workspace,
                            workspace_bytes, stream);
}

size_t glad_actor_critic_workspace_size(int64_t B) {
  const int64_t b = B < 0 ? 0 : B;
  return actor_ws(nullptr, b).bytes + up256((size_t)b * kD * 2) + up256((size_t)b * kCriticEnc * 2);
}

namespace {
int actor_critic_impl(const GladActorWeights* wa, const GladCriticWeights* wc, const void* policy_obs,
                      const void* critic_obs, int obs_dtype, int64_t B, int64_t ld_policy,
                      int64_t ld_critic, int act_mode, const GumbelArgs* gumbel, float* mean_out,
                      float* value_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!wc) return fail(GLAD_ERR_INVALID_ARG, "critic weights are NULL");
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (B == 0) return GLAD_OK;
  if (!mean_out || !value_out || !critic_obs) return fail(GLAD_ERR_INVALID_ARG, "mean_out, value_out and critic_obs must be set");
  const GladLinear16& pe = wc->proprio_emb;
  if (!pe.weight) return fail(GLAD_ERR_INVALID_ARG, "the critic proprio embedding must be the fp16 Linear");
  const int Pc = pe.in_features;
  if (Pc < 1 || Pc > 104 || pe.out_features != kD)
    return fail(GLAD_ERR_INVALID_ARG, "critic proprio embedding %dx%d; 1..104 inputs, 64 outputs", pe.out_features, Pc);
  const int hk[4] = {128 + Pc, 512, 256, 128}, hn[4] = {512, 256, 128, 1};
  for (int i = 0; i < 4; ++i) {
    const GladLinear16& L = wc->mlp[i];
    if (!L.weight || L.in_features != hk[i] || L.out_features != hn[i])
      return fail(GLAD_ERR_INVALID_ARG, "critic MLP layer %d must be fp16 %dx%d", i, hn[i], hk[i]);
  }
  if (ld_critic < Pc) return fail(GLAD_ERR_INVALID_ARG, "ld_critic %lld < %d", (long long)ld_critic, Pc);
  if (!aligned(critic_obs, obs_dtype == GLAD_DTYPE_F32 ? 4 : 2))
    return fail(GLAD_ERR_INVALID_ARG, "critic_obs is not element-aligned");
  const size_t need = glad_actor_critic_workspace_size(B);
  if (!workspace || workspace_bytes < need)
    return fail(GLAD_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  const size_t abytes = actor_ws(nullptr, B).bytes;
  uint8_t* extra = reinterpret_cast<uint8_t*>(workspace) + abytes;
  DualArgs dual{wc, critic_obs, ld_critic, value_out, reinterpret_cast<__half*>(extra),
                reinterpret_cast<__half*>(extra + up256((size_t)B * kD * 2))};
  return actor_forward_impl(wa, policy_obs, obs_dtype, B, ld_policy, act_mode, nullptr, gumbel, mean_out,
                            nullptr, workspace, abytes, stream, &dual);
}
}  // namespace

int glad_actor_critic_forward(const GladActorWeights* wa, const GladCriticWeights* wc, const void* policy_obs,
                              const void* critic_obs, int obs_dtype, int64_t B, int64_t ld_policy,
                              int64_t ld_critic, int act_mode, float* mean_out, float* value_out,
                              void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  return actor_critic_impl(wa, wc, policy_obs, critic_obs, obs_dtype, B, ld_policy, ld_critic, act_mode,
                           nullptr, mean_out, value_out, workspace, workspace_bytes, stream);
}

int glad_actor_critic_forward_train(const GladActorWeights* wa, const GladCriticWeights* wc,
                                    const void* policy_obs, const void* critic_obs, int obs_dtype,
                                    int64_t B, int64_t ld_policy, int64_t ld_critic, int act_mode,
                                    uint64_t gumbel_seed, unsigned long long* gumbel_offset,
                                    float* mean_out, float* value_out, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  if (!gumbel_offset) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset (device word) must be set");
  if (!aligned(gumbel_offset, 8)) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset must be 8-byte aligned");
  const GumbelArgs g{gumbel_seed, gumbel_offset};
  return actor_critic_impl(wa, wc, policy_obs, critic_obs, obs_dtype, B, ld_policy, ld_critic, act_mode,
                           &g, mean_out, value_out, workspace, workspace_bytes, stream);
}

namespace {
int actor_forward_impl(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                       int64_t ld_obs, int act_mode, const float* topk_noise, const GumbelArgs* gumbel,
                       float* mean_out, const GladActorAux* aux, void* workspace,
                       size_t workspace_bytes, void* stream, const DualArgs* dual) {
  if (!w) return fail(GLAD_ERR_INVALID_ARG, "weights are NULL");
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (act_mode != GLAD_ACT_STATIC && act_mode != GLAD_ACT_DYNAMIC)
    return fail(GLAD_ERR_INVALID_ARG, "unknown act_mode %d", act_mode);
  if (obs_dtype != GLAD_DTYPE_F16 && obs_dtype != GLAD_DTYPE_F32)
    return fail(GLAD_ERR_INVALID_ARG, "unknown obs dtype %d", obs_dtype);
  const int P = w->proprio_emb.in_features;
  if (P != 96)
    return fail(GLAD_ERR_INVALID_ARG, "actor proprio width %d; the fused path is built for 96", P);
  if (ld_obs < P + kMap) return fail(GLAD_ERR_INVALID_ARG, "ld_obs %lld < %d", (long long)ld_obs, P + kMap);
  if (B == 0) return GLAD_OK;
  if (!obs) return fail(GLAD_ERR_INVALID_ARG, "obs must be set");
  if (!mean_out && !(aux && aux->encoded))
    return fail(GLAD_ERR_INVALID_ARG, "encoder-only call (mean_out NULL) needs aux->encoded");
  if (!aligned(obs, obs_dtype == GLAD_DTYPE_F32 ? 4 : 2))
    return fail(GLAD_ERR_INVALID_ARG, "obs is not element-aligned");
  int rc = check_conv(&w->conv, true, true);
  if (rc) return rc;
  const GladObsNorm& nm = w->obs_norm;
  if ((rc = check_norm(nm, P + kMap, obs_dtype))) return rc;
  if (dual && (nm.mean || dual->wc->obs_norm.mean))
    return fail(GLAD_ERR_INVALID_ARG, "the fused actor + critic call reads one scan for both heads and takes "
                "no observation normalisers; run the two heads separately");
  if ((rc = check_ql(&w->proprio_emb, "actor_proprio_embedding", 96, 64, false))) return rc;
  if ((rc = check_ql(&w->query_proj, "query_projector", 128, 64))) return rc;
  const int mk[4] = {224, 512, 256, 128}, mn[4] = {512, 256, 128, kActions};
  for (int i = 0; i < 4; ++i)
    if ((rc = check_ql(&w->mlp[i], "actor MLP layer", mk[i], mn[i]))) return rc;
  if (!w->gps_w || !w->gps_b || !w->scorer_w || !w->scorer_b || !w->mha_in_w || !w->mha_in_b ||
      !w->mha_out_w || !w->mha_out_b)
    return fail(GLAD_ERR_INVALID_ARG, "fp16 encoder weights must be set");
  if (!aligned(w->mha_in_w, 16) || !aligned(w->mha_out_w, 16) || !aligned(w->query_proj.w8, 16))
    return fail(GLAD_ERR_INVALID_ARG, "MHA / query_projector weights must be 16-byte aligned");
  const ActorWs ws = actor_ws(workspace, B);
  if (!workspace || workspace_bytes < ws.bytes)
    return fail(GLAD_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", ws.bytes,
                workspace_bytes);
  if (!aligned(workspace, 256)) return fail(GLAD_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const GladActorAux none{};
  const GladActorAux& ax = aux ? *aux : none;
  int8_t* z8 = ax.z8 ? ax.z8 : ws.z8;
  __half* score_local = ax.score_local ? reinterpret_cast<__half*>(ax.score_local) : ws.score_local;
  __half* enc = ax.encoded ? reinterpret_cast<__half*>(ax.encoded) : ws.enc;
  __half* pe = ax.proprio_emb ? reinterpret_cast<__half*>(ax.proprio_emb) : ws.pe;
  if (!aligned(z8, 16) || !aligned(enc, 16) || !aligned(pe, 16) || (ax.query && !aligned(ax.query, 4)))
    return fail(GLAD_ERR_INVALID_ARG, "aux z8 / encoded / proprio_emb must be 16-byte aligned, query 4-byte");

  stage_mark(0, st);
  GLAD_CHECK_CUDA(clear_slots(ws.slots, st), "workspace reset");
  // Dynamic s_z of the proprio embedding: reduced inside the front kernel (grid
  // barrier) when its whole grid fits on the device at once, else by a separate pass.
  const bool ws_front = use_front_ws(dual != nullptr, nm.mean != nullptr);
  const int front_per_sm = ws_front ? 1 : front_fused_blocks_per_sm();
  const bool pe_absmax_in_front = act_mode == GLAD_ACT_DYNAMIC && front_per_sm > 0;
  const int fgrid = front_grid(B, d, front_per_sm > 0 && front_per_sm < 2 ? front_per_sm : 2);
  // the front follows the clear kernel or the absmax pass and waits for it before its
  // first slot access, so it may always launch early
  const bool front_pdl = true;
  if (act_mode == GLAD_ACT_DYNAMIC && !pe_absmax_in_front)
    GLAD_CHECK_CUDA(launch_absmax(obs, obs_dtype, B, ld_obs, P, w->proprio_emb.alpha,
                                  w->proprio_emb.beta, 1, &ws.slots[0], d.sms, st, nm.mean, nm.var, nm.eps),
                    "absmax launch");
  stage_mark(1, st);
  FrontParams fp{};
  fp.in = obs;
  fp.ld = ld_obs;
  fp.in_dtype = obs_dtype;
  fp.prop_dim = P;
  fp.B = B;
  fp.conv = w->conv;
  fp.gps_w = reinterpret_cast<const __half*>(w->gps_w);
  fp.gps_b = reinterpret_cast<const __half*>(w->gps_b);
  fp.scorer_w = reinterpret_cast<const __half*>(w->scorer_w);
  fp.pe = w->proprio_emb;
  fp.qp = w->query_proj;
  fp.act_mode = act_mode;
  fp.ld_enc = kEnc;
  fp.z8_out = z8;
  fp.feat_out = reinterpret_cast<__half*>(ax.local);
  fp.score_local = score_local;
  fp.gc_w_out = reinterpret_cast<__half*>(ax.gc_weights);
  fp.enc = enc;
  fp.pe_out = pe;
  fp.slots = ws.slots;
  fp.pe_absmax = pe_absmax_in_front ? 1 : 0;
  fp.norm_mean = nm.mean;
  fp.norm_var = nm.var;
  fp.norm_eps = nm.eps;
  if (dual) {
    fp.dual = 1;
    fp.in_c = dual->critic_obs;
    fp.ld_c = dual->ld_c;
    fp.prop_dim_c = dual->wc->proprio_emb.in_features;
    fp.pec_w = reinterpret_cast<const __half*>(dual->wc->proprio_emb.weight);
    fp.pec_b = reinterpret_cast<const __half*>(dual->wc->proprio_emb.bias);
    fp.ld_enc_c = kCriticEnc;
    fp.enc_c = dual->enc_c;
    fp.pe_c_out = dual->pe_c;
  }
  GLAD_CHECK_CUDA(ws_front ? launch_front_ws(fp, fgrid, st, front_pdl) : launch_front<kModeFront>(fp, fgrid, st, front_pdl),
                  "front launch");
  stage_mark(2, st);

  TailParams tp{};
  tp.B = B;
  tp.conv = w->conv;
  tp.qp = w->query_proj;
  tp.scorer_w = reinterpret_cast<const __half*>(w->scorer_w);
  tp.scorer_b = reinterpret_cast<const __half*>(w->scorer_b);
  tp.in_w = reinterpret_cast<const __half*>(w->mha_in_w);
  tp.in_b = reinterpret_cast<const __half*>(w->mha_in_b);
  tp.out_w = reinterpret_cast<const __half*>(w->mha_out_w);
  tp.out_b = reinterpret_cast<const __half*>(w->mha_out_b);
  tp.a0_alpha = w->mlp[0].alpha;
  tp.a0_beta = w->mlp[0].beta;
  tp.a0_absmax = 1;
  tp.qp_slot = 1;
  tp.act_mode = act_mode;
  tp.ld_enc = kEnc;
  tp.prop_dim = P;
  tp.noise = topk_noise;
  tp.gumbel = gumbel ? 1 : 0;
  tp.gumbel_seed = gumbel ? gumbel->seed : 0;
  tp.gumbel_offset = gumbel ? gumbel->offset : nullptr;
  tp.done_slot = kSlotTailDone;
  tp.z8 = z8;
  tp.score_local = score_local;
  tp.pe = pe;
  tp.enc = enc;
  tp.topk_logits_out = reinterpret_cast<__half*>(ax.topk_logits);
  tp.topk_idx_out = ax.topk_idx;
  tp.attn_w_out = reinterpret_cast<__half*>(ax.attn_weights);
  tp.query_out = reinterpret_cast<__half*>(ax.query);
  tp.slots = ws.slots;
  GLAD_CHECK_CUDA(launch_tail(tp, tail_grid(B, d.sms), st, true), "tail launch");
  stage_mark(3, st);

  // Actor MLP: one fused kernel when the grid fits on the device at once (its
  // dynamic-s_z grid barrier needs every CTA resident), else one GEMM per layer.
  // GLAD_MLP_FUSED=0 selects the per-layer kernels.
  bool fused_mlp = false;
  if (mean_out) {
    bool w_ok = true;
    for (int i = 0; i < 4; ++i) w_ok = w_ok && aligned(w->mlp[i].w8, 16);
    if (w_ok && use_fused_mlp(B, act_mode, st)) {
      GLAD_CHECK_CUDA(launch_mlp(w->mlp, act_mode, enc, B, kEnc, mean_out, kActions, ws.slots, st, true),
                      "fused actor MLP launch");
      fused_mlp = true;
      for (int i = 0; i < 4; ++i) stage_mark(4 + i, st);
    }
  }
  __half* hs[4] = {enc, ws.h1, ws.h2, ws.h3};
  for (int i = 0; i < (mean_out && !fused_mlp ? 4 : 0); ++i) {
    GemmParams g{};
    g.L = w->mlp[i];
    g.act_mode = act_mode;
    g.slot = 2 + i;
    g.x = hs[i];
    g.x_dtype = GLAD_DTYPE_F16;
    g.M = B;
    g.ldx = mk[i];
    g.slots = ws.slots;
    if (i < 3) {
      g.y = hs[i + 1];
      g.ldy = mn[i];
      g.elu = 1;
      g.next_alpha = w->mlp[i + 1].alpha;
      g.next_beta = w->mlp[i + 1].beta;
      g.next_let = w->mlp[i + 1].alpha != nullptr;
      g.next_slot = 3 + i;
      // N tile chosen so each layer launches ~B/128 x 4 CTAs
      cudaError_t le = mn[i] >= 512 ? launch_qgemm<128>(g, st, true)
                       : mn[i] >= 256 ? launch_qgemm<64>(g, st, true) : launch_qgemm<32>(g, st, true);
      GLAD_CHECK_CUDA(le, "actor MLP launch");
    } else {
      g.y32 = mean_out;
      g.ldy32 = kActions;
      g.y32_round16 = 1;                   // mean = fp16 output .float() (integration.py:206)
      g.next_slot = -1;
      GLAD_CHECK_CUDA(launch_qgemm<32>(g, st, true), "actor head launch");
    }
    stage_mark(4 + i, st);
  }
  if (dual) {
    // critic head on the shared front: its own query, top-32, attention, fp16 MLP
    TailParams tc = tp;
    tc.a0_absmax = 0;
    tc.qp_slot = kSlotCriticQp;
    tc.ld_enc = kCriticEnc;
    tc.prop_dim = dual->wc->proprio_emb.in_features;
    tc.noise = nullptr;
    // train mode: the critic draws its own Gumbel term at the offset the actor tail
    // has advanced (the MLP launched in between waits for the actor tail to finish)
    tc.done_slot = kSlotCriticTailDone;
    tc.pe = dual->pe_c;
    tc.enc = dual->enc_c;
    tc.topk_logits_out = nullptr;
    tc.topk_idx_out = nullptr;
    tc.attn_w_out = nullptr;
    tc.query_out = nullptr;
    GLAD_CHECK_CUDA(launch_tail(tc, tail_grid(B, d.sms), st, true), "critic tail launch");
    GladLinear16 L[4] = {dual->wc->mlp[0], dual->wc->mlp[1], dual->wc->mlp[2], dual->wc->mlp[3]};
    GLAD_CHECK_CUDA(launch_f16mlp(L, dual->enc_c, B, kCriticEnc, dual->value_out, 1,
                                  reinterpret_cast<unsigned int*>(&ws.slots[kSlotStatus]), st, true),
                    "critic MLP launch");
  }
  if (ax.act_scales) {
    const float* sz[6] = {w->proprio_emb.s_z, w->query_proj.s_z, w->mlp[0].s_z,
                          w->mlp[1].s_z, w->mlp[2].s_z, w->mlp[3].s_z};
    const int let[6] = {w->proprio_emb.alpha != nullptr, w->query_proj.alpha != nullptr,
                        w->mlp[0].alpha != nullptr, w->mlp[1].alpha != nullptr,
                        w->mlp[2].alpha != nullptr, w->mlp[3].alpha != nullptr};
    GLAD_CHECK_CUDA(launch_act_scales(ws.slots, act_mode, sz, let, ax.act_scales, st),
                    "scale launch");
  }
  return GLAD_OK;
}

}  // namespace


size_t glad_critic_workspace_size(int64_t B) {
  return actor_ws(nullptr, B < 0 ? 0 : B, kCriticEnc).bytes;
}

namespace {
int critic_forward_impl(const GladCriticWeights* w, const void* obs, int obs_dtype, int64_t B,
                        int64_t ld_obs, int act_mode, const float* topk_noise, const GumbelArgs* gumbel,
                        float* value_out, const GladActorAux* aux, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!w) return fail(GLAD_ERR_INVALID_ARG, "weights are NULL");
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (act_mode != GLAD_ACT_STATIC && act_mode != GLAD_ACT_DYNAMIC)
    return fail(GLAD_ERR_INVALID_ARG, "unknown act_mode %d", act_mode);
  if (obs_dtype != GLAD_DTYPE_F16 && obs_dtype != GLAD_DTYPE_F32)
    return fail(GLAD_ERR_INVALID_ARG, "unknown obs dtype %d", obs_dtype);
  const bool pe16 = w->proprio_emb.weight != nullptr;
  int rc;
  int P;
  if (pe16) {
    P = w->proprio_emb.in_features;
    if (w->proprio_emb.out_features != kD)
      return fail(GLAD_ERR_INVALID_ARG, "critic_proprio_embedding must have 64 outputs");
  } else {
    if ((rc = check_ql(&w->proprio_emb_q, "proprio embedding", 0, kD, false))) return rc;
    P = w->proprio_emb_q.in_features;
  }
  if (P <= 0 || P > 104) return fail(GLAD_ERR_INVALID_ARG, "critic proprio width %d outside [1, 104]", P);
  if (ld_obs < P + kMap) return fail(GLAD_ERR_INVALID_ARG, "ld_obs %lld < %d", (long long)ld_obs, P + kMap);
  if (B == 0) return GLAD_OK;
  if (!obs) return fail(GLAD_ERR_INVALID_ARG, "obs must be set");
  if (!value_out && !(aux && aux->encoded))
    return fail(GLAD_ERR_INVALID_ARG, "encoder-only call (value_out NULL) needs aux->encoded");
  if (!aligned(obs, obs_dtype == GLAD_DTYPE_F32 ? 4 : 2))
    return fail(GLAD_ERR_INVALID_ARG, "obs is not element-aligned");
  if ((rc = check_conv(&w->conv, true, true))) return rc;
  if ((rc = check_norm(w->obs_norm, P + kMap, obs_dtype))) return rc;
  if ((rc = check_ql(&w->query_proj, "query_projector", 128, 64))) return rc;
  const int hk[4] = {128 + P, 512, 256, 128}, hn[4] = {512, 256, 128, 1};
  for (int i = 0; i < 4; ++i) {
    const GladLinear16& L = w->mlp[i];
    if (!L.weight || L.in_features != hk[i] || L.out_features != hn[i])
      return fail(GLAD_ERR_INVALID_ARG, "critic MLP layer %d must be %d -> %d", i, hk[i], hn[i]);
  }
  if (!w->gps_w || !w->gps_b || !w->scorer_w || !w->scorer_b || !w->mha_in_w || !w->mha_in_b ||
      !w->mha_out_w || !w->mha_out_b)
    return fail(GLAD_ERR_INVALID_ARG, "fp16 encoder weights must be set");
  const ActorWs ws = actor_ws(workspace, B, kCriticEnc);
  if (!workspace || workspace_bytes < ws.bytes)
    return fail(GLAD_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", ws.bytes, workspace_bytes);
  if (!aligned(workspace, 256)) return fail(GLAD_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const GladActorAux none{};
  const GladActorAux& ax = aux ? *aux : none;
  int8_t* z8 = ax.z8 ? ax.z8 : ws.z8;
  __half* score_local = ax.score_local ? reinterpret_cast<__half*>(ax.score_local) : ws.score_local;
  __half* enc = ax.encoded ? reinterpret_cast<__half*>(ax.encoded) : ws.enc;
  __half* pe = ax.proprio_emb ? reinterpret_cast<__half*>(ax.proprio_emb) : ws.pe;
  if (!aligned(z8, 16) || !aligned(enc, 16) || !aligned(pe, 16) || (ax.query && !aligned(ax.query, 4)))
    return fail(GLAD_ERR_INVALID_ARG, "aux z8 / encoded / proprio_emb must be 16-byte aligned, query 4-byte");

  GLAD_CHECK_CUDA(clear_slots(ws.slots, st), "workspace reset");
  const bool absmax_pass = !pe16 && act_mode == GLAD_ACT_DYNAMIC;
  const bool front_pdl = true;          // after the clear kernel or the absmax pass (both kernels)
  if (absmax_pass)
    GLAD_CHECK_CUDA(launch_absmax(obs, obs_dtype, B, ld_obs, P, w->proprio_emb_q.alpha,
                                  w->proprio_emb_q.beta, 1, &ws.slots[0], d.sms, st, w->obs_norm.mean,
                                  w->obs_norm.var, w->obs_norm.eps),
                    "absmax launch");
  FrontParams fp{};
  fp.in = obs;
  fp.ld = ld_obs;
  fp.in_dtype = obs_dtype;
  fp.prop_dim = P;
  fp.B = B;
  fp.conv = w->conv;
  fp.gps_w = reinterpret_cast<const __half*>(w->gps_w);
  fp.gps_b = reinterpret_cast<const __half*>(w->gps_b);
  fp.scorer_w = reinterpret_cast<const __half*>(w->scorer_w);
  fp.pe_f16 = pe16 ? 1 : 0;
  fp.pe = w->proprio_emb_q;
  fp.pe16_w = reinterpret_cast<const __half*>(w->proprio_emb.weight);
  fp.pe16_b = reinterpret_cast<const __half*>(w->proprio_emb.bias);
  fp.norm_mean = w->obs_norm.mean;
  fp.norm_var = w->obs_norm.var;
  fp.norm_eps = w->obs_norm.eps;
  fp.qp = w->query_proj;
  fp.act_mode = act_mode;
  fp.ld_enc = kCriticEnc;
  fp.z8_out = z8;
  fp.feat_out = reinterpret_cast<__half*>(ax.local);
  fp.score_local = score_local;
  fp.gc_w_out = reinterpret_cast<__half*>(ax.gc_weights);
  fp.enc = enc;
  fp.pe_out = pe;
  fp.slots = ws.slots;
  GLAD_CHECK_CUDA(launch_front<kModeFront>(fp, front_grid(B, d, 2), st, front_pdl), "front launch");

  TailParams tp{};
  tp.B = B;
  tp.conv = w->conv;
  tp.qp = w->query_proj;
  tp.scorer_w = reinterpret_cast<const __half*>(w->scorer_w);
  tp.scorer_b = reinterpret_cast<const __half*>(w->scorer_b);
  tp.in_w = reinterpret_cast<const __half*>(w->mha_in_w);
  tp.in_b = reinterpret_cast<const __half*>(w->mha_in_b);
  tp.out_w = reinterpret_cast<const __half*>(w->mha_out_w);
  tp.out_b = reinterpret_cast<const __half*>(w->mha_out_b);
  tp.a0_absmax = 0;                 // the critic MLP is fp16: no scale to reduce
  tp.qp_slot = 1;
  tp.noise = topk_noise;
  tp.gumbel = gumbel ? 1 : 0;
  tp.gumbel_seed = gumbel ? gumbel->seed : 0;
  tp.gumbel_offset = gumbel ? gumbel->offset : nullptr;
  tp.done_slot = kSlotTailDone;
  tp.act_mode = act_mode;
  tp.ld_enc = kCriticEnc;
  tp.prop_dim = P;
  tp.z8 = z8;
  tp.score_local = score_local;
  tp.pe = pe;
  tp.enc = enc;
  tp.topk_logits_out = reinterpret_cast<__half*>(ax.topk_logits);
  tp.topk_idx_out = ax.topk_idx;
  tp.attn_w_out = reinterpret_cast<__half*>(ax.attn_weights);
  tp.query_out = reinterpret_cast<__half*>(ax.query);
  tp.slots = ws.slots;
  GLAD_CHECK_CUDA(launch_tail(tp, tail_grid(B, d.sms), st, true), "tail launch");

  // fp16 critic MLP: one cluster kernel (fp16 activations, tcgen05 kind::f16)
  if (value_out) {
    GladLinear16 L[4] = {w->mlp[0], w->mlp[1], w->mlp[2], w->mlp[3]};
    GLAD_CHECK_CUDA(launch_f16mlp(L, enc, B, kCriticEnc, value_out, 1,
                                  reinterpret_cast<unsigned int*>(&ws.slots[kSlotStatus]), st, true),
                    "critic MLP launch");
  }
  return GLAD_OK;
}
}  // namespace

int glad_critic_forward(const GladCriticWeights* w, const void* obs, int obs_dtype, int64_t B,
                        int64_t ld_obs, int act_mode, const float* topk_noise, float* value_out,
                        const GladActorAux* aux, void* workspace, size_t workspace_bytes,
                        void* stream) {
  g_err[0] = 0;
  return critic_forward_impl(w, obs, obs_dtype, B, ld_obs, act_mode, topk_noise, nullptr, value_out, aux,
                             workspace, workspace_bytes, stream);
}

int glad_critic_forward_train(const GladCriticWeights* w, const void* obs, int obs_dtype, int64_t B,
                              int64_t ld_obs, int act_mode, uint64_t gumbel_seed,
                              unsigned long long* gumbel_offset, float* value_out, const GladActorAux* aux,
                              void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  if (!gumbel_offset) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset (device word) must be set");
  if (!aligned(gumbel_offset, 8)) return fail(GLAD_ERR_INVALID_ARG, "gumbel_offset must be 8-byte aligned");
  const GumbelArgs g{gumbel_seed, gumbel_offset};
  return critic_forward_impl(w, obs, obs_dtype, B, ld_obs, act_mode, nullptr, &g, value_out, aux, workspace,
                             workspace_bytes, stream);
}

namespace {
int check_w4(const GladW4Linear* mlp) {
  if (!mlp) return fail(GLAD_ERR_INVALID_ARG, "W4A16 layers are NULL");
  const int mk[4] = {224, 512, 256, 128}, mn[4] = {512, 256, 128, kActions};
  for (int i = 0; i < 4; ++i) {
    const GladW4Linear& L = mlp[i];
    if (!L.packed || !L.scales)
      return fail(GLAD_ERR_INVALID_ARG, "W4A16 layer %d: packed weights and scales must be set", i);
    if (L.in_features != mk[i] || L.out_features != mn[i])
      return fail(GLAD_ERR_INVALID_ARG, "W4A16 layer %d: %dx%d, expected %dx%d", i, L.out_features,
                  L.in_features, mn[i], mk[i]);
    if (!aligned(L.packed, 16) || !aligned(L.scales, 2) || (L.bias && !aligned(L.bias, 2)))
      return fail(GLAD_ERR_INVALID_ARG, "W4A16 layer %d: packed weights must be 16-byte aligned", i);
  }
  return GLAD_OK;
}
}  // namespace

int glad_w4a16_mlp_forward(const GladW4Linear* mlp, const void* x, int64_t M, int64_t ldx, float* mean_out,
                           void* stream) {
  g_err[0] = 0;
  int rc = check_w4(mlp);
  if (rc) return rc;
  if (M < 0) return fail(GLAD_ERR_INVALID_ARG, "M must be >= 0");
  if (M == 0) return GLAD_OK;
  if (!x || !mean_out) return fail(GLAD_ERR_INVALID_ARG, "x and mean_out must be set");
  if (ldx < 224 || ldx % 8 != 0 || !aligned(x, 16))
    return fail(GLAD_ERR_INVALID_ARG, "x: 16-byte aligned rows, ldx a multiple of 8 and >= 224");
  DeviceInfo d;
  if ((rc = device_info(&d))) return rc;
  GladW4Linear L[4] = {mlp[0], mlp[1], mlp[2], mlp[3]};
  GLAD_CHECK_CUDA(launch_w4mlp(L, reinterpret_cast<const __half*>(x), M, ldx, mean_out, kActions, nullptr,
                               (cudaStream_t)stream, false),
                  "W4A16 MLP launch");
  return GLAD_OK;
}

int glad_actor_forward_w4a16(const GladActorWeights* w, const GladW4Linear* mlp, const void* obs,
                             int obs_dtype, int64_t B, int64_t ld_obs, int act_mode, float* mean_out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  int rc = check_w4(mlp);
  if (rc) return rc;
  if (!mean_out) return fail(GLAD_ERR_INVALID_ARG, "mean_out must be set");
  if (B <= 0) return B == 0 ? GLAD_OK : fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  // the INT8 encoder writes `encoded` into the workspace; then the W4A16 MLP reads it
  const ActorWs ws = actor_ws(workspace, B);
  GladActorAux ax{};
  ax.encoded = ws.enc;
  if ((rc = actor_forward_impl(w, obs, obs_dtype, B, ld_obs, act_mode, nullptr, nullptr, nullptr, &ax,
                               workspace, workspace_bytes, stream)))
    return rc;
  GladW4Linear L[4] = {mlp[0], mlp[1], mlp[2], mlp[3]};
  GLAD_CHECK_CUDA(launch_w4mlp(L, ws.enc, B, kEnc, mean_out, kActions,
                               reinterpret_cast<unsigned int*>(&ws.slots[kSlotStatus]), (cudaStream_t)stream,
                               true),
                  "W4A16 MLP launch");
  return GLAD_OK;
}

int glad_actor_mlp_fused(int64_t B, int act_mode) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (act_mode != GLAD_ACT_STATIC && act_mode != GLAD_ACT_DYNAMIC)
    return fail(GLAD_ERR_INVALID_ARG, "unknown act_mode %d", act_mode);
  DeviceInfo d;
  int rc = device_info(&d);
  if (rc) return rc;
  return use_fused_mlp(B, act_mode, 0) ? 1 : 0;
}

int glad_actor_kernel_count(int64_t B, int act_mode) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (act_mode != GLAD_ACT_STATIC && act_mode != GLAD_ACT_DYNAMIC)
    return fail(GLAD_ERR_INVALID_ARG, "unknown act_mode %d", act_mode);
  DeviceInfo d;
  int rc = device_info(&d);
  if (rc) return rc;
  if (B == 0) return 0;
  const bool absmax_pass =
      act_mode == GLAD_ACT_DYNAMIC && !use_front_ws(false, false) && front_fused_blocks_per_sm() <= 0;
  return 3 + (absmax_pass ? 1 : 0) + (use_fused_mlp(B, act_mode, 0) ? 1 : 4);   // clear + front + tail + MLP
}

int glad_actor_stage_events(void* const* events, int n) {
  g_err[0] = 0;
  if (n < 0 || n > 16 || (n > 0 && !events))
    return fail(GLAD_ERR_INVALID_ARG, "0..16 events required");
  for (int i = 0; i < n; ++i) g_stage_ev[i] = reinterpret_cast<cudaEvent_t>(events[i]);
  g_stage_n = n;
  return GLAD_OK;
}

int glad_workspace_status(void* workspace, uint32_t* status, void* stream) {
  g_err[0] = 0;
  if (!workspace || !status) return fail(GLAD_ERR_INVALID_ARG, "workspace and status must be set");
  cudaStream_t st = (cudaStream_t)stream;
  float* slots = reinterpret_cast<float*>(workspace);
  GLAD_CHECK_CUDA(cudaMemcpyAsync(status, slots + kSlotStatus, sizeof(uint32_t),
                                  cudaMemcpyDeviceToHost, st),
                  "status copy");
  GLAD_CHECK_CUDA(cudaMemsetAsync(slots + kSlotStatus, 0, sizeof(uint32_t), st),
                  "status clear");
  GLAD_CHECK_CUDA(cudaStreamSynchronize(st), "status sync");
  return *status ? fail(GLAD_ERR_DEVICE, "device status 0x%x (a bounded device-side wait ran out: the "
                        "results of the launches since the last status read are not valid)", *status)
                 : GLAD_OK;
}

int glad_requant_qlinear(const GladQLinearSrc* layers, int n, void* stream) {
  g_err[0] = 0;
  if (n < 0 || n > 16) return fail(GLAD_ERR_INVALID_ARG, "between 0 and 16 layers per call");
  if (n == 0) return GLAD_OK;
  if (!layers) return fail(GLAD_ERR_INVALID_ARG, "layers is NULL");
  for (int i = 0; i < n; ++i) {
    const GladQLinearSrc& l = layers[i];
    if (!l.weight || !l.w8 || !l.dq_scale || !l.s_w || !l.b_prime || !l.s_z)
      return fail(GLAD_ERR_INVALID_ARG, "layer %d: buffers must be set", i);
    if (l.N <= 0 || l.K <= 0 || l.Np < l.N)
      return fail(GLAD_ERR_INVALID_ARG, "layer %d: bad sizes N=%d K=%d Np=%d", i, l.N, l.K, l.Np);
    if (l.w_dtype != GLAD_DTYPE_F16 && l.w_dtype != GLAD_DTYPE_F32)
      return fail(GLAD_ERR_INVALID_ARG, "layer %d: unknown dtype", i);
  }
  GLAD_CHECK_CUDA(launch_requant_qlinear(layers, n, (cudaStream_t)stream), "requant launch");
  return GLAD_OK;
}

int glad_requant_qcnn(const GladQCNNSrc* s, void* stream) {
  g_err[0] = 0;
  if (s && s->dtype != GLAD_DTYPE_F16 && s->dtype != GLAD_DTYPE_F32)
    return fail(GLAD_ERR_INVALID_ARG, "QuantCNN requant: unknown dtype %d", s->dtype);
  if (s && (s->alpha == nullptr) != (s->beta == nullptr))
    return fail(GLAD_ERR_INVALID_ARG, "QuantCNN requant: alpha and beta must both be set or NULL");
  if (!s || !s->conv1_w || !s->conv1_b || !s->bn1_w || !s->bn1_b || !s->bn1_mean || !s->bn1_var ||
      !s->conv2_w || !s->conv2_b || !s->bn2_w || !s->bn2_b || !s->bn2_mean || !s->bn2_var ||
      !s->s_z || !s->w1p || !s->b1f || !s->qa || !s->qc || !s->w8 || !s->dq || !s->b2f || !s->a2 ||
      !s->c2)
    return fail(GLAD_ERR_INVALID_ARG, "QuantCNN requant: every buffer must be set");
  GLAD_CHECK_CUDA(launch_requant_qcnn(*s, (cudaStream_t)stream), "requant launch");
  return GLAD_OK;
}

int glad_cast_copy(const GladCastCopy* items, int n, void* stream) {
  g_err[0] = 0;
  if (n < 0) return fail(GLAD_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return GLAD_OK;
  if (!items) return fail(GLAD_ERR_INVALID_ARG, "items is NULL");
  for (int i = 0; i < n; ++i) {
    const GladCastCopy& c = items[i];
    if ((!c.src || !c.dst) && c.n > 0) return fail(GLAD_ERR_INVALID_ARG, "item %d: NULL pointer", i);
    if ((c.src_dtype != GLAD_DTYPE_F16 && c.src_dtype != GLAD_DTYPE_F32) ||
        (c.dst_dtype != GLAD_DTYPE_F16 && c.dst_dtype != GLAD_DTYPE_F32))
      return fail(GLAD_ERR_INVALID_ARG, "item %d: unknown dtype", i);
  }
  GLAD_CHECK_CUDA(launch_cast_copy(items, n, (cudaStream_t)stream), "cast-copy launch");
  return GLAD_OK;
}

int glad_ppo_epilogue(const float* mean, int64_t B, int64_t ld_mean, const float* std, int n_actions,
                      uint64_t seed, unsigned long long* rng_state, float* actions, int64_t ld_actions,
                      float* log_prob, float* sigma_out, void* stream) {
  g_err[0] = 0;
  if (B < 0) return fail(GLAD_ERR_INVALID_ARG, "B must be >= 0");
  if (n_actions < 1 || n_actions > 64) return fail(GLAD_ERR_INVALID_ARG, "n_actions %d; 1..64", n_actions);
  if (B == 0) return GLAD_OK;
  if (!mean || !std || !rng_state || !actions || !log_prob)
    return fail(GLAD_ERR_INVALID_ARG, "mean, std, rng_state, actions and log_prob must be set");
  if (ld_mean < n_actions || ld_actions < n_actions)
    return fail(GLAD_ERR_INVALID_ARG, "row strides must be >= n_actions");
  if (!aligned(rng_state, 8)) return fail(GLAD_ERR_INVALID_ARG, "rng_state must be 8-byte aligned");
  if (!aligned(mean, 4) || !aligned(std, 4) || !aligned(actions, 4) || !aligned(log_prob, 4) ||
      !aligned(sigma_out, 4))
    return fail(GLAD_ERR_INVALID_ARG, "f32 buffers must be 4-byte aligned");
  PpoParams p{};
  p.mean = mean;
  p.ld_mean = ld_mean;
  p.std = std;
  p.n = n_actions;
  p.B = B;
  p.seed = seed;
  p.rng = rng_state;
  p.actions = actions;
  p.ld_act = ld_actions;
  p.log_prob = log_prob;
  p.sigma = sigma_out;
  GLAD_CHECK_CUDA(launch_ppo_epilogue(p, (cudaStream_t)stream, true), "PPO epilogue launch");
  return GLAD_OK;
}

}  // extern "C"
