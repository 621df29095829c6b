/*
 * glad_b200.h -- C ABI of the B200 (sm_100a) GLAD rollout forward.
 *
 * Plain pointers and sizes only. Every device pointer is a CUDA device
 * address owned by the caller; `stream` is a cudaStream_t passed as void*.
 * Functions return GLAD_OK (0) or a negative GLAD_ERR_* code; no exception
 * crosses the ABI and glad_last_error() returns a message for the calling
 * thread's last failure. Launches are asynchronous on `stream` and allocate
 * nothing: scratch memory is the caller's `workspace`.
 *
 * Data types: "f16" = IEEE binary16, "f32" = binary32, "i8" = int8.
 * Tensor layouts are the ones of the reference's qrt package (RL_Quant).
 */
#ifndef GLAD_B200_H_
#define GLAD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLAD_OK 0
#define GLAD_ERR_INVALID_ARG (-1)  /* bad pointer, size, alignment or mode */
#define GLAD_ERR_CUDA (-2)         /* a CUDA runtime call failed            */
#define GLAD_ERR_DEVICE (-3)       /* a kernel reported a device-side error */
#define GLAD_ERR_UNSUPPORTED (-4)  /* no sm_100 device / feature not built   */
#define GLAD_ERR_WORKSPACE (-5)    /* workspace missing or too small         */

#define GLAD_DTYPE_F32 0
#define GLAD_DTYPE_F16 1

#define GLAD_ACT_STATIC 0   /* qrt QuantLinear act_mode="static"  (qrt/qlinear.py:132-135) */
#define GLAD_ACT_DYNAMIC 1  /* qrt QuantLinear act_mode="dynamic" (qrt/qlinear.py:125-131) */

/* Last error message of the calling thread ("" when none). */
const char* glad_last_error(void);

/* ABI version (major * 100 + minor). */
int glad_abi_version(void);

/* ---- weights ---------------------------------------------------------------
 * QuantCNN buffers (qrt/qconv.py:236-244, filled by requantize_ :247-284):
 *   w1p [128,16] f16 (k = kh*16 + kw*3 + c), b1f/qa/qc [16] f32,
 *   w8 [3,64,64] i8 (kh; ks = kw*16 + c; n), dq/b2f/a2/c2 [64] f32.        */
typedef struct GladConvWeights {
  const void* w1p;
  const float* b1f;
  const float* qa;
  const float* qc;
  const int8_t* w8;
  const float* dq;
  const float* b2f;
  const float* a2;
  const float* c2;
} GladConvWeights;

/* QuantLinear buffers (qrt/qlinear.py:58-81): w8 [Np,K] i8 row-major,
 * dq_scale/s_w/b_prime [Np] f32, alpha/beta [K] f32 (NULL without LET),
 * s_z/inv_sz 0-d f32. Np = out_features rounded up to a multiple of 8.     */
typedef struct GladQLinear {
  const int8_t* w8;
  const float* dq_scale;
  const float* s_w;
  const float* b_prime;
  const float* alpha;
  const float* beta;
  const float* s_z;
  const float* inv_sz;
  int32_t in_features;
  int32_t out_features;
} GladQLinear;

/* rsl_rl EmpiricalNormalization of one observation group
 * (rsl_rl/networks/normalization.py:44-47), applied while the rows are loaded:
 * x' = (x - mean) / (sqrt(var) + eps), every step an fp32 operation, then the
 * fp16 cast of qrt's `actor_obs.half()` (qrt/integration.py:206). sqrt(var) is
 * the module's `_std`, which it recomputes from `_var`; `_mean` and `_var` are
 * updated in place, so captured graphs stay valid. mean = NULL: identity.
 * n = the group's width; the observations must be f32.                       */
typedef struct GladObsNorm {
  const float* mean;             /* [n] f32 (_mean)                          */
  const float* var;              /* [n] f32 (_var)                           */
  float eps;                     /* the module's eps as f32                  */
  int32_t n;
} GladObsNorm;

/* Every tensor the fused actor forward reads (qrt full mode: QuantCNN,
 * LET W8A8 on actor_proprio_embedding, query_projector, actor.0/2/4/6;
 * fp16 GPS selector, top-k scorer and MHA, qrt/integration.py:42-43).     */
typedef struct GladActorWeights {
  GladConvWeights conv;          /* map_cnn (QuantCNN)                      */
  GladQLinear proprio_emb;       /* actor_proprio_embedding, 96 -> 64        */
  GladQLinear query_proj;        /* query_projector, 128 -> 64               */
  const void* gps_w;             /* global_pool_selector.weight f16 [1,64]   */
  const void* gps_b;             /* global_pool_selector.bias   f16 [1]      */
  const void* scorer_w;          /* topk_scorer.weight f16 [1,128]           */
  const void* scorer_b;          /* topk_scorer.bias   f16 [1]               */
  const void* mha_in_w;          /* mha.in_proj_weight f16 [192,64]          */
  const void* mha_in_b;          /* mha.in_proj_bias   f16 [192]             */
  const void* mha_out_w;         /* mha.out_proj.weight f16 [64,64]          */
  const void* mha_out_b;         /* mha.out_proj.bias   f16 [64]             */
  GladQLinear mlp[4];            /* actor.0 224->512, .2 ->256, .4 ->128, .6 ->29 */
  GladObsNorm obs_norm;          /* actor_obs_normalizer (mean NULL: identity) */
} GladActorWeights;

/* Plain fp16 Linear (weight [out,in] f16 row-major, bias [out] f16 or NULL). */
typedef struct GladLinear16 {
  const void* weight;
  const void* bias;
  int32_t in_features;
  int32_t out_features;
} GladLinear16;

/* The critic forward's tensors (qrt/integration.py:133-135): the shared
 * encoder (QuantCNN, INT8 query_projector, fp16 GPS/scorer/MHA), the critic
 * proprio embedding and the fp16 critic MLP (not quantised,
 * qrt/integration.py:42-43). When the critic observation has the actor's
 * proprio width the reference encodes it with actor_proprio_embedding
 * (rsl_rl actor_critic_encoder.py:226-229): then set proprio_emb_q and leave
 * proprio_emb.weight NULL.                                                    */
typedef struct GladCriticWeights {
  GladConvWeights conv;
  GladLinear16 proprio_emb;      /* critic_proprio_embedding, P -> 64 (fp16)    */
  GladQLinear proprio_emb_q;     /* used when proprio_emb.weight is NULL       */
  GladQLinear query_proj;
  const void* gps_w;
  const void* gps_b;
  const void* scorer_w;
  const void* scorer_b;
  const void* mha_in_w;
  const void* mha_in_b;
  const void* mha_out_w;
  const void* mha_out_b;
  GladLinear16 mlp[4];           /* critic.0 (128+P)->512, .2 ->256, .4 ->128, .6 ->1 */
  GladObsNorm obs_norm;          /* critic_obs_normalizer (mean NULL: identity) */
} GladCriticWeights;

/* Optional per-call outputs of the fused forward (any field may be NULL). */
typedef struct GladActorAux {
  int8_t* z8;            /* [B*187,16] i8   conv1 output (QuantCNN z8)          */
  void* local;           /* [B,187,64] f16  local features (conv2 output)       */
  void* gc_weights;      /* [B,187]   f16   global softmax pool weights         */
  void* score_local;     /* [B,187]   f16   scorer logits of the local half     */
  void* topk_logits;     /* [B,187]   f16   logits the top-32 ran on (+noise)   */
  int64_t* topk_idx;     /* [B,32]    i64   value desc, ties by lower index     */
  void* attn_weights;    /* [B,32]    f16   head-mean attention weights         */
  void* encoded;         /* [B,224]   f16   cat(foothold, gc, proprio)          */
  float* act_scales;     /* [6]       f32   per-layer s_z used by this call     */
  void* proprio_emb;     /* [B,64]    f16   actor_proprio_embedding output, 16-byte aligned */
  void* query;           /* [B,64]    f16   query_projector output (qrt/encoder_opt.py:78-79) */
} GladActorAux;

/* ---- qrt operator replacements -------------------------------------------- */

/* torch.ops.qrt.conv1_fused_q (qrt/qconv.py:170-183, kernel :54-103):
 * x_nhwc f16 [B,21,33,3] -> z8 i8 [B*187,16]. conv1 5x5/s2/p2 + bias + ReLU +
 * BN1 + quantisation (round half away from zero, clamp to [-128,127]).     */
int glad_conv1_fused_q(const void* x_nhwc, int64_t B, const GladConvWeights* w,
                       int8_t* z8_out, void* stream);

/* torch.ops.qrt.conv2_int8_fused (qrt/qconv.py:186-198, kernel :116-163):
 * z8 i8 [B*187,16] -> f16 [B*187,64]. int8 x int8 -> int32 implicit GEMM,
 * acc*dq + b, ReLU, BN2. `acc_out` (NULL or i32 [B*187,64]) receives the
 * int32 accumulators.                                                     */
int glad_conv2_int8_fused(const int8_t* z8, int64_t B, const GladConvWeights* w,
                          void* feat_out, int32_t* acc_out, void* stream);

/* QuantCNN.forward eval branch (qrt/qconv.py:297-303): both ops in one
 * kernel; z8 never leaves the SM unless `z8_out` is non-NULL.              */
int glad_conv_chain(const void* x_nhwc, int64_t B, const GladConvWeights* w,
                    void* feat_out, int8_t* z8_out, void* stream);

/* QuantLinear.forward inference branch (qrt/qlinear.py:111-138):
 * x [M,K] (f16 or f32, row stride ldx elements) -> y f16 [M,N] (stride ldy).
 * act_mode GLAD_ACT_STATIC uses the calibrated inv_sz; GLAD_ACT_DYNAMIC
 * computes s_z = absmax(alpha*x+beta)/127 over the whole input first.
 * `s_z_out` (NULL or f32 [1]) receives the scale used.                     */
size_t glad_qlinear_workspace_size(void);
int glad_qlinear_forward(const GladQLinear* L, int act_mode, const void* x, int x_dtype,
                         int64_t M, int64_t ldx, void* y, int64_t ldy, float* s_z_out,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---- fused rollout forward ---------------------------------------------------
 * The compiled actor function of qrt full mode (qrt/integration.py:129-131;
 * runtime.py:98-99): _encode_terrain_opt (qrt/encoder_opt.py:41-123) over
 * QuantCNN/QuantLinear, then the INT8 actor MLP. obs [B, 96+2079] (f32 or
 * f16, row stride ld_obs elements) -> mean f32 [B,29]. With mean_out NULL
 * only the encoder runs (aux->encoded must then be set).
 * `topk_noise` (NULL or f32 [B,187]) is added to the top-k logits before
 * selection (the Gumbel term of train-mode rollouts, qrt/encoder_opt.py:87-91). */
size_t glad_actor_workspace_size(int64_t B);
int glad_actor_forward(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                       int64_t ld_obs, int act_mode, const float* topk_noise, float* mean_out,
                       const GladActorAux* aux, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Actor and critic of one rollout step (eval mode) from ONE read of the
 * height scan: the policy group `policy_obs` [B, 96+2079] supplies the scan,
 * the actor proprio and the actor head; the critic group `critic_obs` (row
 * stride ld_critic) supplies only its first P_c proprio columns -- its scan
 * must equal the policy group's, as in the reference's benchmarks
 * (qrt/bench/_common.py:60). The encoder weights (conv, GPS, scorer, query
 * projector, MHA) are taken from `wa` for both heads (GLAD shares them);
 * `wc` supplies the fp16 critic proprio embedding and critic MLP. Results are
 * those of glad_actor_forward + glad_critic_forward. No counterpart in the
 * reference, which encodes the shared scan twice.                           */
size_t glad_actor_critic_workspace_size(int64_t B);
int glad_actor_critic_forward(const GladActorWeights* wa, const GladCriticWeights* wc, const void* policy_obs,
                              const void* critic_obs, int obs_dtype, int64_t B, int64_t ld_policy,
                              int64_t ld_critic, int act_mode, float* mean_out, float* value_out,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Train-mode rollout forward (qrt/encoder_opt.py:87-91 with qrt's default
 * rollout_training=True): as glad_actor_forward, with the Gumbel term drawn
 * inside the kernel instead of read from memory. Token i of environment e
 * uses word (i & 3) of Philox4x32-10 (Salmon et al., SC 2011) with counter
 * {i >> 2, e, e >> 32, offset} and key {seed, seed >> 32}; U = (word >> 21) /
 * 2048 and the noise is -log(-log(U)) evaluated in fp16 steps like the
 * reference. `gumbel_offset` is a device word holding this call's offset; the
 * call adds one to it on the device, so replays of a captured graph draw
 * fresh noise. The reference draws with torch.rand: equal in distribution,
 * not bit for bit.                                                          */
int glad_actor_forward_train(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                             int64_t ld_obs, int act_mode, uint64_t gumbel_seed,
                             unsigned long long* gumbel_offset, float* mean_out, const GladActorAux* aux,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Train-mode glad_actor_critic_forward: each head adds its own Gumbel term to
 * its top-k logits, as the reference's two compiled functions each draw one
 * (qrt/integration.py:204-216, qrt/encoder_opt.py:87-91). The actor uses
 * offset *gumbel_offset, the critic *gumbel_offset + 1 (both with the Philox
 * layout of glad_actor_forward_train); the call adds two to the device word. */
int glad_actor_critic_forward_train(const GladActorWeights* wa, const GladCriticWeights* wc,
                                    const void* policy_obs, const void* critic_obs, int obs_dtype,
                                    int64_t B, int64_t ld_policy, int64_t ld_critic, int act_mode,
                                    uint64_t gumbel_seed, unsigned long long* gumbel_offset,
                                    float* mean_out, float* value_out, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* PPO.act epilogue of a rollout step (rsl_rl/algorithms/ppo.py:129-140): the
 * action distribution Normal(mean, std) (rsl_rl/modules/actor_critic_encoder.py:
 * 329-335) sampled once per environment and scored (:366-367):
 *   actions[e,j]  = mean[e,j] + std[j] * z[e,j]
 *   log_prob[e]   = sum_j ( -(a-mean)^2 / (2 std^2) - log(std) - log(sqrt(2 pi)) )
 *   sigma_out[e,j] = std[j]                       (optional, action_sigma)
 * with every operation in fp32 as torch.distributions.Normal evaluates it; the
 * sum over the n_actions terms is a fixed butterfly (lane j holds terms j and
 * j+32; partners 16, 8, 4, 2, 1 apart). z ~ N(0,1) by the Box-Muller transform:
 * pair q = j/2 of environment e takes words (2(q&1), 2(q&1)+1) of Philox4x32-10
 * with counter {0x80000000 | q/2, e, e >> 32, offset} and key {seed, seed >> 32}:
 * u1 = ((w0 >> 8) + 1) / 2^24, u2 = (w1 >> 8) / 2^24, r = sqrt(-2 log u1),
 * z[2q] = r cos(2 pi u2), z[2q+1] = r sin(2 pi u2). rng_state is a device pair
 * {offset, scratch counter} (zero-initialise once); each call uses offset
 * rng_state[0] and adds one to it on the device. The reference samples with
 * torch.normal: equal in distribution, not bit for bit. n_actions 1..64;
 * mean/actions f32 with row strides ld_mean/ld_actions, std f32 [n_actions],
 * log_prob f32 [B].                                                        */
int glad_ppo_epilogue(const float* mean, int64_t B, int64_t ld_mean, const float* std, int n_actions,
                      uint64_t seed, unsigned long long* rng_state, float* actions, int64_t ld_actions,
                      float* log_prob, float* sigma_out, void* stream);

/* The compiled critic function of qrt full mode (qrt/integration.py:133-135):
 * the same encoder over the critic observation group, then the fp16 critic
 * MLP. obs [B, P+2079] (P <= 104), value_out f32 [B,1] (the fp16 output
 * widened, as `.float()` at qrt/integration.py:214). topk_noise and aux as
 * for the actor (encoded has row stride 232 when set).                        */
size_t glad_critic_workspace_size(int64_t B);
int glad_critic_forward(const GladCriticWeights* w, const void* obs, int obs_dtype, int64_t B,
                        int64_t ld_obs, int act_mode, const float* topk_noise, float* value_out,
                        const GladActorAux* aux, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Train-mode glad_critic_forward: the critic head's Gumbel term of the top-k
 * logits drawn inside the kernel (Philox4x32-10, the layout of
 * glad_actor_forward_train) instead of read from memory, as the reference's
 * train-mode critic draws its own (qrt/integration.py:212-216,
 * qrt/encoder_opt.py:87-91); the call adds one to the device word
 * *gumbel_offset. value_out NULL runs the encoder only (aux->encoded set).   */
int glad_critic_forward_train(const GladCriticWeights* w, const void* obs, int obs_dtype, int64_t B,
                              int64_t ld_obs, int act_mode, uint64_t gumbel_seed,
                              unsigned long long* gumbel_offset, float* value_out, const GladActorAux* aux,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostics: record CUDA events (cudaEvent_t, passed as void*) between the
 * stages of the following glad_actor_forward calls on this host thread:
 * events[0] before the first launch, then one after each stage (absmax, front,
 * tail, actor.0, actor.2, actor.4, actor.6), so n = 8 covers a dynamic-mode
 * call. When the fused MLP kernel runs, the actor.0 stage spans all four
 * layers and the other three are empty. n = 0 switches recording off. Not
 * part of the reference interface.                                          */
int glad_actor_stage_events(void* const* events, int n);

/* 1 if glad_actor_forward runs the actor MLP as one fused kernel for a B-row
 * call in `act_mode` on the current device, 0 if it runs one GEMM kernel per
 * layer, < 0 on error. The fused kernel's dynamic-s_z grid barrier needs all
 * of its CTAs resident at once (B <= 128 x the device's resident 4-CTA
 * clusters); the environment variable GLAD_MLP_FUSED=0 disables it. Both
 * paths give identical results. Not part of the reference interface.       */
int glad_actor_mlp_fused(int64_t B, int act_mode);

/* Number of kernels one glad_actor_forward call with mean_out set launches for
 * a B-row batch on the current device (the slot-reset kernel included), aux
 * outputs aside; < 0 on error. Not part of the reference interface.         */
int glad_actor_kernel_count(int64_t B, int act_mode);

/* Allocation-free variant of glad_actor_forward. No counterpart in the
 * reference: it serves callers that cannot allocate device memory for this
 * library -- a host runtime that owns all device memory through its own pool
 * and forbids plugins to call cudaMalloc, or that cannot afford the
 * synchronisation and fragmentation of allocating inside a rollout loop.
 * The scratch is a static device array owned by the library, sized for at
 * most GLAD_NOALLOC_MAX_B environments (about 11.2 MiB held on every GPU that
 * loads the library until exit); larger B is rejected with
 * GLAD_ERR_INVALID_ARG. The first call on a device resolves the array's
 * address: make it before any stream capture (a first call on a capturing
 * stream returns GLAD_ERR_INVALID_ARG); the address is kept until exit, so
 * cudaDeviceReset is not supported together with this entry point. Calls
 * share the array: calls that overlap on the GPU race, so serialise them on
 * one stream. Arguments and results are those of glad_actor_forward.        */
#define GLAD_NOALLOC_MAX_B 2048
int glad_actor_forward_noalloc(const GladActorWeights* w, const void* obs, int obs_dtype, int64_t B,
                               int64_t ld_obs, int act_mode, const float* topk_noise,
                               float* mean_out, const GladActorAux* aux, void* stream);

/* Device-side status word of the last glad_actor_forward_noalloc call on the
 * current device (the static scratch's copy of what glad_workspace_status
 * reads from a workspace): 0 = fine, bits = a bounded wait ran out, in which
 * case the call's outputs are not valid and GLAD_ERR_DEVICE is returned.
 * Synchronises `stream`. Companion of the allocation-free entry point; no
 * counterpart in the reference.                                             */
int glad_actor_noalloc_status(uint32_t* status, void* stream);

/* Device-side status word of a workspace: every bounded wait inside the
 * kernels (mbarrier waits on the tensor core, the grid barriers of the dynamic
 * scales) gives up after its limit, ORs a GLAD_DEVERR_* bit into this word and
 * lets the kernel finish, so the device stays usable but that call's results
 * are not valid. The word lives outside what each call clears: it collects
 * every launch since the previous glad_workspace_status call on this
 * workspace, which reads it into *status, clears it and returns
 * GLAD_ERR_DEVICE when it was not 0. A workspace must be zeroed (at least its
 * first 256 bytes) before its first use. Synchronises `stream`.           */
#define GLAD_DEVERR_MMA_TIMEOUT 1u       /* a tensor-core completion wait ran out     */
#define GLAD_DEVERR_COPY_TIMEOUT 2u      /* an asynchronous-copy completion wait ran out */
#define GLAD_DEVERR_BAD_SHAPE 4u         /* a kernel met a shape it was not built for */
#define GLAD_DEVERR_BARRIER_TIMEOUT 8u   /* a grid barrier ran out (CTAs not co-resident) */
int glad_workspace_status(void* workspace, uint32_t* status, void* stream);

/* Test hook of the failure path, not part of the reference interface: the
 * fused actor MLP's grid barriers (launched after this call) wait for
 * `extra_arrivals` CTAs more than the grid holds and give up after
 * `limit_ns` nanoseconds (0: the normal 2 s), so a forward reports
 * GLAD_DEVERR_BARRIER_TIMEOUT through its status word without hanging.
 * (0, 0) restores normal operation. Process-wide.                          */
int glad_debug_mlp_barrier(uint32_t extra_arrivals, uint64_t limit_ns);

/* ---- W4A16 actor MLP (no reference implementation: INT4 is named only as
 * future work in the reference, README.md:259) ------------------------------
 * Format: q int4 in [-8, 7], packed two per byte along K (q[n,2j] in the low
 * nibble of byte j of row n), one fp16 scale per 64 consecutive inputs of a
 * row (the last group of a row may be shorter); W'[n,k] = fp16(q * s). The
 * layer computes y = fp16(x @ W'^T + b) with fp32 accumulation; hidden layers
 * apply ELU in fp16. Shapes are those of the actor MLP: 224->512->256->128->29. */
typedef struct GladW4Linear {
  const void* packed;   /* uint8 [N, K/2], 16-byte aligned */
  const void* scales;   /* fp16 [N, ceil(K/64)] */
  const void* bias;     /* fp16 [N] or NULL */
  int in_features, out_features;
} GladW4Linear;

/* The four W4A16 layers on fp16 rows x [M, ldx] (K = 224) -> mean f32 [M, 29]
 * (float of the fp16 head output). Any M; no workspace. */
int glad_w4a16_mlp_forward(const GladW4Linear* mlp, const void* x, int64_t M, int64_t ldx,
                           float* mean_out, void* stream);

/* The actor forward with the INT8 encoder of glad_actor_forward (its
 * weights from `w`; w->mlp is not read) and the W4A16 MLP `mlp[4]`. The
 * workspace is glad_actor_workspace_size(B) bytes.                          */
int glad_actor_forward_w4a16(const GladActorWeights* w, const GladW4Linear* mlp, const void* obs,
                             int obs_dtype, int64_t B, int64_t ld_obs, int act_mode, float* mean_out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ---- weight refresh (qrt/runtime.py:195-271) ------------------------------- */

/* QuantLinear.requantize_ (qrt/qlinear.py:84-102) in place, for `n` layers in
 * one launch. Source weights are the module's fp16 (or f32) parameters.     */
typedef struct GladQLinearSrc {
  const void* weight;   /* [N,K] */
  const void* bias;     /* [N] or NULL */
  int32_t w_dtype;      /* GLAD_DTYPE_F16 / F32, for weight and bias */
  int32_t N, K, Np;
  const float* alpha;   /* [K] or NULL */
  const float* beta;    /* [K] or NULL */
  const float* s_z;     /* 0-d */
  int8_t* w8;           /* [Np,K] out */
  float* dq_scale;      /* [Np] out   */
  float* s_w;           /* [Np] out   */
  float* b_prime;       /* [Np] out   */
} GladQLinearSrc;
int glad_requant_qlinear(const GladQLinearSrc* layers, int n, void* stream);

/* QuantCNN.requantize_ (qrt/qconv.py:247-284) in place. Parameters are the
 * inference copy's (conv weights/biases, BN weight/bias/running stats) in
 * `dtype`; the BN affine is evaluated in that dtype as the reference does.
 * s_z 0-d f32; eps the BatchNorm eps.                                       */
typedef struct GladQCNNSrc {
  const void* conv1_w; const void* conv1_b;
  const void* bn1_w; const void* bn1_b; const void* bn1_mean; const void* bn1_var;
  const void* conv2_w; const void* conv2_b;
  const void* bn2_w; const void* bn2_b; const void* bn2_mean; const void* bn2_var;
  const float* s_z;
  float eps1, eps2;
  void* w1p; float* b1f; float* qa; float* qc;
  int8_t* w8; float* dq; float* b2f; float* a2; float* c2;
  int32_t dtype;          /* GLAD_DTYPE_F16 (fp16 copy) or F32, for every parameter */
  const float* alpha;     /* [16] LET of conv2's input, or NULL (qrt/qconv.py:256-258,271-272) */
  const float* beta;      /* [16] or NULL */
} GladQCNNSrc;
int glad_requant_qcnn(const GladQCNNSrc* src, void* stream);

/* ---- weight hand-over across GPUs -------------------------------------------
 * After the PPO update one rank refreshes its inference copy (sync_weights_from,
 * qrt/runtime.py:224-271); the other ranks receive it in ONE collective when
 * every tensor the forward reads lives in one contiguous device blob. An item is
 * one tensor: its device address and size; glad_pack_layout assigns the offsets
 * (item i at the first 256-byte boundary after item i-1, item 0 at 0) and
 * returns the blob size. glad_pack_weights copies the tensors into the blob,
 * glad_unpack_weights copies them back out (one launch each per 128 items);
 * the broadcast itself is the caller's (NCCL). No counterpart in the
 * reference, which runs on one GPU.                                         */
typedef struct GladPackItem {
  void* tensor;         /* device address of the tensor                     */
  size_t nbytes;        /* its size in bytes                                */
  size_t offset;        /* its place in the blob (set by glad_pack_layout)   */
} GladPackItem;
size_t glad_pack_layout(GladPackItem* items, int n);
int glad_pack_weights(const GladPackItem* items, int n, void* blob, size_t blob_bytes, void* stream);
int glad_unpack_weights(const GladPackItem* items, int n, const void* blob, size_t blob_bytes, void* stream);

/* The cast-copy half of sync_weights_from (qrt/runtime.py:251-253): n
 * element-wise copies with dtype conversion in one launch.                  */
typedef struct GladCastCopy {
  const void* src; void* dst; int64_t n; int32_t src_dtype; int32_t dst_dtype;
} GladCastCopy;
int glad_cast_copy(const GladCastCopy* items, int n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GLAD_B200_H_ */
