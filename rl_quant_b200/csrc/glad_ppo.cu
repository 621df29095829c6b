// PPO.act epilogue of a rollout step (rsl_rl/algorithms/ppo.py:129-140): the
// action distribution Normal(mean, std) of the policy (rsl_rl/modules/
// actor_critic_encoder.py:329-335) is sampled once per environment and the
// sample scored with Normal.log_prob summed over the action dimension
// (actor_critic_encoder.py:366-367).
//
// One warp per environment; lane j owns actions j and j + 32. Every operation
// is an fp32 operation in the order torch.distributions.Normal evaluates it:
//   a  = mean + std * z
//   lp = (-(a - mean)^2) / (2 * std^2) - log(std) - log(sqrt(2 pi))
// and the per-environment sum is a fixed xor butterfly, so the result does not
// depend on the launch shape. z comes from the Box-Muller transform of
// Philox4x32-10 uniforms (counter domain bit 31 set, apart from the Gumbel
// draws of the tail kernel).
#include <cuda_runtime.h>

#include "glad_common.cuh"

namespace glad {

constexpr int kPpoWarps = 8;

__device__ __forceinline__ float ppo_normal(uint64_t seed, uint64_t offset, int64_t env, int j) {
  const int q = j >> 1;
  uint32_t c[4] = {0x80000000u | (uint32_t)(q >> 1), (uint32_t)env, (uint32_t)((uint64_t)env >> 32),
                   (uint32_t)offset};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const int h = q & 1;
  const uint32_t w0 = h ? c[2] : c[0];
  const uint32_t w1 = h ? c[3] : c[1];
  const float u1 = __fmul_rn((float)((w0 >> 8) + 1u), 5.9604644775390625e-8f);   // (0, 1]
  const float u2 = __fmul_rn((float)(w1 >> 8), 5.9604644775390625e-8f);          // [0, 1)
  const float r = sqrtf(__fmul_rn(-2.0f, logf(u1)));
  float sn, cs;
  sincospif(__fmul_rn(2.0f, u2), &sn, &cs);
  return __fmul_rn(r, (j & 1) ? sn : cs);
}

__device__ __forceinline__ float ppo_term(float mean, float s, float a) {
  const float d = __fsub_rn(a, mean);
  const float t = __fdiv_rn(-__fmul_rn(d, d), __fmul_rn(2.0f, __fmul_rn(s, s)));
  return __fsub_rn(__fsub_rn(t, logf(s)), 0.918938533204672742f);
}

__global__ void __launch_bounds__(kPpoWarps * 32) ppo_epilogue_kernel(const __grid_constant__ PpoParams p) {
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t env = (int64_t)blockIdx.x * kPpoWarps + warp;
  grid_dep_wait();                      // the means of the preceding kernel are visible from here
  const uint64_t off = p.rng[0];
  if (env < p.B) {
    float v = 0.0f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = lane + 32 * h;
      float lp = 0.0f;
      if (j < p.n) {
        const float m = p.mean[env * p.ld_mean + j];
        const float s = p.std[j];
        const float a = __fadd_rn(m, __fmul_rn(s, ppo_normal(p.seed, off, env, j)));
        p.actions[env * p.ld_act + j] = a;
        if (p.sigma) p.sigma[env * p.n + j] = s;
        lp = ppo_term(m, s, a);
      }
      v = h == 0 ? lp : __fadd_rn(v, lp);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) p.log_prob[env] = v;
  }
  if (threadIdx.x == 0) {
    // the last block to finish advances the offset (every block has read it) and
    // clears the counter for the next call
    __threadfence();
    if (atomicAdd(&p.rng[1], 1ull) == (unsigned long long)gridDim.x - 1) {
      p.rng[1] = 0ull;
      atomicAdd(&p.rng[0], 1ull);
    }
  }
}

cudaError_t launch_ppo_epilogue(const PpoParams& p, cudaStream_t st, bool pdl) {
  const int64_t blocks = (p.B + kPpoWarps - 1) / kPpoWarps;
  return launch_k(ppo_epilogue_kernel, dim3((unsigned)blocks), dim3(kPpoWarps * 32), 0, st, pdl, p);
}

}  // namespace glad
