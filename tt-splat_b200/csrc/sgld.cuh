// SGLD step of 3DGS-MCMC for one gaussian (shared by the single-GPU and the peer-exchange paths).
#pragma once
#include "common.cuh"

namespace tts {

// add_sgld_noise (spike/mcmc.py:25-34) for gaussian g on its current parameters.
__device__ __forceinline__ void sgld_one(float* __restrict__ params, const ParamLayout& L, int g, double lr_means,
                                         float noise_lr, const float* __restrict__ eps_noise, int step,
                                         unsigned long long seed) {
  const float o = sigmoidf(params[L.opacity() + g]);
  float s[3];
#pragma unroll
  for (int c = 0; c < 3; c++) s[c] = expf(params[L.log_scales() + 3LL * g + c]);
  float q[4];
#pragma unroll
  for (int c = 0; c < 4; c++) q[c] = params[L.quats() + 4LL * g + c];
  const float n = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
  const float w = q[0] / n, x = q[1] / n, y = q[2] / n, z = q[3] / n;
  const float R[3][3] = {{1.f - 2.f * (y * y + z * z), 2.f * (x * y - w * z), 2.f * (x * z + w * y)},
                         {2.f * (x * y + w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - w * x)},
                         {2.f * (x * z - w * y), 2.f * (y * z + w * x), 1.f - 2.f * (x * x + y * y)}};
  float e[3];
  if (eps_noise) {
#pragma unroll
    for (int c = 0; c < 3; c++) e[c] = eps_noise[3LL * g + c];
  } else {
    const U4 r = philox4x32_10(U4{(uint32_t)g, 0u, (uint32_t)step, 0x5347u}, (uint32_t)seed, (uint32_t)(seed >> 32));
    float n3;
    box_muller(r.x, r.y, e[0], e[1]);
    box_muller(r.z, r.w, e[2], n3);
  }
  // op_sigmoid(1 - o) = sigmoid(100 ((1 - o) - 0.995)) (spike/mcmc.py:13-15)
  const float gate = sigmoidf(100.f * ((1.f - o) - 0.995f));
  const float weight = gate * (float)((double)noise_lr * lr_means);
#pragma unroll
  for (int i = 0; i < 3; i++) {
    const float d = (R[i][0] * s[0] * e[0] + R[i][1] * s[1] * e[1] + R[i][2] * s[2] * e[2]) * weight;
    params[L.means() + 3LL * g + i] += d;
  }
}

}  // namespace tts
