// Fused Adam + SGLD over the flat parameter buffer (thread per gaussian).
//
// Adam follows torch.optim.Adam's single-tensor update (spike/train.py:19,29; the per-group
// learning rates of spike/model.py:82-95) element by element in fp32 with the same operation
// order (m.lerp_(g, 1-b1); v = v*b2 + (1-b2)*g*g; p += (-lr/bc1)*m / (sqrt(v)/sqrt(bc2) + eps)),
// so a replica on any GPU reproduces the CPU optimizer to the last bits of its arithmetic.
// SGLD (spike/mcmc.py:25-34) then perturbs the means with covariance-shaped noise gated to
// near-transparent gaussians, using the freshly updated parameters, like the reference which
// calls add_sgld_noise after opt.step().
#include "common.cuh"

namespace tts {

struct AdamScalars {
  float w1, b2, w2, neg_step_size, bc2_sqrt, eps;
};

__device__ __forceinline__ void adam_elem(float* p, const float* g, float* m, float* v, long long i, const AdamScalars& a,
                                          float neg_step_size) {
  const float gr = g[i];
  float mm = m[i], vv = v[i];
  mm = __fadd_rn(mm, __fmul_rn(a.w1, __fsub_rn(gr, mm)));
  vv = __fadd_rn(__fmul_rn(vv, a.b2), __fmul_rn(__fmul_rn(a.w2, gr), gr));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vv), a.bc2_sqrt), a.eps);
  p[i] = __fadd_rn(p[i], __fdiv_rn(__fmul_rn(neg_step_size, mm), denom));
  m[i] = mm;
  v[i] = vv;
}

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

__global__ void __launch_bounds__(256)
    k_adam_sgld(float* __restrict__ params, const float* __restrict__ grads, float* __restrict__ m,
                float* __restrict__ v, int G, int sh_degree, const int* __restrict__ step_ptr,
                const double* __restrict__ lr7, double beta1, double beta2, double eps, float noise_lr,
                const float* __restrict__ eps_noise, unsigned long long seed) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const ParamLayout L{G};
  const int step = *step_ptr;
  // scalars in double like the Python-side arithmetic of torch's Adam, cast to fp32 at use
  const double bc1 = 1.0 - pow(beta1, (double)step);
  const double bc2 = 1.0 - pow(beta2, (double)step);
  AdamScalars a;
  a.w1 = (float)(1.0 - beta1);
  a.b2 = (float)beta2;
  a.w2 = (float)(1.0 - beta2);
  a.bc2_sqrt = (float)sqrt(bc2);
  a.eps = (float)eps;
  if (g == 0) adam_elem(params, grads, m, v, L.w_b_raw(), a, (float)(-lr7[6] / bc1));
  if (g >= G) return;
  const float nss[6] = {(float)(-lr7[0] / bc1), (float)(-lr7[1] / bc1), (float)(-lr7[2] / bc1),
                        (float)(-lr7[3] / bc1), (float)(-lr7[4] / bc1), (float)(-lr7[5] / bc1)};
#pragma unroll
  for (int c = 0; c < 3; c++) adam_elem(params, grads, m, v, L.means() + 3LL * g + c, a, nss[0]);
#pragma unroll
  for (int c = 0; c < 3; c++) adam_elem(params, grads, m, v, L.log_scales() + 3LL * g + c, a, nss[1]);
#pragma unroll
  for (int c = 0; c < 4; c++) adam_elem(params, grads, m, v, L.quats() + 4LL * g + c, a, nss[2]);
  adam_elem(params, grads, m, v, L.opacity() + (long long)g, a, nss[3]);
#pragma unroll
  for (int c = 0; c < 3; c++) adam_elem(params, grads, m, v, L.color_dc() + 3LL * g + c, a, nss[4]);
  if (sh_degree > 0) {
    // torch skips parameters without a gradient: colour rest only trains when SH is on
    for (int c = 0; c < 45; c++) adam_elem(params, grads, m, v, L.color_rest() + 45LL * g + c, a, nss[5]);
  }
  if (noise_lr <= 0.f) return;
  sgld_one(params, L, g, lr7[0], noise_lr, eps_noise, step, seed);
}

__global__ void __launch_bounds__(256) k_sgld(float* __restrict__ params, int G, double lr_means, float noise_lr,
                                              const float* __restrict__ eps_noise, const int* __restrict__ step_ptr,
                                              unsigned long long seed) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  sgld_one(params, ParamLayout{G}, g, lr_means, noise_lr, eps_noise, *step_ptr, seed);
}

__global__ void k_step_begin(int* step) { *step += 1; }

}  // namespace tts

using namespace tts;

extern "C" int tts_step_begin(int32_t* step, void* stream) {
  TTS_REQUIRE(step, "null step");
  k_step_begin<<<1, 1, 0, as_stream(stream)>>>(step);
  return check_launch("step_begin");
}

extern "C" int tts_adam_sgld(float* params, const float* grads, float* m, float* v, int G, int sh_degree,
                             const int32_t* step, const double* lr7, double beta1, double beta2, double eps, float noise_lr,
                             const float* eps_noise, uint64_t seed, void* stream) {
  TTS_REQUIRE(G >= 0 && params && grads && m && v && step && lr7, "null pointer or negative G");
  TTS_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0, "betas must be in [0, 1)");
  const int blocks = G > 0 ? (G + 255) / 256 : 1;
  k_adam_sgld<<<blocks, 256, 0, as_stream(stream)>>>(params, grads, m, v, G, sh_degree, step, lr7, beta1, beta2, eps,
                                                      noise_lr, eps_noise, seed);
  return check_launch("adam_sgld");
}

extern "C" int tts_sgld(float* params, int G, double lr_means, float noise_lr, const float* eps_noise,
                        const int32_t* step, uint64_t seed, void* stream) {
  TTS_REQUIRE(G >= 0 && params && step, "null pointer or negative G");
  if (G == 0) return TTS_OK;
  k_sgld<<<(G + 255) / 256, 256, 0, as_stream(stream)>>>(params, G, lr_means, noise_lr, eps_noise, step, seed);
  return check_launch("sgld");
}
