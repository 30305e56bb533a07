// Fused Adam + SGLD over the flat parameter buffer (thread per gaussian).
//
// Adam follows torch.optim.Adam's single-tensor update (spike/train.py:19,29; the per-group
// learning rates of spike/model.py:82-95) element by element in fp32 with the same operation
// order (m.lerp_(g, 1-b1); v = v*b2 + (1-b2)*g*g; p += (-lr/bc1)*m / (sqrt(v)/sqrt(bc2) + eps)),
// so a replica on any GPU reproduces the CPU optimizer to the last bits of its arithmetic.
// SGLD (spike/mcmc.py:25-34) then perturbs the means with covariance-shaped noise gated to
// near-transparent gaussians, using the freshly updated parameters, like the reference which
// calls add_sgld_noise after opt.step().
#include "sgld.cuh"

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

// Element-parallel Adam over [0, n) of the flat buffer: each thread updates four consecutive
// elements (one 16-byte vector of p, g, m, v when aligned); the group learning rate of an
// element follows from its index (segment boundaries at 3G, 6G, 10G, 11G, 14G).
__device__ __forceinline__ float lr_of(long long i, long long G, const float nss[6]) {
  return i < 3 * G ? nss[0] : i < 6 * G ? nss[1] : i < 10 * G ? nss[2] : i < 11 * G ? nss[3] : i < 14 * G ? nss[4] : nss[5];
}

// One wave of blocks (ADAM_BLOCKS_PER_SM per SM) walks the buffer grid-stride, one 16-byte vector
// of each array per thread per pass, with the next pass's four vectors requested before the
// current one is updated (a register double buffer); the first pass's loads are issued before the
// block waits for its scalars, so the double-precision bias corrections cost no memory time.
constexpr int ADAM_BLOCKS_PER_SM = 4;

__global__ void __launch_bounds__(256, ADAM_BLOCKS_PER_SM)
    k_adam(float* __restrict__ params, const float* __restrict__ grads, float* __restrict__ m,
           float* __restrict__ v, int G, long long n, const int* __restrict__ step_ptr,
           const double* __restrict__ lr7, double beta1, double beta2, double eps) {
  __shared__ AdamScalars s_a;
  __shared__ float s_nss[7];
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nv = n / 4, stride = (long long)gridDim.x * blockDim.x;
  float4* P = reinterpret_cast<float4*>(params);
  const float4* Gr = reinterpret_cast<const float4*>(grads);
  float4* M = reinterpret_cast<float4*>(m);
  float4* Vv = reinterpret_cast<float4*>(v);
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 pa = z4, ga = z4, ma = z4, va = z4;
  if (tid < nv) {
    pa = P[tid];
    ma = M[tid];
    va = Vv[tid];
    ga = Gr[tid];
  }
  // scalars in double like the Python-side arithmetic of torch's Adam, cast to fp32 at use;
  // computed once per block (the double pow is far costlier than the per-element update)
  if (threadIdx.x == 0) {
    const int step = *step_ptr;
    const double bc1 = 1.0 - pow(beta1, (double)step);
    const double bc2 = 1.0 - pow(beta2, (double)step);
    s_a.w1 = (float)(1.0 - beta1);
    s_a.b2 = (float)beta2;
    s_a.w2 = (float)(1.0 - beta2);
    s_a.bc2_sqrt = (float)sqrt(bc2);
    s_a.eps = (float)eps;
    for (int k = 0; k < 7; k++) s_nss[k] = (float)(-lr7[k] / bc1);
  }
  __syncthreads();
  const AdamScalars a = s_a;
  float nss[6];
#pragma unroll
  for (int k = 0; k < 6; k++) nss[k] = s_nss[k];
  if (tid == 0) adam_elem(params, grads, m, v, 59LL * G, a, s_nss[6]);   // w_b_raw
  auto update4 = [&](long long e0, float4& p4, const float4& g4, float4& m4, float4& v4) {
    float* pp = &p4.x;
    const float* gg = &g4.x;
    float* mm = &m4.x;
    float* vv = &v4.x;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float gr = gg[j];
      const float mj = __fadd_rn(mm[j], __fmul_rn(a.w1, __fsub_rn(gr, mm[j])));
      const float vj = __fadd_rn(__fmul_rn(vv[j], a.b2), __fmul_rn(__fmul_rn(a.w2, gr), gr));
      const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vj), a.bc2_sqrt), a.eps);
      pp[j] = __fadd_rn(pp[j], __fdiv_rn(__fmul_rn(lr_of(e0 + j, G, nss), mj), denom));
      mm[j] = mj;
      vv[j] = vj;
    }
  };
  for (long long i = tid; i < nv; i += stride) {
    const long long j = i + stride;
    float4 pb = z4, gb = z4, mb = z4, vb = z4;
    if (j < nv) {
      pb = P[j];
      mb = M[j];
      vb = Vv[j];
      gb = Gr[j];
    }
    update4(4 * i, pa, ga, ma, va);
    P[i] = pa;
    M[i] = ma;
    Vv[i] = va;
    pa = pb;
    ga = gb;
    ma = mb;
    va = vb;
  }
  for (long long e = 4 * nv + tid; e < n; e += stride) adam_elem(params, grads, m, v, e, a, lr_of(e, G, nss));
}

// SGLD for every gaussian; the means learning rate is read from the device (lr_ptr[0], the
// optimizer's lr vector) or, when lr_ptr is null, given by value.
__global__ void __launch_bounds__(256) k_sgld(float* __restrict__ params, int G, const double* __restrict__ lr_ptr,
                                              double lr_means, float noise_lr, const float* __restrict__ eps_noise,
                                              const int* __restrict__ step_ptr, unsigned long long seed) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  sgld_one(params, ParamLayout{G}, g, lr_ptr ? lr_ptr[0] : lr_means, noise_lr, eps_noise, *step_ptr, seed);
}

// torch.optim.Adam on a short vector with one learning rate (the depth group of
// spike/model.py:93: depth_beta, depth_tau), same arithmetic as k_adam.
__global__ void k_adam_vec(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                           float* __restrict__ v, int n, const int* __restrict__ step_ptr, double lr, double beta1,
                           double beta2, double eps) {
  const int step = *step_ptr;
  const double bc1 = 1.0 - pow(beta1, (double)step);
  const double bc2 = 1.0 - pow(beta2, (double)step);
  AdamScalars a;
  a.w1 = (float)(1.0 - beta1);
  a.b2 = (float)beta2;
  a.w2 = (float)(1.0 - beta2);
  a.bc2_sqrt = (float)sqrt(bc2);
  a.eps = (float)eps;
  const float nss = (float)(-lr / bc1);
  for (int i = threadIdx.x; i < n; i += blockDim.x) adam_elem(p, g, m, v, i, a, nss);
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
  TTS_REQUIRE(aligned16(params) && aligned16(grads) && aligned16(m) && aligned16(v), "buffers must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  // torch skips parameters without a gradient: the colour rest trains only with SH on
  const long long n = sh_degree > 0 ? 59LL * G : 14LL * G;
  // two 16-byte vectors per thread per pass, one wave of blocks looping over the buffer
  long long blocks = (n + 8 * 256 - 1) / (8 * 256);
  if (blocks > 148 * ADAM_BLOCKS_PER_SM) blocks = 148 * ADAM_BLOCKS_PER_SM;
  k_adam<<<(unsigned)(blocks > 0 ? blocks : 1), 256, 0, st>>>(params, grads, m, v, G, n, step, lr7, beta1, beta2, eps);
  if (int rc = check_launch("adam")) return rc;
  if (noise_lr > 0.f && G > 0) {
    k_sgld<<<(G + 255) / 256, 256, 0, st>>>(params, G, lr7, 0.0, noise_lr, eps_noise, step, seed);
    return check_launch("sgld");
  }
  return TTS_OK;
}

extern "C" int tts_adam_vec(float* p, const float* g, float* m, float* v, int n, const int32_t* step, double lr,
                            double beta1, double beta2, double eps, void* stream) {
  TTS_REQUIRE(n >= 0 && n <= 1024 && p && g && m && v && step, "null pointer or n outside [0, 1024]");
  TTS_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0, "betas must be in [0, 1)");
  if (n == 0) return TTS_OK;
  k_adam_vec<<<1, ((n + 31) / 32) * 32, 0, as_stream(stream)>>>(p, g, m, v, n, step, lr, beta1, beta2, eps);
  return check_launch("adam_vec");
}

extern "C" int tts_sgld(float* params, int G, double lr_means, float noise_lr, const float* eps_noise,
                        const int32_t* step, uint64_t seed, void* stream) {
  TTS_REQUIRE(G >= 0 && params && step, "null pointer or negative G");
  if (G == 0) return TTS_OK;
  k_sgld<<<(G + 255) / 256, 256, 0, as_stream(stream)>>>(params, G, nullptr, lr_means, noise_lr, eps_noise, step, seed);
  return check_launch("sgld");
}
