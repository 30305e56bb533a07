// Dense (un-binned) WSR poly-splat, the entry point of spike/backward.py:61-63 (wsr_polysplat):
// C[P,3] = (sum_g w[p,g] color[g] + w_b c_b) / (sum_g w[p,g] + w_b),
// w = o * keep * relu(Phi . theta_u)^2, for an arbitrary per-pixel basis Phi[P,6].
// O(P*G): meant for the small problems the reference's dense oracle is used on; the binned
// kernels are the hot path.
#include "common.cuh"

namespace tts {

constexpr int DN_CHUNK = 256;

__global__ void __launch_bounds__(256)
    k_wsr_dense_fwd(const float* __restrict__ th, const float* __restrict__ o, const float* __restrict__ col,
                    const float* __restrict__ w_b, const float* __restrict__ Phi, const float* __restrict__ c_b,
                    const float* __restrict__ keep, int P, int G, float* __restrict__ C, float* __restrict__ den) {
  __shared__ float sg[DN_CHUNK][10];
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  float ph[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (p < P)
#pragma unroll
    for (int j = 0; j < 6; j++) ph[j] = Phi[6LL * p + j];
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  for (int base = 0; base < G; base += DN_CHUNK) {
    const int n = min(DN_CHUNK, G - base);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int g = base + i;
      const float ok = o[g] * (keep ? keep[g] : 1.f);
#pragma unroll
      for (int j = 0; j < 6; j++) sg[i][j] = th[6LL * g + j];
      sg[i][6] = ok;
      sg[i][7] = col[3LL * g];
      sg[i][8] = col[3LL * g + 1];
      sg[i][9] = col[3LL * g + 2];
    }
    __syncthreads();
    for (int i = 0; i < n; ++i) {
      float u = 0.f;
#pragma unroll
      for (int j = 0; j < 6; j++) u = fmaf(ph[j], sg[i][j], u);
      const float r = fmaxf(u, 0.f);
      const float w = sg[i][6] * r * r;
      a0 = fmaf(w, sg[i][7], a0);
      a1 = fmaf(w, sg[i][8], a1);
      a2 = fmaf(w, sg[i][9], a2);
      a3 += w;
    }
  }
  if (p >= P) return;
  const float wb = *w_b;
  const float d = a3 + wb;
  C[3LL * p] = (a0 + wb * c_b[0]) / d;
  C[3LL * p + 1] = (a1 + wb * c_b[1]) / d;
  C[3LL * p + 2] = (a2 + wb * c_b[2]) / d;
  den[p] = d;
}

// Thread per gaussian; pixels staged in chunks (Phi, gnum, gden).  Block 0 also accumulates
// the w_b gradient over all pixels.
__global__ void __launch_bounds__(256)
    k_wsr_dense_bwd(const float* __restrict__ th, const float* __restrict__ o, const float* __restrict__ col,
                    const float* __restrict__ Phi, const float* __restrict__ c_b, const float* __restrict__ keep, int P,
                    int G, const float* __restrict__ C, const float* __restrict__ den, const float* __restrict__ gC,
                    float* __restrict__ gth, float* __restrict__ go, float* __restrict__ gcol,
                    float* __restrict__ gwb_partial) {
  __shared__ float sp[DN_CHUNK][10];
  __shared__ float red[8];
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  float t[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, og = 0.f, kf = 0.f, cl[3] = {0.f, 0.f, 0.f};
  if (g < G) {
#pragma unroll
    for (int j = 0; j < 6; j++) t[j] = th[6LL * g + j];
    og = o[g];
    kf = keep ? keep[g] : 1.f;
#pragma unroll
    for (int c = 0; c < 3; c++) cl[c] = col[3LL * g + c];
  }
  float acc_t[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, acc_o = 0.f, acc_c[3] = {0.f, 0.f, 0.f}, wbp = 0.f;
  for (int base = 0; base < P; base += DN_CHUNK) {
    const int n = min(DN_CHUNK, P - base);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const long long p = base + i;
      const float d = den[p];
      const float g0 = gC[3 * p], g1 = gC[3 * p + 1], g2 = gC[3 * p + 2];
      const float gn0 = g0 / d, gn1 = g1 / d, gn2 = g2 / d;
      const float gd = -(g0 * C[3 * p] + g1 * C[3 * p + 1] + g2 * C[3 * p + 2]) / d;
#pragma unroll
      for (int j = 0; j < 6; j++) sp[i][j] = Phi[6 * p + j];
      sp[i][6] = gn0;
      sp[i][7] = gn1;
      sp[i][8] = gn2;
      sp[i][9] = gd;
      if (blockIdx.x == 0) wbp += gn0 * c_b[0] + gn1 * c_b[1] + gn2 * c_b[2] + gd;
    }
    __syncthreads();
    for (int i = 0; i < n; ++i) {
      float u = 0.f;
#pragma unroll
      for (int j = 0; j < 6; j++) u = fmaf(sp[i][j], t[j], u);
      const float r = fmaxf(u, 0.f);
      const float wg = r * r * kf;
      const float w = og * wg;
      acc_c[0] = fmaf(w, sp[i][6], acc_c[0]);
      acc_c[1] = fmaf(w, sp[i][7], acc_c[1]);
      acc_c[2] = fmaf(w, sp[i][8], acc_c[2]);
      const float gw = sp[i][6] * cl[0] + sp[i][7] * cl[1] + sp[i][8] * cl[2] + sp[i][9];
      acc_o = fmaf(gw, wg, acc_o);
      const float gu = gw * og * kf * 2.f * r;
#pragma unroll
      for (int j = 0; j < 6; j++) acc_t[j] = fmaf(gu, sp[i][j], acc_t[j]);
    }
  }
  if (blockIdx.x == 0) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) wbp += __shfl_xor_sync(0xffffffffu, wbp, d);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = wbp;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int i = 0; i < 8; i++) s += red[i];
      gwb_partial[0] = s;
    }
  }
  if (g >= G) return;
#pragma unroll
  for (int j = 0; j < 6; j++) gth[6LL * g + j] = acc_t[j];
  go[g] = acc_o;
#pragma unroll
  for (int c = 0; c < 3; c++) gcol[3LL * g + c] = acc_c[c];
}

}  // namespace tts

using namespace tts;

extern "C" int tts_wsr_dense_fwd(const float* theta_u, const float* o, const float* color, const float* w_b,
                                 const float* Phi, const float* c_b, const float* keep, int P, int G, float* C,
                                 float* den, void* stream) {
  TTS_REQUIRE(P >= 0 && G >= 0, "negative size");
  TTS_REQUIRE(theta_u && o && color && w_b && Phi && c_b && C && den, "null pointer");
  if (P == 0) return TTS_OK;
  k_wsr_dense_fwd<<<(P + 255) / 256, 256, 0, as_stream(stream)>>>(theta_u, o, color, w_b, Phi, c_b, keep, P, G, C, den);
  return check_launch("wsr_dense_fwd");
}

extern "C" int tts_wsr_dense_bwd(const float* theta_u, const float* o, const float* color, const float* w_b,
                                 const float* Phi, const float* c_b, const float* keep, int P, int G, const float* C,
                                 const float* den, const float* gC, float* gtheta, float* go, float* gcolor,
                                 float* gw_b_partial, void* stream) {
  (void)w_b;
  TTS_REQUIRE(P >= 0 && G >= 0, "negative size");
  TTS_REQUIRE(theta_u && o && color && Phi && c_b && C && den && gC && gtheta && go && gcolor && gw_b_partial,
              "null pointer");
  const int blocks = G > 0 ? (G + 255) / 256 : 1;
  k_wsr_dense_bwd<<<blocks, 256, 0, as_stream(stream)>>>(theta_u, o, color, Phi, c_b, keep, P, G, C, den, gC, gtheta,
                                                         go, gcolor, gw_b_partial);
  return check_launch("wsr_dense_bwd");
}
