// Photometric loss (1-l) L1 + l (1 - SSIM) and its gradient (replaces metrics.loss_fn,
// spike/metrics.py:26-28, with the manual gradient of tools/loss_manual.py:78-105).
//
// SSIM uses the valid separable Gaussian window (tools/loss_manual.py:28-55; pytorch_msssim
// convention) on inputs clamped to [0,1] (spike/metrics.py:6-7).  Two tiled kernels per
// (view, channel):
//   k_ssim_fwd : output tile 32x16 of the SSIM map.  Loads the (32+win-1)x(16+win-1) input
//                halo into shared memory, filters the five maps x, y, x^2, y^2, xy along the
//                rows then the columns, and writes dS/dmu_x, dS/d(x^2 filtered),
//                dS/d(xy filtered) plus a per-block partial of sum(S).
//   k_ssim_bwd : input tile 32x16.  Applies the transposed filter to the three dS maps
//                (zero outside the valid region), combines them with x and y into the SSIM
//                gradient, adds the L1 gradient, and writes a per-block partial of sum|x-y|.
// A final one-block-per-view kernel reduces the partials in a fixed order (deterministic).
#include "common.cuh"

namespace tts {

constexpr int LT_W = 32, LT_H = 16, LWIN_MAX = 11;
constexpr int LI_W = LT_W + LWIN_MAX - 1, LI_H = LT_H + LWIN_MAX - 1;
constexpr float SSIM_C1 = 0.01f * 0.01f, SSIM_C2 = 0.03f * 0.03f;

struct Window {
  float g[LWIN_MAX];
  int win;
};

__global__ void __launch_bounds__(256)
    k_ssim_fwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, Window wd,
               float* __restrict__ maps, float* __restrict__ part) {
  __shared__ float sx[LI_H][LI_W + 1], sy[LI_H][LI_W + 1];
  __shared__ float h[5][LI_H][LT_W + 1];
  __shared__ float red[8];
  const int win = wd.win;
  const int Ho = H - win + 1, Wo = W - win + 1;
  const int vc = blockIdx.z, v = vc / 3, ch = vc % 3;
  const int ox0 = blockIdx.x * LT_W, oy0 = blockIdx.y * LT_H;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  const int IW = LT_W + win - 1, IH = LT_H + win - 1;
  for (int i = tid; i < IH * IW; i += 256) {
    const int r = i / IW, c = i % IW;
    const int gy = oy0 + r, gx = ox0 + c;
    float x = 0.f, y = 0.f;
    if (gy < H && gx < W) {
      const long long q = (((long long)v * H + gy) * W + gx) * 3 + ch;
      x = fminf(fmaxf(img[q], 0.f), 1.f);
      y = fminf(fmaxf(tgt[q], 0.f), 1.f);
    }
    sx[r][c] = x;
    sy[r][c] = y;
  }
  __syncthreads();
  for (int i = tid; i < IH * LT_W; i += 256) {
    const int r = i / LT_W, c = i % LT_W;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, a4 = 0.f;
    for (int k = 0; k < win; ++k) {
      const float x = sx[r][c + k], y = sy[r][c + k], gk = wd.g[k];
      a0 = fmaf(gk, x, a0);
      a1 = fmaf(gk, y, a1);
      a2 = fmaf(gk, x * x, a2);
      a3 = fmaf(gk, y * y, a3);
      a4 = fmaf(gk, x * y, a4);
    }
    h[0][r][c] = a0; h[1][r][c] = a1; h[2][r][c] = a2; h[3][r][c] = a3; h[4][r][c] = a4;
  }
  __syncthreads();
  float ssum = 0.f;
  const long long plane = (long long)Ho * Wo;
  float* mbase = maps + (long long)vc * 3 * plane;
  for (int i = tid; i < LT_H * LT_W; i += 256) {
    const int r = i / LT_W, c = i % LT_W;
    const int oy = oy0 + r, ox = ox0 + c;
    if (oy >= Ho || ox >= Wo) continue;
    float f[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < win; ++k) {
      const float gk = wd.g[k];
#pragma unroll
      for (int m = 0; m < 5; m++) f[m] = fmaf(gk, h[m][r + k][c], f[m]);
    }
    const float mux = f[0], muy = f[1];
    const float mux2 = mux * mux, muy2 = muy * muy;
    const float sxx = f[2] - mux2, syy = f[3] - muy2, sxy = f[4] - mux * muy;
    const float A1 = 2.f * mux * muy + SSIM_C1, A2 = 2.f * sxy + SSIM_C2;
    const float B1 = mux2 + muy2 + SSIM_C1, B2 = sxx + syy + SSIM_C2;
    const float D = B1 * B2;
    const float S = (A1 * A2) / D;
    ssum += S;
    const long long q = (long long)oy * Wo + ox;
    mbase[q] = (2.f / D) * (muy * (A2 - A1) - S * mux * (B2 - B1));   // dS/dmu_x
    mbase[plane + q] = -S / B2;                                       // dS/d filt(x^2)
    mbase[2 * plane + q] = 2.f * A1 / D;                              // dS/d filt(xy)
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
  if ((tid & 31) == 0) red[tid >> 5] = ssum;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    part[(long long)vc * gridDim.x * gridDim.y + blockIdx.y * gridDim.x + blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(256)
    k_ssim_bwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, Window wd, float lambda,
               float grad_scale, const float* __restrict__ maps, float* __restrict__ gimg, float* __restrict__ part) {
  __shared__ float sm[3][LI_H][LI_W + 1];
  __shared__ float h[3][LI_H][LT_W + 1];
  __shared__ float red[8];
  const int win = wd.win;
  const int Ho = H - win + 1, Wo = W - win + 1;
  const int vc = blockIdx.z, v = vc / 3, ch = vc % 3;
  const int x0 = blockIdx.x * LT_W, y0 = blockIdx.y * LT_H;
  const int tid = threadIdx.y * blockDim.x + threadIdx.x;
  const int IW = LT_W + win - 1, IH = LT_H + win - 1;
  const long long plane = (long long)Ho * Wo;
  const float* mbase = maps + (long long)vc * 3 * plane;
  // map rows [y0-win+1, y0+LT_H), cols [x0-win+1, x0+LT_W); zero outside the valid region
  for (int i = tid; i < IH * IW; i += 256) {
    const int r = i / IW, c = i % IW;
    const int my = y0 - (win - 1) + r, mx = x0 - (win - 1) + c;
    float a = 0.f, b = 0.f, d = 0.f;
    if (my >= 0 && my < Ho && mx >= 0 && mx < Wo) {
      const long long q = (long long)my * Wo + mx;
      a = mbase[q];
      b = mbase[plane + q];
      d = mbase[2 * plane + q];
    }
    sm[0][r][c] = a;
    sm[1][r][c] = b;
    sm[2][r][c] = d;
  }
  __syncthreads();
  for (int i = tid; i < IH * LT_W; i += 256) {
    const int r = i / LT_W, c = i % LT_W;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int k = 0; k < win; ++k) {
      const float gk = wd.g[k];
      const int cc = c + (win - 1) - k;
      a0 = fmaf(gk, sm[0][r][cc], a0);
      a1 = fmaf(gk, sm[1][r][cc], a1);
      a2 = fmaf(gk, sm[2][r][cc], a2);
    }
    h[0][r][c] = a0; h[1][r][c] = a1; h[2][r][c] = a2;
  }
  __syncthreads();
  const float Ns = (float)(3.0 * (double)Ho * (double)Wo);
  const float N = (float)(3.0 * (double)H * (double)W);
  float l1 = 0.f;
  for (int i = tid; i < LT_H * LT_W; i += 256) {
    const int r = i / LT_W, c = i % LT_W;
    const int gy = y0 + r, gx = x0 + c;
    if (gy >= H || gx >= W) continue;
    float t0 = 0.f, t1 = 0.f, t2 = 0.f;
    for (int k = 0; k < win; ++k) {
      const float gk = wd.g[k];
      const int rr = r + (win - 1) - k;
      t0 = fmaf(gk, h[0][rr][c], t0);
      t1 = fmaf(gk, h[1][rr][c], t1);
      t2 = fmaf(gk, h[2][rr][c], t2);
    }
    const long long q = (((long long)v * H + gy) * W + gx) * 3 + ch;
    const float xr = img[q], yr = tgt[q];
    const float x = fminf(fmaxf(xr, 0.f), 1.f), y = fminf(fmaxf(yr, 0.f), 1.f);
    const float mask = (xr >= 0.f && xr <= 1.f) ? 1.f : 0.f;
    const float dmean = (t0 + 2.f * x * t1 + y * t2) / Ns;
    const float diff = xr - yr;
    const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
    l1 += fabsf(diff);
    gimg[q] = grad_scale * ((1.f - lambda) * sgn / N + lambda * (-dmean) * mask);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  if ((tid & 31) == 0) red[tid >> 5] = l1;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    part[(long long)vc * gridDim.x * gridDim.y + blockIdx.y * gridDim.x + blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(256) k_loss_reduce(const float* __restrict__ spart, int nsb, const float* __restrict__ lpart,
                                                     int nlb, int H, int W, int win, float lambda, float* __restrict__ loss) {
  __shared__ double rs[256], rl[256];
  const int v = blockIdx.x;
  double s = 0.0, l = 0.0;
  for (int i = threadIdx.x; i < 3 * nsb; i += blockDim.x) s += spart[(long long)v * 3 * nsb + i];
  for (int i = threadIdx.x; i < 3 * nlb; i += blockDim.x) l += lpart[(long long)v * 3 * nlb + i];
  rs[threadIdx.x] = s;
  rl[threadIdx.x] = l;
  __syncthreads();
  for (int st = blockDim.x >> 1; st > 0; st >>= 1) {
    if ((int)threadIdx.x < st) {
      rs[threadIdx.x] += rs[threadIdx.x + st];
      rl[threadIdx.x] += rl[threadIdx.x + st];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double Ns = 3.0 * (double)(H - win + 1) * (double)(W - win + 1);
    const double N = 3.0 * (double)H * (double)W;
    loss[v] = (float)((1.0 - lambda) * rl[0] / N + lambda * (1.0 - rs[0] / Ns));
  }
}

static size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

static void window_for(int H, int W, Window& wd) {
  // spike/metrics.py:15-19 (window shrink), tools/loss_manual.py:28-31 (weights, float64)
  int win = H < W ? H : W;
  if (win > LWIN_MAX) win = LWIN_MAX;
  if (win % 2 == 0) win -= 1;
  if (win < 3) win = 3;
  double g[LWIN_MAX], sum = 0.0;
  for (int i = 0; i < win; i++) {
    const double c = (double)(i - win / 2);
    g[i] = exp(-(c * c) / (2.0 * 1.5 * 1.5));
    sum += g[i];
  }
  for (int i = 0; i < LWIN_MAX; i++) wd.g[i] = i < win ? (float)(g[i] / sum) : 0.f;
  wd.win = win;
}

struct LossGeom {
  int win, Ho, Wo, fbx, fby, bbx, bby;
};
static LossGeom loss_geom(int H, int W) {
  Window wd;
  window_for(H, W, wd);
  LossGeom lg;
  lg.win = wd.win;
  lg.Ho = H - wd.win + 1;
  lg.Wo = W - wd.win + 1;
  lg.fbx = (lg.Wo + LT_W - 1) / LT_W;
  lg.fby = (lg.Ho + LT_H - 1) / LT_H;
  lg.bbx = (W + LT_W - 1) / LT_W;
  lg.bby = (H + LT_H - 1) / LT_H;
  return lg;
}

}  // namespace tts

using namespace tts;

extern "C" size_t tts_loss_workspace_bytes(int V, int H, int W) {
  if (V < 1 || H < 3 || W < 3) return 0;
  const LossGeom lg = loss_geom(H, W);
  return a256((size_t)V * 9 * lg.Ho * lg.Wo * 4) + a256((size_t)V * 3 * lg.fbx * lg.fby * 4) +
         a256((size_t)V * 3 * lg.bbx * lg.bby * 4);
}

extern "C" int tts_loss_l1_ssim(const float* img, const float* target, int V, int H, int W, float lambda,
                                float grad_scale, float* gimg, float* loss, void* workspace, size_t workspace_bytes,
                                void* stream) {
  TTS_REQUIRE(V >= 1 && H >= 3 && W >= 3, "images must be at least 3x3");
  TTS_REQUIRE(img && target && gimg && loss && workspace, "null pointer");
  if (workspace_bytes < tts_loss_workspace_bytes(V, H, W)) return fail(TTS_ERR_CAPACITY, "loss workspace too small");
  Window wd;
  window_for(H, W, wd);
  const LossGeom lg = loss_geom(H, W);
  char* p = static_cast<char*>(workspace);
  float* maps = reinterpret_cast<float*>(p);
  p += a256((size_t)V * 9 * lg.Ho * lg.Wo * 4);
  float* spart = reinterpret_cast<float*>(p);
  p += a256((size_t)V * 3 * lg.fbx * lg.fby * 4);
  float* lpart = reinterpret_cast<float*>(p);
  cudaStream_t st = as_stream(stream);
  k_ssim_fwd<<<dim3(lg.fbx, lg.fby, V * 3), dim3(32, 8), 0, st>>>(img, target, H, W, wd, maps, spart);
  if (int rc = check_launch("ssim_fwd")) return rc;
  k_ssim_bwd<<<dim3(lg.bbx, lg.bby, V * 3), dim3(32, 8), 0, st>>>(img, target, H, W, wd, lambda, grad_scale, maps,
                                                                   gimg, lpart);
  if (int rc = check_launch("ssim_bwd")) return rc;
  k_loss_reduce<<<V, 256, 0, st>>>(spart, lg.fbx * lg.fby, lpart, lg.bbx * lg.bby, H, W, lg.win, lambda, loss);
  return check_launch("loss_reduce");
}
