// Photometric loss (1-l) L1 + l (1 - SSIM) and its gradient (replaces metrics.loss_fn,
// spike/metrics.py:26-28, with the manual gradient of tools/loss_manual.py:78-105).
//
// SSIM uses the valid separable Gaussian window (tools/loss_manual.py:28-55; pytorch_msssim
// convention) on inputs clamped to [0,1] (spike/metrics.py:6-7).  Two tiled kernels, each a
// separable filter with register blocking so that every shared-memory load feeds several FMAs
// (a thread slides an RB-long window along a row, then along a column).  Both run as persistent
// blocks over (view, channel, tile) with the next tile's halo streaming into a second shared
// buffer by cp.async while the current one is filtered:
//   k_ssim_fwd : output tile 64x32 of the SSIM map.  Loads the (64+win-1)x(32+win-1) input
//                halo, filters the five maps x, y, x^2, y^2, xy along rows then columns, and
//                writes dS/dmu_x, dS/d(filtered x^2), dS/d(filtered xy) plus a per-block
//                partial of sum(S).
//   k_ssim_bwd : input tile 64x32.  Applies the transposed filter to the three dS maps (zero
//                outside the valid region), combines them with x and y into the SSIM gradient,
//                adds the L1 gradient, and writes a per-block partial of sum|x - y|.
// A one-block-per-view kernel reduces the partials in a fixed order (deterministic).
#include "common.cuh"

namespace tts {

constexpr int LT_W = 64, LT_H = 32, LWIN_MAX = 11, RB = 8;
constexpr float SSIM_C1 = 0.01f * 0.01f, SSIM_C2 = 0.03f * 0.03f;

struct Window {
  float g[LWIN_MAX];
  int win;
};

// shared-memory geometry for a window WIN: input rows/cols with odd strides (bank-conflict free
// when lanes walk down rows)
template <int WIN>
struct LGeom {
  static constexpr int IH = LT_H + WIN - 1, IW = LT_W + WIN - 1;
  static constexpr int XS = IW | 1;        // odd row stride of the input tiles
  static constexpr int HS = LT_W + 1;      // odd row stride of the row-filtered maps
};

// 4-byte asynchronous global->shared copy; src_bytes = 0 writes a zero (halo outside the image).
__device__ __forceinline__ void cp_async4(float* dst, const float* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

struct TileId {
  int v, ch, bx, by;
};
// channel fastest, so the three channel tiles of one image region run side by side (L2 reuse of
// the interleaved [H,W,3] rows)
__device__ __forceinline__ TileId decode_tile(int tile, int gx, int gy) {
  TileId t;
  t.ch = tile % 3;
  tile /= 3;
  t.bx = tile % gx;
  tile /= gx;
  t.by = tile % gy;
  t.v = tile / gy;
  return t;
}

// Persistent blocks walk the tiles with stride gridDim.x; the halo of the next tile streams into
// the second buffer (cp.async) while the current one is filtered.
template <int WIN>
__global__ void __launch_bounds__(256)
    k_ssim_fwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, int gx, int gy, int ntiles,
               Window wd, float* __restrict__ maps, float* __restrict__ part) {
  using LG = LGeom<WIN>;
  constexpr int BUF = LG::IH * LG::XS;
  extern __shared__ float smem[];
  float* sx = smem;                            // [2][IH][XS]
  float* sy = sx + 2 * BUF;                    // [2][IH][XS]
  float* h = sy + 2 * BUF;                     // [5][IH][HS]
  __shared__ float red[8];
  const int Ho = H - WIN + 1, Wo = W - WIN + 1;
  const int tid = threadIdx.x;
  float g[WIN];
#pragma unroll
  for (int k = 0; k < WIN; k++) g[k] = wd.g[k];
  auto issue = [&](int tile, int b) {
    const TileId id = decode_tile(tile, gx, gy);
    const int ox0 = id.bx * LT_W, oy0 = id.by * LT_H;
    for (int i = tid; i < LG::IH * LG::IW; i += 256) {
      const int r = i / LG::IW, c = i % LG::IW;
      const int yy = oy0 + r, xx = ox0 + c;
      const bool in = yy < H && xx < W;
      const long long q = in ? (((long long)id.v * H + yy) * W + xx) * 3 + id.ch : 0;
      cp_async4(sx + b * BUF + r * LG::XS + c, img + q, in ? 4 : 0);
      cp_async4(sy + b * BUF + r * LG::XS + c, tgt + q, in ? 4 : 0);
    }
    cp_async_commit();
  };
  int buf = 0;
  if ((int)blockIdx.x < ntiles) issue(blockIdx.x, 0);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int next = tile + gridDim.x;
    if (next < ntiles) issue(next, buf ^ 1);
    else cp_async_commit();
    cp_async_wait_1();
    __syncthreads();
    const TileId id = decode_tile(tile, gx, gy);
    const int vc = id.v * 3 + id.ch;
    const int ox0 = id.bx * LT_W, oy0 = id.by * LT_H;
    const float* bx_ = sx + buf * BUF;
    const float* by_ = sy + buf * BUF;
    // rows: item = (row r, segment of RB outputs); lanes walk down rows (odd stride)
    for (int it = tid; it < LG::IH * (LT_W / RB); it += 256) {
      const int r = it % LG::IH, c0 = (it / LG::IH) * RB;
      float a[5][RB];
#pragma unroll
      for (int m = 0; m < 5; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) a[m][o] = 0.f;
#pragma unroll
      for (int i = 0; i < RB + WIN - 1; i++) {
        // SSIM sees the inputs clamped to [0, 1] (spike/metrics.py:6-7)
        const float x = fminf(fmaxf(bx_[r * LG::XS + c0 + i], 0.f), 1.f);
        const float y = fminf(fmaxf(by_[r * LG::XS + c0 + i], 0.f), 1.f);
        const float xx = x * x, yy = y * y, xy = x * y;
#pragma unroll
        for (int o = 0; o < RB; o++) {
          const int k = i - o;
          if (k >= 0 && k < WIN) {
            a[0][o] = fmaf(g[k], x, a[0][o]);
            a[1][o] = fmaf(g[k], y, a[1][o]);
            a[2][o] = fmaf(g[k], xx, a[2][o]);
            a[3][o] = fmaf(g[k], yy, a[3][o]);
            a[4][o] = fmaf(g[k], xy, a[4][o]);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 5; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) h[(m * LG::IH + r) * LG::HS + c0 + o] = a[m][o];
    }
    __syncthreads();
    float ssum = 0.f;
    const long long plane = (long long)Ho * Wo;
    float* mbase = maps + (long long)vc * 3 * plane;
    for (int it = tid; it < LT_W * (LT_H / RB); it += 256) {
      const int c = it % LT_W, r0 = (it / LT_W) * RB;
      float f[5][RB];
#pragma unroll
      for (int m = 0; m < 5; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) f[m][o] = 0.f;
#pragma unroll
      for (int i = 0; i < RB + WIN - 1; i++) {
        float hv[5];
#pragma unroll
        for (int m = 0; m < 5; m++) hv[m] = h[(m * LG::IH + r0 + i) * LG::HS + c];
#pragma unroll
        for (int o = 0; o < RB; o++) {
          const int k = i - o;
          if (k >= 0 && k < WIN) {
#pragma unroll
            for (int m = 0; m < 5; m++) f[m][o] = fmaf(g[k], hv[m], f[m][o]);
          }
        }
      }
      const int ox = ox0 + c;
#pragma unroll
      for (int o = 0; o < RB; o++) {
        const int oy = oy0 + r0 + o;
        if (oy >= Ho || ox >= Wo) continue;
        const float mux = f[0][o], muy = f[1][o];
        const float mux2 = mux * mux, muy2 = muy * muy;
        const float sxx = f[2][o] - mux2, syy = f[3][o] - muy2, sxy = f[4][o] - mux * muy;
        const float A1 = 2.f * mux * muy + SSIM_C1, A2 = 2.f * sxy + SSIM_C2;
        const float B1 = mux2 + muy2 + SSIM_C1, B2 = sxx + syy + SSIM_C2;
        const float iD = 1.f / (B1 * B2), iB2 = 1.f / B2;
        const float S = (A1 * A2) * iD;
        ssum += S;
        const long long q = (long long)oy * Wo + ox;
        mbase[q] = 2.f * iD * (muy * (A2 - A1) - S * mux * (B2 - B1));   // dS/dmu_x
        mbase[plane + q] = -S * iB2;                                     // dS/d filt(x^2)
        mbase[2 * plane + q] = 2.f * A1 * iD;                            // dS/d filt(xy)
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if ((tid & 31) == 0) red[tid >> 5] = ssum;
    __syncthreads();
    if (tid == 0) {
      float s = 0.f;
      for (int i = 0; i < 8; ++i) s += red[i];
      part[(long long)vc * gx * gy + id.by * gx + id.bx] = s;
    }
    buf ^= 1;
  }
}

template <int WIN>
__global__ void __launch_bounds__(256)
    k_ssim_bwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, int gx, int gy, int ntiles,
               Window wd, float lambda, float grad_scale, const float* __restrict__ maps, float* __restrict__ gimg,
               float* __restrict__ part) {
  using LG = LGeom<WIN>;
  constexpr int BUF = 3 * LG::IH * LG::XS;
  extern __shared__ float smem[];
  float* sm = smem;                            // [2][3][IH][XS]
  float* h = sm + 2 * BUF;                     // [3][IH][HS]
  __shared__ float red[8];
  const int Ho = H - WIN + 1, Wo = W - WIN + 1;
  const int tid = threadIdx.x;
  float g[WIN];
#pragma unroll
  for (int k = 0; k < WIN; k++) g[k] = wd.g[k];
  const long long plane = (long long)Ho * Wo;
  // map rows [y0-WIN+1, y0+LT_H), cols [x0-WIN+1, x0+LT_W); zero outside the valid region
  auto issue = [&](int tile, int b) {
    const TileId id = decode_tile(tile, gx, gy);
    const int x0 = id.bx * LT_W, y0 = id.by * LT_H;
    const float* mbase = maps + (long long)(id.v * 3 + id.ch) * 3 * plane;
    for (int i = tid; i < LG::IH * LG::IW; i += 256) {
      const int r = i / LG::IW, c = i % LG::IW;
      const int my = y0 - (WIN - 1) + r, mx = x0 - (WIN - 1) + c;
      const bool in = my >= 0 && my < Ho && mx >= 0 && mx < Wo;
      const long long q = in ? (long long)my * Wo + mx : 0;
      float* d = sm + b * BUF + r * LG::XS + c;
      cp_async4(d, mbase + q, in ? 4 : 0);
      cp_async4(d + LG::IH * LG::XS, mbase + plane + q, in ? 4 : 0);
      cp_async4(d + 2 * LG::IH * LG::XS, mbase + 2 * plane + q, in ? 4 : 0);
    }
    cp_async_commit();
  };
  const float Ns = (float)(3.0 * (double)Ho * (double)Wo);
  const float N = (float)(3.0 * (double)H * (double)W);
  int buf = 0;
  if ((int)blockIdx.x < ntiles) issue(blockIdx.x, 0);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int next = tile + gridDim.x;
    if (next < ntiles) issue(next, buf ^ 1);
    else cp_async_commit();
    cp_async_wait_1();
    __syncthreads();
    const TileId id = decode_tile(tile, gx, gy);
    const int vc = id.v * 3 + id.ch;
    const int x0 = id.bx * LT_W, y0 = id.by * LT_H;
    const float* smb = sm + buf * BUF;
    // transposed row filter: t[r][c] = sum_k g[k] m[r][c + WIN-1 - k]
    for (int it = tid; it < LG::IH * (LT_W / RB); it += 256) {
      const int r = it % LG::IH, c0 = (it / LG::IH) * RB;
      float a[3][RB];
#pragma unroll
      for (int m = 0; m < 3; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) a[m][o] = 0.f;
#pragma unroll
      for (int i = 0; i < RB + WIN - 1; i++) {
        float mv[3];
#pragma unroll
        for (int m = 0; m < 3; m++) mv[m] = smb[(m * LG::IH + r) * LG::XS + c0 + i];
#pragma unroll
        for (int o = 0; o < RB; o++) {
          const int k = (WIN - 1) - (i - o);
          if (k >= 0 && k < WIN) {
#pragma unroll
            for (int m = 0; m < 3; m++) a[m][o] = fmaf(g[k], mv[m], a[m][o]);
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 3; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) h[(m * LG::IH + r) * LG::HS + c0 + o] = a[m][o];
    }
    __syncthreads();
    float l1 = 0.f;
    for (int it = tid; it < LT_W * (LT_H / RB); it += 256) {
      const int c = it % LT_W, r0 = (it / LT_W) * RB;
      float t[3][RB];
#pragma unroll
      for (int m = 0; m < 3; m++)
#pragma unroll
        for (int o = 0; o < RB; o++) t[m][o] = 0.f;
#pragma unroll
      for (int i = 0; i < RB + WIN - 1; i++) {
        float hv[3];
#pragma unroll
        for (int m = 0; m < 3; m++) hv[m] = h[(m * LG::IH + r0 + i) * LG::HS + c];
#pragma unroll
        for (int o = 0; o < RB; o++) {
          const int k = (WIN - 1) - (i - o);
          if (k >= 0 && k < WIN) {
#pragma unroll
            for (int m = 0; m < 3; m++) t[m][o] = fmaf(g[k], hv[m], t[m][o]);
          }
        }
      }
      const int xx = x0 + c;
#pragma unroll
      for (int o = 0; o < RB; o++) {
        const int yy = y0 + r0 + o;
        if (yy >= H || xx >= W) continue;
        const long long q = (((long long)id.v * H + yy) * W + xx) * 3 + id.ch;
        const float xr = img[q], yr = tgt[q];
        const float x = fminf(fmaxf(xr, 0.f), 1.f), y = fminf(fmaxf(yr, 0.f), 1.f);
        const float mask = (xr >= 0.f && xr <= 1.f) ? 1.f : 0.f;
        const float dmean = (t[0][o] + 2.f * x * t[1][o] + y * t[2][o]) / Ns;
        const float diff = xr - yr;
        const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
        l1 += fabsf(diff);
        gimg[q] = grad_scale * ((1.f - lambda) * sgn / N + lambda * (-dmean) * mask);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    if ((tid & 31) == 0) red[tid >> 5] = l1;
    __syncthreads();
    if (tid == 0) {
      float s = 0.f;
      for (int i = 0; i < 8; ++i) s += red[i];
      part[(long long)vc * gx * gy + id.by * gx + id.bx] = s;
    }
    buf ^= 1;
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

template <int WIN>
static int launch_loss(const float* img, const float* target, int V, int H, int W, float lambda, float grad_scale,
                       const Window& wd, const LossGeom& lg, float* maps, float* spart, float* lpart, float* gimg,
                       cudaStream_t st) {
  using LG = LGeom<WIN>;
  const size_t fsm = (size_t)(4 * LG::IH * LG::XS + 5 * LG::IH * LG::HS) * 4;
  const size_t bsm = (size_t)(6 * LG::IH * LG::XS + 3 * LG::IH * LG::HS) * 4;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(k_ssim_fwd<WIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsm);
    cudaFuncSetAttribute(k_ssim_bwd<WIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm);
    attr_set = true;
  }
  const int nf = V * 3 * lg.fbx * lg.fby, nb = V * 3 * lg.bbx * lg.bby;
  const int resident = 148 * 2;     // two blocks per SM fit the double-buffered tiles
  k_ssim_fwd<WIN><<<(unsigned)(nf < resident ? nf : resident), 256, fsm, st>>>(img, target, H, W, lg.fbx, lg.fby, nf, wd,
                                                                                maps, spart);
  if (int rc = check_launch("ssim_fwd")) return rc;
  k_ssim_bwd<WIN><<<(unsigned)(nb < resident ? nb : resident), 256, bsm, st>>>(img, target, H, W, lg.bbx, lg.bby, nb, wd,
                                                                                lambda, grad_scale, maps, gimg, lpart);
  return check_launch("ssim_bwd");
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
  int rc;
  switch (wd.win) {
    case 3: rc = launch_loss<3>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, st); break;
    case 5: rc = launch_loss<5>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, st); break;
    case 7: rc = launch_loss<7>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, st); break;
    case 9: rc = launch_loss<9>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, st); break;
    default: rc = launch_loss<11>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, st); break;
  }
  if (rc) return rc;
  k_loss_reduce<<<V, 256, 0, st>>>(spart, lg.fbx * lg.fby, lpart, lg.bbx * lg.bby, H, W, lg.win, lambda, loss);
  return check_launch("loss_reduce");
}
