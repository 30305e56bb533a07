// Photometric loss (1-l) L1 + l (1 - SSIM) and its gradient (replaces metrics.loss_fn,
// spike/metrics.py:26-28, with the manual gradient of tools/loss_manual.py:78-105).
//
// SSIM uses the valid separable Gaussian window (tools/loss_manual.py:28-55; pytorch_msssim
// convention) on inputs clamped to [0,1] (spike/metrics.py:6-7).  Two tiled kernels, each a
// separable filter with register blocking so that every shared-memory load feeds several FMAs
// (a thread slides an RB-long window along a row, then along a column), with the maps paired in
// sm_100a .f32x2 FMAs:
//   k_ssim_fwd : output tile 64x32 of the SSIM map.  Loads the (64+win-1)x(32+win-1) input
//                halo, filters the four maps x, y, x^2 + y^2, xy along rows then columns (SSIM
//                sees the variances only through their sum sigma_x^2 + sigma_y^2, so x^2 and
//                y^2 are filtered as one map), and writes dS/dmu_x, dS/d(filtered x^2),
//                dS/d(filtered xy) plus a per-block partial of sum(S).
//   k_ssim_bwd : input tile 64x32.  Applies the transposed filter to the three dS maps (zero
//                outside the valid region), combines them with x and y into the SSIM gradient,
//                adds the L1 gradient, and writes a per-block partial of sum|x - y|.
// A one-block-per-view kernel reduces the partials in a fixed order (deterministic).
#include "common.cuh"

namespace tts {

constexpr int LT_W = 64, LT_H = 32, LWIN_MAX = 11, RB = 8;
// Row passes: each of the IH rows is cut into 6 segments of 11, 11, 11, 11, 10, 10 outputs, so
// that IH x 6 = 252 items keep the 256 threads busy in one round (segments of RB = 8 would give
// 336 items: two rounds, the second a third full).
constexpr int RSEGS = 6, RBR = 11;
static_assert(4 * 11 + 2 * 10 == LT_W, "row segments cover the tile width");
__device__ __forceinline__ void row_seg(int s, int& c0, int& width) {
  c0 = s < 4 ? 11 * s : 44 + 10 * (s - 4);
  width = s < 4 ? 11 : 10;
}
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

// Packed f32x2 arithmetic on (x, y) and (x^2 + y^2, xy): the four filtered maps cost two .f32x2
// FMAs per tap.
template <int WIN>
__global__ void __launch_bounds__(256)
    k_ssim_fwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, int gx, int gy, Window wd,
               float* __restrict__ maps, float* __restrict__ part, unsigned* __restrict__ reduce_counter) {
  using LG = LGeom<WIN>;
  extern __shared__ float smem[];
  f32x2* sxy = reinterpret_cast<f32x2*>(smem);                    // [IH][XS] (x, y) clamped
  f32x2* hxy = sxy + LG::IH * LG::XS;                             // [IH][HS] row-filtered (x, y)
  f32x2* hqp = hxy + LG::IH * LG::HS;                             // [IH][HS] row-filtered (x^2 + y^2, xy)
  __shared__ float red[8];
  const int Ho = H - WIN + 1, Wo = W - WIN + 1;
  const TileId id = decode_tile(blockIdx.x, gx, gy);
  const int vc = id.v * 3 + id.ch;
  const int ox0 = id.bx * LT_W, oy0 = id.by * LT_H;
  const int tid = threadIdx.x;
  if (blockIdx.x == 0 && tid == 0) *reduce_counter = 0u;   // for the last-block total of k_loss_reduce
  float g[WIN];
  f32x2 g2[WIN];
#pragma unroll
  for (int k = 0; k < WIN; k++) {
    g[k] = wd.g[k];
    g2[k] = mk2(g[k], g[k]);
  }
  {
    // issue every load of the halo tile before the first shared-memory store: thread -> one
    // column and every RPT-th row (no per-element index division)
    constexpr int RPT = 256 / LG::IW, NR = (LG::IH + RPT - 1) / RPT;
    const int lc = tid % LG::IW, lr0 = tid / LG::IW;
    if (lr0 < RPT) {
      const int xx = ox0 + lc;
      // this thread's rows lr0, lr0 + RPT, ... inside both the halo tile and the image: the
      // first kn of them (bounds hoisted out of the loads)
      const int rows = min(LG::IH, H - oy0);
      const int kn = xx < W ? (rows - lr0 + RPT - 1) / RPT : 0;
      const long long base = (((long long)id.v * H + oy0 + lr0) * W + xx) * 3 + id.ch;
      const int step = 3 * W * RPT;
      float xv[NR], yv[NR];
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        xv[k] = 0.f;
        yv[k] = 0.f;
        if (k < kn) {
          xv[k] = __ldg(img + base + k * step);
          yv[k] = __ldg(tgt + base + k * step);
        }
      }
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        const int r = lr0 + RPT * k;
        // SSIM sees the inputs clamped to [0, 1] (spike/metrics.py:6-7)
        if (r < LG::IH) sxy[r * LG::XS + lc] = mk2(fminf(fmaxf(xv[k], 0.f), 1.f), fminf(fmaxf(yv[k], 0.f), 1.f));
      }
    }
  }
  __syncthreads();
  // rows: item = (row r, segment of up to RBR outputs); lanes walk down rows (odd stride).  The
  // last input read of a 10-wide segment is the row's padding column, never used.
  for (int it = tid; it < LG::IH * RSEGS; it += 256) {
    const int r = it % LG::IH;
    int c0, width;
    row_seg(it / LG::IH, c0, width);
    const f32x2 z = mk2(0.f, 0.f);
    f32x2 axy[RBR], aqp[RBR];
#pragma unroll
    for (int o = 0; o < RBR; o++) {
      axy[o] = z;
      aqp[o] = z;
    }
#pragma unroll
    for (int i = 0; i < RBR + WIN - 1; i++) {
      const f32x2 XY = sxy[r * LG::XS + c0 + i];
      float x, y;
      split2(XY, x, y);
      const f32x2 QP = mk2(fmaf(x, x, y * y), x * y);
#pragma unroll
      for (int o = 0; o < RBR; o++) {
        const int k = i - o;
        if (k >= 0 && k < WIN) {
          axy[o] = fma2(g2[k], XY, axy[o]);
          aqp[o] = fma2(g2[k], QP, aqp[o]);
        }
      }
    }
#pragma unroll
    for (int o = 0; o < RBR; o++) {
      if (o < width) {
        hxy[r * LG::HS + c0 + o] = axy[o];
        hqp[r * LG::HS + c0 + o] = aqp[o];
      }
    }
  }
  __syncthreads();
  // columns: item = (column c, segment of RB output rows); lanes walk along columns
  float ssum = 0.f;
  const long long plane = (long long)Ho * Wo;
  float4* mbase = reinterpret_cast<float4*>(maps) + (long long)vc * plane;   // (M0, M1, M2, 0) per position
  for (int it = tid; it < LT_W * (LT_H / RB); it += 256) {
    const int c = it % LT_W, r0 = (it / LT_W) * RB;
    const f32x2 z = mk2(0.f, 0.f);
    f32x2 fxy[RB], fqp[RB];
#pragma unroll
    for (int o = 0; o < RB; o++) {
      fxy[o] = z;
      fqp[o] = z;
    }
#pragma unroll
    for (int i = 0; i < RB + WIN - 1; i++) {
      const f32x2 XY = hxy[(r0 + i) * LG::HS + c];
      const f32x2 QP = hqp[(r0 + i) * LG::HS + c];
#pragma unroll
      for (int o = 0; o < RB; o++) {
        const int k = i - o;
        if (k >= 0 && k < WIN) {
          fxy[o] = fma2(g2[k], XY, fxy[o]);
          fqp[o] = fma2(g2[k], QP, fqp[o]);
        }
      }
    }
    const int ox = ox0 + c;
    const int on = ox < Wo ? min(RB, Ho - oy0 - r0) : 0;     // outputs of this item in the map
    float4* mp = mbase + (long long)(oy0 + r0) * Wo + ox;
#pragma unroll
    for (int o = 0; o < RB; o++) {
      if (o >= on) continue;
      float mux, muy, fss, fxy1;
      split2(fxy[o], mux, muy);
      split2(fqp[o], fss, fxy1);
      const float mm = mux * mux + muy * muy;       // mu_x^2 + mu_y^2
      const float sxy_ = fxy1 - mux * muy;
      const float A1 = 2.f * mux * muy + SSIM_C1, A2 = 2.f * sxy_ + SSIM_C2;
      const float B1 = mm + SSIM_C1, B2 = (fss - mm) + SSIM_C2;   // sigma_x^2 + sigma_y^2 + C2
      // hardware reciprocals (rcp.approx, within 1 ulp): the loss and gradient tolerances are
      // orders of magnitude wider, and the correctly rounded form costs ~20 instructions more
      float iD, iB2;
      asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(iD) : "f"(B1 * B2));
      asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(iB2) : "f"(B2));
      const float S = (A1 * A2) * iD;
      ssum += S;
      mp[o * Wo] = make_float4(2.f * iD * (muy * (A2 - A1) - S * mux * (B2 - B1)),   // dS/dmu_x
                             -S * iB2,                                             // dS/d filt(x^2)
                             2.f * A1 * iD, 0.f);                                  // dS/d filt(xy)
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
}

// Transposed filter of (dS/dmu_x, dS/d filt(x^2)) as one .f32x2 pair and dS/d filt(xy) alone.
template <int WIN>
__global__ void __launch_bounds__(256)
    k_ssim_bwd(const float* __restrict__ img, const float* __restrict__ tgt, int H, int W, int gx, int gy, Window wd,
               float lambda, float grad_scale, const float* __restrict__ maps, float* __restrict__ gimg,
               float* __restrict__ part) {
  using LG = LGeom<WIN>;
  extern __shared__ float smem[];
  f32x2* s01 = reinterpret_cast<f32x2*>(smem);                    // [IH][XS] (m0, m1)
  float* s2 = reinterpret_cast<float*>(s01 + LG::IH * LG::XS);    // [IH][XS] m2
  f32x2* h01 = reinterpret_cast<f32x2*>(smem + 3 * LG::IH * LG::XS + (LG::IH * LG::XS & 1));
  float* h2 = reinterpret_cast<float*>(h01 + LG::IH * LG::HS);
  __shared__ float red[8];
  const int Ho = H - WIN + 1, Wo = W - WIN + 1;
  const TileId id = decode_tile(blockIdx.x, gx, gy);
  const int vc = id.v * 3 + id.ch;
  const int x0 = id.bx * LT_W, y0 = id.by * LT_H;
  const int tid = threadIdx.x;
  float g[WIN];
  f32x2 g2[WIN];
#pragma unroll
  for (int k = 0; k < WIN; k++) {
    g[k] = wd.g[k];
    g2[k] = mk2(g[k], g[k]);
  }
  const long long plane = (long long)Ho * Wo;
  const float4* mbase = reinterpret_cast<const float4*>(maps) + (long long)vc * plane;
  // the image/target values of this thread's epilogue (one column item per thread: LT_W x LT_H/RB
  // = 256 items) are fetched up front, together with the map halo
  static_assert(LT_W * (LT_H / RB) == 256, "one column item per thread");
  const int ec = tid % LT_W, er0 = (tid / LT_W) * RB;
  // rows of this item inside the image, and the image offset of its first pixel
  const int en = x0 + ec < W ? min(RB, H - y0 - er0) : 0;
  const long long eb = (((long long)id.v * H + y0 + er0) * W + x0 + ec) * 3 + id.ch;
  float ximg[RB], xtgt[RB];
#pragma unroll
  for (int o = 0; o < RB; o++) {
    ximg[o] = 0.f;
    xtgt[o] = 0.f;
    if (o < en) {
      ximg[o] = __ldg(img + eb + o * 3 * W);
      xtgt[o] = __ldg(tgt + eb + o * 3 * W);
    }
  }
  {
    // map rows [y0-WIN+1, y0+LT_H), cols [x0-WIN+1, x0+LT_W); zero outside the valid region;
    // thread -> one column and every RPT-th row
    constexpr int RPT = 256 / LG::IW, NR = (LG::IH + RPT - 1) / RPT;
    const int lc = tid % LG::IW, lr0 = tid / LG::IW;
    if (lr0 < RPT) {
      const int mx = x0 - (WIN - 1) + lc;
      const bool colok = mx >= 0 && mx < Wo;
      // this thread's rows lr0 + RPT k with map row my in [0, Ho) and r < IH: k in [klo, khi)
      const int m0 = y0 - (WIN - 1) + lr0;                       // map row of k = 0
      const int klo = m0 >= 0 ? 0 : (-m0 + RPT - 1) / RPT;
      const int khi = colok ? min((LG::IH - lr0 + RPT - 1) / RPT, (Ho - m0 + RPT - 1) / RPT) : 0;
      const long long mb0 = (long long)m0 * Wo + mx;
      float av[NR], bv[NR], dv[NR];
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        av[k] = 0.f;
        bv[k] = 0.f;
        dv[k] = 0.f;
        if (k >= klo && k < khi) {
          const float4 mm = __ldg(mbase + (mb0 + (long long)k * RPT * Wo));
          av[k] = mm.x;
          bv[k] = mm.y;
          dv[k] = mm.z;
        }
      }
#pragma unroll
      for (int k = 0; k < NR; ++k) {
        const int r = lr0 + RPT * k;
        if (r < LG::IH) {
          s01[r * LG::XS + lc] = mk2(av[k], bv[k]);
          s2[r * LG::XS + lc] = dv[k];
        }
      }
    }
  }
  __syncthreads();
  // transposed row filter: t[r][c] = sum_k g[k] m[r][c + WIN-1 - k]
  for (int it = tid; it < LG::IH * RSEGS; it += 256) {
    const int r = it % LG::IH;
    int c0, width;
    row_seg(it / LG::IH, c0, width);
    const f32x2 z = mk2(0.f, 0.f);
    f32x2 a01[RBR];
    float a2[RBR];
#pragma unroll
    for (int o = 0; o < RBR; o++) {
      a01[o] = z;
      a2[o] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < RBR + WIN - 1; i++) {
      const f32x2 M01 = s01[r * LG::XS + c0 + i];
      const float M2 = s2[r * LG::XS + c0 + i];
#pragma unroll
      for (int o = 0; o < RBR; o++) {
        const int k = (WIN - 1) - (i - o);
        if (k >= 0 && k < WIN) {
          a01[o] = fma2(g2[k], M01, a01[o]);
          a2[o] = fmaf(g[k], M2, a2[o]);
        }
      }
    }
#pragma unroll
    for (int o = 0; o < RBR; o++) {
      if (o < width) {
        h01[r * LG::HS + c0 + o] = a01[o];
        h2[r * LG::HS + c0 + o] = a2[o];
      }
    }
  }
  __syncthreads();
  const float inv_Ns = (float)(1.0 / (3.0 * (double)Ho * (double)Wo));
  const float l1w = (float)((1.0 - (double)lambda) / (3.0 * (double)H * (double)W));
  float l1 = 0.f;
  {
    const int c = ec, r0 = er0;
    const f32x2 z = mk2(0.f, 0.f);
    f32x2 t01[RB];
    float t2[RB];
#pragma unroll
    for (int o = 0; o < RB; o++) {
      t01[o] = z;
      t2[o] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < RB + WIN - 1; i++) {
      const f32x2 H01 = h01[(r0 + i) * LG::HS + c];
      const float H2 = h2[(r0 + i) * LG::HS + c];
#pragma unroll
      for (int o = 0; o < RB; o++) {
        const int k = (WIN - 1) - (i - o);
        if (k >= 0 && k < WIN) {
          t01[o] = fma2(g2[k], H01, t01[o]);
          t2[o] = fmaf(g[k], H2, t2[o]);
        }
      }
    }
#pragma unroll
    for (int o = 0; o < RB; o++) {
      if (o >= en) continue;
      const long long q = eb + o * 3 * W;
      const float xr = ximg[o], yr = xtgt[o];
      const float x = fminf(fmaxf(xr, 0.f), 1.f), y = fminf(fmaxf(yr, 0.f), 1.f);
      const float mask = (xr >= 0.f && xr <= 1.f) ? 1.f : 0.f;
      float t0, t1;
      split2(t01[o], t0, t1);
      const float dmean = (t0 + 2.f * x * t1 + y * t2[o]) * inv_Ns;
      const float diff = xr - yr;
      const float sgn = diff > 0.f ? 1.f : (diff < 0.f ? -1.f : 0.f);
      l1 += fabsf(diff);
      gimg[q] = grad_scale * (l1w * sgn + lambda * (-dmean) * mask);
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
}

// lambda == 0 (the L1 loss alone, spike/metrics.py:22-23 / loss_fn with lambda_ssim = 0): the
// L1 gradient grad_scale * sign(x - y) / N and a per-block partial of sum|x - y|, no SSIM pass.
__global__ void __launch_bounds__(256)
    k_l1_only(const float* __restrict__ img, const float* __restrict__ tgt, long long n_per_view, int blocks_per_view,
              float gscale, float* __restrict__ gimg, float* __restrict__ part) {
  __shared__ float red[8];
  const int v = blockIdx.x / blocks_per_view, b = blockIdx.x % blocks_per_view;
  const long long base = (long long)v * n_per_view;
  float l1 = 0.f;
  for (long long i = (long long)b * 256 + threadIdx.x; i < n_per_view; i += (long long)blocks_per_view * 256) {
    const float d = img[base + i] - tgt[base + i];
    l1 += fabsf(d);
    gimg[base + i] = gscale * (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = l1;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += red[i];
    part[blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(256) k_loss_reduce(const float* __restrict__ spart, int nsb, const float* __restrict__ lpart,
                                                     int nlb, int H, int W, int win, float lambda, float* __restrict__ loss,
                                                     float* __restrict__ loss_sum, unsigned* __restrict__ counter) {
  __shared__ double rs[8], rl[8];
  __shared__ bool s_last;
  const int v = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  // fixed-order sums (deterministic): four independent partials per thread, then the warps'
  // xor butterflies, then the 8 warp sums in warp order
  auto part_sum = [&](const float* p, int n) {
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
    int i = tid;
    for (; i + 768 < n; i += 1024) {
      a0 += p[i];
      a1 += p[i + 256];
      a2 += p[i + 512];
      a3 += p[i + 768];
    }
    for (; i < n; i += 256) a0 += p[i];
    return (a0 + a1) + (a2 + a3);
  };
  double s = part_sum(spart + (long long)v * 3 * nsb, 3 * nsb);
  double l = part_sum(lpart + (long long)v * 3 * nlb, 3 * nlb);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    l += __shfl_xor_sync(0xffffffffu, l, o);
  }
  if (lane == 0) {
    rs[wid] = s;
    rl[wid] = l;
  }
  __syncthreads();
  if (tid == 0) {
    double S = 0.0, Lt = 0.0;
    for (int w = 0; w < 8; ++w) {
      S += rs[w];
      Lt += rl[w];
    }
    const double Ns = 3.0 * (double)(H - win + 1) * (double)(W - win + 1);
    const double N = 3.0 * (double)H * (double)W;
    loss[v] = (float)((1.0 - lambda) * Lt / N + lambda * (1.0 - S / Ns));
  }
  if (loss_sum == nullptr) return;
  // the last block to finish adds the V losses in view order
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    const volatile float* lv = loss;
    float tot = 0.f;
    for (int i = 0; i < (int)gridDim.x; ++i) tot += lv[i];
    *loss_sum = tot;
    *counter = 0u;
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
                       unsigned* counter, cudaStream_t st) {
  using LG = LGeom<WIN>;
  const size_t fsm = (size_t)(LG::IH * LG::XS * 2 + LG::IH * LG::HS * 4) * 4;
  const size_t bsm = (size_t)(LG::IH * LG::XS * 3 + (LG::IH * LG::XS & 1) + LG::IH * LG::HS * 3) * 4;
  static std::atomic<unsigned long long> attr_done{0};
  once_per_device(attr_done, [&] {
    cudaFuncSetAttribute(k_ssim_fwd<WIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsm);
    cudaFuncSetAttribute(k_ssim_bwd<WIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm);
  });
  k_ssim_fwd<WIN><<<(unsigned)(V * 3 * lg.fbx * lg.fby), 256, fsm, st>>>(img, target, H, W, lg.fbx, lg.fby, wd, maps,
                                                                        spart, counter);
  if (int rc = check_launch("ssim_fwd")) return rc;
  k_ssim_bwd<WIN><<<(unsigned)(V * 3 * lg.bbx * lg.bby), 256, bsm, st>>>(img, target, H, W, lg.bbx, lg.bby, wd, lambda,
                                                                        grad_scale, maps, gimg, lpart);
  return check_launch("ssim_bwd");
}

}  // namespace tts

using namespace tts;

extern "C" size_t tts_loss_workspace_bytes(int V, int H, int W) {
  if (V < 1 || H < 3 || W < 3) return 0;
  const LossGeom lg = loss_geom(H, W);
  return a256((size_t)V * 12 * lg.Ho * lg.Wo * 4) + a256((size_t)V * 3 * lg.fbx * lg.fby * 4) +
         a256((size_t)V * 3 * lg.bbx * lg.bby * 4) + 256;   // + the reduce counter
}

extern "C" int tts_loss_l1_ssim(const float* img, const float* target, int V, int H, int W, float lambda,
                                float grad_scale, float* gimg, float* loss, float* loss_sum, void* workspace,
                                size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(V >= 1 && H >= 3 && W >= 3, "images must be at least 3x3");
  TTS_REQUIRE(img && target && gimg && loss && workspace, "null pointer");
  if (workspace_bytes < tts_loss_workspace_bytes(V, H, W)) return fail(TTS_ERR_CAPACITY, "loss workspace too small");
  Window wd;
  window_for(H, W, wd);
  const LossGeom lg = loss_geom(H, W);
  char* p = static_cast<char*>(workspace);
  float* maps = reinterpret_cast<float*>(p);
  p += a256((size_t)V * 12 * lg.Ho * lg.Wo * 4);
  float* spart = reinterpret_cast<float*>(p);
  p += a256((size_t)V * 3 * lg.fbx * lg.fby * 4);
  float* lpart = reinterpret_cast<float*>(p);
  p += a256((size_t)V * 3 * lg.bbx * lg.bby * 4);
  unsigned* counter = reinterpret_cast<unsigned*>(p);
  cudaStream_t st = as_stream(stream);
  if (lambda == 0.f) {
    // L1 alone: one pass over the pixels, partials reduced per view in block order
    const long long npv = 3LL * H * W, cap = 3LL * lg.bbx * lg.bby;   // partials: the lpart slots
    const long long want = (npv + 255) / 256 < cap ? (npv + 255) / 256 : cap;
    const int bpv = (int)((want + 2) / 3 * 3);                         // a multiple of 3, <= cap
    if (cudaMemsetAsync(counter, 0, sizeof(unsigned), st) != cudaSuccess) return check_launch("memset loss counter");
    k_l1_only<<<(unsigned)(V * bpv), 256, 0, st>>>(img, target, npv, bpv, (float)((double)grad_scale / (double)npv),
                                                   gimg, lpart);
    if (int rc = check_launch("l1_only")) return rc;
    k_loss_reduce<<<V, 256, 0, st>>>(spart, 0, lpart, bpv / 3, H, W, lg.win, lambda, loss, loss_sum, counter);
    return check_launch("loss_reduce");
  }
  int rc;
  switch (wd.win) {
    case 3: rc = launch_loss<3>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, counter, st); break;
    case 5: rc = launch_loss<5>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, counter, st); break;
    case 7: rc = launch_loss<7>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, counter, st); break;
    case 9: rc = launch_loss<9>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, counter, st); break;
    default: rc = launch_loss<11>(img, target, V, H, W, lambda, grad_scale, wd, lg, maps, spart, lpart, gimg, counter, st); break;
  }
  if (rc) return rc;
  k_loss_reduce<<<V, 256, 0, st>>>(spart, lg.fbx * lg.fby, lpart, lg.bbx * lg.bby, H, W, lg.win, lambda, loss,
                                   loss_sum, counter);
  return check_launch("loss_reduce");
}
