// Fused per-tile poly-splat + WSR forward and backward (one CTA per 16x16 tile per view).
//
// Forward (replaces _DevRenderBinned.forward, tools/m4_train_binned.py:156-166): the tile's
// slot rows (theta_u[6] | color_o[3] | o_col) are staged in shared memory by one bulk copy
// (cp.async.bulk, completion on an mbarrier); one warp renders the tile, each lane owning eight
// adjacent pixels of one tile row (four sm_100a packed .f32x2 pairs, so the per-slot row terms
// are shared by eight pixels), and loops over the slots with the rows broadcast from shared
// memory:
//   u = theta . Phi(px, py) = (t0 px + (t2 py + t3)) px + ((t1 py + t4) py + t5)
//   w = max(u, 0)^2;  num += w color_o;  den += w o_col
// u = 1 - Q/k with Q >= 0 for the positive-definite conics the projection produces, so u <= 1
// and max(u, 0) is the last FMA of u saturated to [0, 1] (both kernels).
// then C = (num + w_b c_b) / (den + w_b).  The [256 x K] weight matrix never leaves registers.
//
// Backward (replaces _DevRenderBinned.backward :169-186 / WSRPolySplatHot.backward,
// spike/backward.py:43-58): one thread per slot, looping over the tile's 256 pixels whose
// (gnum = gC/den, gden = -(gC.C)/den) are broadcast from shared memory; every per-slot sum
// (gcolor_o = w^T gnum, go_col = w^T gden, gtheta = Phi^T (2 relu(u) gw)) stays in the
// thread's registers, so no cross-thread reduction is needed.  gtheta is accumulated per row
// through the moments sum(gu), sum(gu px), sum(gu px^2); adjacent pixels run as .f32x2 pairs.
#include "common.cuh"

namespace tts {

constexpr int FWD_THREADS = 32;   // one warp per tile: 8 pixels per lane (half of one row)
constexpr int RV_THREADS = 64;    // arm RV forward: 4 pixels per thread (two adjacent pairs of one row)
constexpr int KMAX = 256;

template <bool BF16>
__global__ void __launch_bounds__(FWD_THREADS)
    k_render_fwd(const void* __restrict__ slots_, const int* __restrict__ count, int ntx, int T, int H, int W, int K,
                 const float* __restrict__ w_b_ptr, int w_b_is_raw, const float* __restrict__ c_b,
                 float* __restrict__ img, float* __restrict__ den_out) {
  extern __shared__ __align__(128) float s_rows[];    // K slot rows (sized at launch: more tiles per SM)
  __shared__ __align__(8) uint64_t bar;
  const int t = blockIdx.x, v = blockIdx.y, lane = threadIdx.x;
  const int n = count[(long long)v * T + t];
  const long long row0 = ((long long)v * T + t) * K;
  if (!BF16) {
    const float* src = static_cast<const float*>(slots_) + row0 * TTS_SLOT_FLOATS;
    if (lane == 0) mbar_init(&bar, 1);
    __syncwarp();
    if (n > 0) {
      if (lane == 0) {
        const uint32_t bytes = (uint32_t)n * TTS_SLOT_FLOATS * 4u;
        mbar_expect_tx(&bar, bytes);
        bulk_g2s(s_rows, src, bytes, &bar);
      }
      if (!mbar_wait_bounded(&bar, 0)) return;   // status recorded; nothing of the tile is written
    }
  } else {
    // compact bf16 rows (32 B: theta hi[6], theta lo[6], color_o[3], o_col) -> fp32 rows in
    // shared memory, theta_u = hi + lo
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(slots_) + row0 * TTS_SLOT_BF16);
    for (int sl = lane; sl < n; sl += FWD_THREADS) {
      const uint4 lo8 = src[2 * sl], hi8 = src[2 * sl + 1];
      const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&lo8);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&hi8);
      float* d = s_rows + sl * TTS_SLOT_FLOATS;
      // a[0..5] theta hi, a[6..7] + b[0..3] theta lo, b[4..6] color_o, b[7] o_col
      d[0] = __bfloat162float(a[0]) + __bfloat162float(a[6]);
      d[1] = __bfloat162float(a[1]) + __bfloat162float(a[7]);
      d[2] = __bfloat162float(a[2]) + __bfloat162float(b[0]);
      d[3] = __bfloat162float(a[3]) + __bfloat162float(b[1]);
      d[4] = __bfloat162float(a[4]) + __bfloat162float(b[2]);
      d[5] = __bfloat162float(a[5]) + __bfloat162float(b[3]);
      d[6] = __bfloat162float(b[4]);
      d[7] = __bfloat162float(b[5]);
      d[8] = __bfloat162float(b[6]);
      d[9] = __bfloat162float(b[7]);
      d[10] = 0.f;
      d[11] = 0.f;
    }
    __syncwarp();
  }

  // the binning marks a slot whose weight is zero at every pixel of the tile (row field 10, see
  // slot_dead); the live rows are moved to the front in slot order (the per-pixel sums keep
  // their order: a dead slot would only add exact zeros).  Each 32-row chunk is read before it is
  // written, and a row only moves down.  Compact bf16 rows carry no mark.
  int n_live = n;
  if (!BF16) {
    n_live = 0;
    for (int c0 = 0; c0 < n; c0 += FWD_THREADS) {
      const int sl = c0 + lane;
      float4 r0 = make_float4(0.f, 0.f, 0.f, 0.f), r1 = r0, r2 = r0;
      if (sl < n) {
        const float4* src = reinterpret_cast<const float4*>(s_rows) + 3 * sl;
        r0 = src[0];
        r1 = src[1];
        r2 = src[2];
      }
      const bool live = sl < n && r2.z == 0.f;
      const unsigned bal = __ballot_sync(0xffffffffu, live);
      if (bal != (c0 + FWD_THREADS <= n ? 0xffffffffu : (1u << (n - c0)) - 1u) || n_live != c0) {
        // something to move in this chunk
        __syncwarp();
        if (live) {
          float4* dst = reinterpret_cast<float4*>(s_rows) + 3 * (n_live + __popc(bal & ((1u << lane) - 1u)));
          dst[0] = r0;
          dst[1] = r1;
          dst[2] = r2;
        }
      }
      n_live += __popc(bal);
    }
    __syncwarp();
  }
  const float wb = w_b_is_raw ? softplusf(*w_b_ptr) : *w_b_ptr;
  // lane -> row ly, pixels x0 .. x0+7 (four adjacent pairs); one row's srow/rrow serve 8 pixels
  const int ly = lane >> 1, x0 = 8 * (lane & 1);
  const float py = (float)ly + 0.5f;
  f32x2 px[4];
#pragma unroll
  for (int j = 0; j < 4; j++) px[j] = mk2((float)(x0 + 2 * j) + 0.5f, (float)(x0 + 2 * j) + 1.5f);
  const f32x2 z = mk2(0.f, 0.f);
  f32x2 a0[4], a1[4], a2[4], a3[4];
#pragma unroll
  for (int j = 0; j < 4; j++) a0[j] = a1[j] = a2[j] = a3[j] = z;
  const float4* rows = reinterpret_cast<const float4*>(s_rows);
  for (int s = 0; s < n_live; ++s) {
    const float4 A = rows[3 * s + 0];   // t0 t1 t2 t3
    const float4 B = rows[3 * s + 1];   // t4 t5 cr cg
    const float4 C = rows[3 * s + 2];   // cb oc 0 0
    const float srow = fmaf(A.z, py, A.w);
    const float rrow = fmaf(fmaf(A.y, py, B.x), py, B.y);
    const f32x2 t0 = mk2(A.x, A.x), s2 = mk2(srow, srow);
    const f32x2 cr = mk2(B.z, B.z), cg = mk2(B.w, B.w), cb = mk2(C.x, C.x), oc = mk2(C.y, C.y);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const f32x2 r = fma_sat2(fma2(t0, px[j], s2), px[j], rrow);
      const f32x2 w = mul2(r, r);
      a0[j] = fma2(w, cr, a0[j]);
      a1[j] = fma2(w, cg, a1[j]);
      a2[j] = fma2(w, cb, a2[j]);
      a3[j] = fma2(w, oc, a3[j]);
    }
  }
  const int tx = t % ntx, ty = t / ntx;
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  const long long p0 = ((long long)v * H + ty * 16 + ly) * W + tx * 16 + x0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    float n0[2], n1[2], n2[2], dd[2];
    split2(a0[j], n0[0], n0[1]);
    split2(a1[j], n1[0], n1[1]);
    split2(a2[j], n2[0], n2[1]);
    split2(a3[j], dd[0], dd[1]);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const long long p = p0 + 2 * j + i;
      const float d = dd[i] + wb;
      img[3 * p + 0] = (n0[i] + wb * cb0) / d;
      img[3 * p + 1] = (n1[i] + wb * cb1) / d;
      img[3 * p + 2] = (n2[i] + wb * cb2) / d;
      den_out[p] = d;
    }
  }
}

__global__ void __launch_bounds__(256, 3)
    k_render_bwd(const float* __restrict__ slots, const int* __restrict__ count, int ntx, int T, int H, int W, int K,
                 const float* __restrict__ c_b, const float* __restrict__ img, const float* __restrict__ den,
                 const float* __restrict__ gimg, float* __restrict__ slot_grads, float* __restrict__ gwb_partial) {
  // per-pixel upstream terms, one array per component so that two adjacent pixels load as a pair
  __shared__ __align__(16) float s_g0[256], s_g1[256], s_g2[256], s_gd[256];
  __shared__ float s_red[32];
  const int t = blockIdx.x, v = blockIdx.y, tid = threadIdx.x;
  const int tx = t % ntx, ty = t / ntx;
  const int n = count[(long long)v * T + t];
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  // gnum = gC/den, gden = -(gC.C)/den (tools/m4_train_binned.py:178-179, spike/backward.py:46-48)
  float wbp = 0.f;
  for (int p = tid; p < 256; p += blockDim.x) {
    const long long q = ((long long)v * H + ty * 16 + (p >> 4)) * W + tx * 16 + (p & 15);
    const float g0 = gimg[3 * q], g1 = gimg[3 * q + 1], g2 = gimg[3 * q + 2];
    const float c0 = img[3 * q], c1 = img[3 * q + 1], c2 = img[3 * q + 2];
    const float inv = __frcp_rn(den[q]);   // one correctly rounded reciprocal instead of four divisions
    const float gn0 = g0 * inv, gn1 = g1 * inv, gn2 = g2 * inv;
    const float gd = -(g0 * c0 + g1 * c1 + g2 * c2) * inv;
    s_g0[p] = gn0;
    s_g1[p] = gn1;
    s_g2[p] = gn2;
    s_gd[p] = gd;
    wbp += gn0 * cb0 + gn1 * cb1 + gn2 * cb2 + gd;
  }
  // deterministic block reduction of the w_b partial
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wbp += __shfl_xor_sync(0xffffffffu, wbp, o);
  if ((tid & 31) == 0) s_red[tid >> 5] = wbp;
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += s_red[i];
    gwb_partial[(long long)v * T + t] = s;
  }
  // a slot the binning marked dead (zero weight at every pixel: every sum below would be +0)
  // writes its zero gradient row and leaves; slots are in ascending distance, so the dead ones
  // gather at the end of the list and whole warps of them skip the pixel loop
  const int k = tid;
  if (k >= n) return;
  const long long row0 = ((long long)v * T + t) * K;
  if (slots[(row0 + k) * TTS_SLOT_FLOATS + 10] != 0.f) {
    float2* out = reinterpret_cast<float2*>(slot_grads + (row0 + k) * TTS_SLOT_GRAD_FLOATS);
    const float2 z2 = make_float2(0.f, 0.f);
    out[0] = z2; out[1] = z2; out[2] = z2; out[3] = z2; out[4] = z2;
    return;
  }
  const long long o = row0 + k;
  const float4* row = reinterpret_cast<const float4*>(slots + o * TTS_SLOT_FLOATS);
  const float4 A = row[0], B = row[1], C = row[2];
  const f32x2 t0 = mk2(A.x, A.x);
  const float t1 = A.y, t2 = A.z, t3 = A.w, t4 = B.x, t5 = B.y;
  const f32x2 cr = mk2(B.z, B.z), cg = mk2(B.w, B.w), cbb = mk2(C.x, C.x), oc = mk2(C.y, C.y);
  const f32x2 z = mk2(0.f, 0.f);
  f32x2 gc0 = z, gc1 = z, gc2 = z, goc = z;
  float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f, g4 = 0.f, g5 = 0.f;
  for (int ly = 0; ly < 16; ++ly) {
    const float py = (float)ly + 0.5f;
    const float srow = fmaf(t2, py, t3);
    const float rrow = fmaf(fmaf(t1, py, t4), py, t5);
    const f32x2 s2 = mk2(srow, srow);
    f32x2 a0 = z, a1 = z, a2 = z;
#pragma unroll
    for (int lp = 0; lp < 8; ++lp) {
      const f32x2 px = mk2((float)(2 * lp) + 0.5f, (float)(2 * lp) + 1.5f);
      const f32x2 pxsq = mk2(((float)(2 * lp) + 0.5f) * ((float)(2 * lp) + 0.5f),
                             ((float)(2 * lp) + 1.5f) * ((float)(2 * lp) + 1.5f));   // exact
      const int pi = ly * 16 + 2 * lp;
      const f32x2 P0 = *reinterpret_cast<const f32x2*>(&s_g0[pi]);
      const f32x2 P1 = *reinterpret_cast<const f32x2*>(&s_g1[pi]);
      const f32x2 P2 = *reinterpret_cast<const f32x2*>(&s_g2[pi]);
      const f32x2 P3 = *reinterpret_cast<const f32x2*>(&s_gd[pi]);
      const f32x2 r = fma_sat2(fma2(t0, px, s2), px, rrow);
      const f32x2 w = mul2(r, r);
      gc0 = fma2(w, P0, gc0);
      gc1 = fma2(w, P1, gc1);
      gc2 = fma2(w, P2, gc2);
      goc = fma2(w, P3, goc);
      const f32x2 gw = fma2(P0, cr, fma2(P1, cg, fma2(P2, cbb, mul2(P3, oc))));
      const f32x2 gu = mul2(r, gw);
      a0 = add2(a0, gu);
      a1 = fma2(gu, px, a1);
      a2 = fma2(gu, pxsq, a2);
    }
    const float s0 = hsum2(a0), s1 = hsum2(a1), s2s = hsum2(a2);
    g0 += s2s;
    g1 = fmaf(py * py, s0, g1);
    g2 = fmaf(py, s1, g2);
    g3 += s1;
    g4 = fmaf(py, s0, g4);
    g5 += s0;
  }
  // rows are 40 B: 8-byte aligned, so store as float2
  float2* out = reinterpret_cast<float2*>(slot_grads + o * TTS_SLOT_GRAD_FLOATS);
  out[0] = make_float2(2.f * g0, 2.f * g1);
  out[1] = make_float2(2.f * g2, 2.f * g3);
  out[2] = make_float2(2.f * g4, 2.f * g5);
  out[3] = make_float2(hsum2(gc0), hsum2(gc1));
  out[4] = make_float2(hsum2(gc2), hsum2(goc));
}

// ---- arm RV: revealage compositing (spike/arms.py:70-83) -------------------------------------
// Per pixel, over the tile's slots with W = w * o_col (w = relu(u)^2):
//   den = sum W + eps,  Cavg = sum w color_o / den,  R = exp(sum log1p(-clamp(W, 0, 1 - 1e-4)))
//   C = Cavg (1 - R) + c_b R          (no w_b: the background enters through R alone)
// The forward writes den and aux = (Cavg, R) per pixel for the backward.
constexpr float RV_EPS = 1e-6f;
constexpr float RV_AMAX = 0.9999f;   // 1 - 1e-4 as the float32 clamp bound

__global__ void __launch_bounds__(RV_THREADS)
    k_render_fwd_rv(const float* __restrict__ slots, const int* __restrict__ count, int ntx, int T, int H, int W,
                    int K, const float* __restrict__ c_b, float* __restrict__ img, float* __restrict__ den_out,
                    float4* __restrict__ aux) {
  extern __shared__ __align__(128) float s_rows[];
  __shared__ __align__(8) uint64_t bar;
  const int t = blockIdx.x, v = blockIdx.y, tid = threadIdx.x;
  const int n = count[(long long)v * T + t];
  const long long row0 = ((long long)v * T + t) * K;
  if (tid == 0) mbar_init(&bar, 1);
  __syncthreads();
  if (n > 0) {
    if (tid == 0) {
      const uint32_t bytes = (uint32_t)n * TTS_SLOT_FLOATS * 4u;
      mbar_expect_tx(&bar, bytes);
      bulk_g2s(s_rows, slots + row0 * TTS_SLOT_FLOATS, bytes, &bar);
    }
    if (!mbar_wait_bounded(&bar, 0)) return;
  }
  const int ly = tid >> 2;
  const int lxa = 2 * (tid & 3), lxb = lxa + 8;
  const float py = (float)ly + 0.5f;
  const f32x2 pxa = mk2((float)lxa + 0.5f, (float)lxa + 1.5f);
  const f32x2 pxb = mk2((float)lxb + 0.5f, (float)lxb + 1.5f);
  const f32x2 z = mk2(0.f, 0.f);
  f32x2 a0 = z, a1 = z, a2 = z, a3 = z, b0 = z, b1 = z, b2 = z, b3 = z;
  float lg[4] = {0.f, 0.f, 0.f, 0.f};
  const float4* rows = reinterpret_cast<const float4*>(s_rows);
  for (int s = 0; s < n; ++s) {
    const float4 A = rows[3 * s + 0];
    const float4 B = rows[3 * s + 1];
    const float4 C = rows[3 * s + 2];
    const float srow = fmaf(A.z, py, A.w);
    const float rrow = fmaf(fmaf(A.y, py, B.x), py, B.y);
    const f32x2 t0 = mk2(A.x, A.x), s2 = mk2(srow, srow), r2 = mk2(rrow, rrow);
    const f32x2 cr = mk2(B.z, B.z), cg = mk2(B.w, B.w), cb = mk2(C.x, C.x), oc = mk2(C.y, C.y);
    const f32x2 ra = relu2(fma2(fma2(t0, pxa, s2), pxa, r2));
    const f32x2 rb = relu2(fma2(fma2(t0, pxb, s2), pxb, r2));
    const f32x2 wa = mul2(ra, ra), wbv = mul2(rb, rb);
    a0 = fma2(wa, cr, a0); a1 = fma2(wa, cg, a1); a2 = fma2(wa, cb, a2); a3 = fma2(wa, oc, a3);
    b0 = fma2(wbv, cr, b0); b1 = fma2(wbv, cg, b1); b2 = fma2(wbv, cb, b2); b3 = fma2(wbv, oc, b3);
    float W4[4];
    split2(mul2(wa, oc), W4[0], W4[1]);
    split2(mul2(wbv, oc), W4[2], W4[3]);
#pragma unroll
    for (int i = 0; i < 4; i++) lg[i] += log1pf(-fminf(fmaxf(W4[i], 0.f), RV_AMAX));
  }
  const int tx = t % ntx, ty = t / ntx;
  const int gy = ty * 16 + ly;
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  float n0[4], n1[4], n2[4], dd[4];
  split2(a0, n0[0], n0[1]); split2(b0, n0[2], n0[3]);
  split2(a1, n1[0], n1[1]); split2(b1, n1[2], n1[3]);
  split2(a2, n2[0], n2[1]); split2(b2, n2[2], n2[3]);
  split2(a3, dd[0], dd[1]); split2(b3, dd[2], dd[3]);
  const int lx[4] = {lxa, lxa + 1, lxb, lxb + 1};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const long long p = ((long long)v * H + gy) * W + tx * 16 + lx[i];
    const float d = dd[i] + RV_EPS;
    const float c0 = n0[i] / d, c1 = n1[i] / d, c2 = n2[i] / d;
    const float R = expf(lg[i]);
    img[3 * p + 0] = c0 * (1.f - R) + cb0 * R;
    img[3 * p + 1] = c1 * (1.f - R) + cb1 * R;
    img[3 * p + 2] = c2 * (1.f - R) + cb2 * R;
    den_out[p] = d;
    aux[p] = make_float4(c0, c1, c2, R);
  }
}

// Backward of the RV blend per (pixel, slot), with g = dL/dC of the pixel:
//   gnum = g (1 - R) / den,  gden = -(g . Cavg)(1 - R) / den,  gL = R g . (c_b - Cavg)
//   dL/dW = gden - gL / (1 - W) [W <= 1 - 1e-4]   (the clamp passes no gradient above its bound)
// and W = w o_col, so the per-slot sums are those of arm A with gden replaced by dL/dW.
__global__ void __launch_bounds__(256)
    k_render_bwd_rv(const float* __restrict__ slots, const int* __restrict__ count, int ntx, int T, int H, int W,
                    int K, const float* __restrict__ c_b, const float* __restrict__ den, const float4* __restrict__ aux,
                    const float* __restrict__ gimg, float* __restrict__ slot_grads, float* __restrict__ gwb_partial) {
  __shared__ __align__(16) float s_g0[256], s_g1[256], s_g2[256], s_gd[256], s_gl[256];
  const int t = blockIdx.x, v = blockIdx.y, tid = threadIdx.x;
  const int tx = t % ntx, ty = t / ntx;
  const int n = count[(long long)v * T + t];
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  for (int p = tid; p < 256; p += blockDim.x) {
    const long long q = ((long long)v * H + ty * 16 + (p >> 4)) * W + tx * 16 + (p & 15);
    const float g0 = gimg[3 * q], g1 = gimg[3 * q + 1], g2 = gimg[3 * q + 2];
    const float4 a = aux[q];
    const float f = (1.f - a.w) / den[q];
    s_g0[p] = g0 * f;
    s_g1[p] = g1 * f;
    s_g2[p] = g2 * f;
    s_gd[p] = -(g0 * a.x + g1 * a.y + g2 * a.z) * f;
    s_gl[p] = a.w * (g0 * (cb0 - a.x) + g1 * (cb1 - a.y) + g2 * (cb2 - a.z));
  }
  if (tid == 0) gwb_partial[(long long)v * T + t] = 0.f;   // w_b does not enter the RV blend
  __syncthreads();
  const int k = tid;
  if (k >= n) return;
  const long long o = ((long long)v * T + t) * K + k;
  const float4* row = reinterpret_cast<const float4*>(slots + o * TTS_SLOT_FLOATS);
  const float4 A = row[0], B = row[1], C = row[2];
  const f32x2 t0 = mk2(A.x, A.x);
  const float t1 = A.y, t2 = A.z, t3 = A.w, t4 = B.x, t5 = B.y;
  const f32x2 cr = mk2(B.z, B.z), cg = mk2(B.w, B.w), cbb = mk2(C.x, C.x), oc = mk2(C.y, C.y);
  const f32x2 z = mk2(0.f, 0.f);
  f32x2 gc0 = z, gc1 = z, gc2 = z, goc = z;
  float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f, g4 = 0.f, g5 = 0.f;
  for (int ly = 0; ly < 16; ++ly) {
    const float py = (float)ly + 0.5f;
    const float srow = fmaf(t2, py, t3);
    const float rrow = fmaf(fmaf(t1, py, t4), py, t5);
    const f32x2 s2 = mk2(srow, srow), r2 = mk2(rrow, rrow);
    f32x2 a0 = z, a1 = z, a2 = z;
#pragma unroll
    for (int lp = 0; lp < 8; ++lp) {
      const f32x2 px = mk2((float)(2 * lp) + 0.5f, (float)(2 * lp) + 1.5f);
      const f32x2 pxsq = mk2(((float)(2 * lp) + 0.5f) * ((float)(2 * lp) + 0.5f),
                             ((float)(2 * lp) + 1.5f) * ((float)(2 * lp) + 1.5f));   // exact
      const int pi = ly * 16 + 2 * lp;
      const f32x2 P0 = *reinterpret_cast<const f32x2*>(&s_g0[pi]);
      const f32x2 P1 = *reinterpret_cast<const f32x2*>(&s_g1[pi]);
      const f32x2 P2 = *reinterpret_cast<const f32x2*>(&s_g2[pi]);
      const f32x2 r = relu2(fma2(fma2(t0, px, s2), px, r2));
      const f32x2 w = mul2(r, r);
      float wl, wh, gdl, gdh;
      split2(mul2(w, oc), wl, wh);
      const float2 gd = *reinterpret_cast<const float2*>(&s_gd[pi]);
      const float2 gl = *reinterpret_cast<const float2*>(&s_gl[pi]);
      gdl = wl <= RV_AMAX ? gd.x - gl.x * __frcp_rn(1.f - fmaxf(wl, 0.f)) : gd.x;
      gdh = wh <= RV_AMAX ? gd.y - gl.y * __frcp_rn(1.f - fmaxf(wh, 0.f)) : gd.y;
      const f32x2 P3 = mk2(gdl, gdh);
      gc0 = fma2(w, P0, gc0);
      gc1 = fma2(w, P1, gc1);
      gc2 = fma2(w, P2, gc2);
      goc = fma2(w, P3, goc);
      const f32x2 gw = fma2(P0, cr, fma2(P1, cg, fma2(P2, cbb, mul2(P3, oc))));
      const f32x2 gu = mul2(r, gw);
      a0 = add2(a0, gu);
      a1 = fma2(gu, px, a1);
      a2 = fma2(gu, pxsq, a2);
    }
    const float s0 = hsum2(a0), s1 = hsum2(a1), s2s = hsum2(a2);
    g0 += s2s;
    g1 = fmaf(py * py, s0, g1);
    g2 = fmaf(py, s1, g2);
    g3 += s1;
    g4 = fmaf(py, s0, g4);
    g5 += s0;
  }
  float2* out = reinterpret_cast<float2*>(slot_grads + o * TTS_SLOT_GRAD_FLOATS);
  out[0] = make_float2(2.f * g0, 2.f * g1);
  out[1] = make_float2(2.f * g2, 2.f * g3);
  out[2] = make_float2(2.f * g4, 2.f * g5);
  out[3] = make_float2(hsum2(gc0), hsum2(gc1));
  out[4] = make_float2(hsum2(gc2), hsum2(goc));
}

// theta_u[VT,6,K], color_o[VT,K,3], o_col[VT,K,1] -> slot rows
__global__ void k_pack_operands(const float* __restrict__ th, const float* __restrict__ col, const float* __restrict__ oc,
                                int VT, int K, float* __restrict__ slots) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)VT * K) return;
  const long long t = i / K;
  const int k = (int)(i % K);
  float* r = slots + i * TTS_SLOT_FLOATS;
#pragma unroll
  for (int j = 0; j < 6; j++) r[j] = th[(t * 6 + j) * K + k];
#pragma unroll
  for (int c = 0; c < 3; c++) r[6 + c] = col[i * 3 + c];
  r[9] = oc[i];
  r[10] = 0.f;
  r[11] = 0.f;
}

__global__ void k_unpack_grads(const float* __restrict__ sg, int VT, int K, float* __restrict__ gth,
                               float* __restrict__ gcol, float* __restrict__ goc) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)VT * K) return;
  const long long t = i / K;
  const int k = (int)(i % K);
  const float* r = sg + i * TTS_SLOT_GRAD_FLOATS;
#pragma unroll
  for (int j = 0; j < 6; j++) gth[(t * 6 + j) * K + k] = r[j];
#pragma unroll
  for (int c = 0; c < 3; c++) gcol[i * 3 + c] = r[6 + c];
  goc[i] = r[9];
}

}  // namespace tts

using namespace tts;

extern "C" int tts_render_fwd(const void* slots, int slots_bf16, const int32_t* count, int V, int H, int W, int K,
                              const float* w_b, int w_b_is_raw, const float* c_b, float* img, float* den,
                              void* stream) {
  TTS_REQUIRE(V >= 1 && H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(K >= 1 && K <= KMAX, "K must be in [1, 256]");
  TTS_REQUIRE(slots && count && w_b && c_b && img && den, "null pointer");
  TTS_REQUIRE(aligned16(slots), "slots must be 16-byte aligned");
  const int ntx = W / 16, T = ntx * (H / 16);
  dim3 grid(T, V);
  cudaStream_t st = as_stream(stream);
  const size_t smem = (size_t)K * TTS_SLOT_FLOATS * sizeof(float);
  if (slots_bf16)
    k_render_fwd<true><<<grid, FWD_THREADS, smem, st>>>(slots, count, ntx, T, H, W, K, w_b, w_b_is_raw, c_b, img, den);
  else
    k_render_fwd<false><<<grid, FWD_THREADS, smem, st>>>(slots, count, ntx, T, H, W, K, w_b, w_b_is_raw, c_b, img, den);
  return check_launch("render_fwd");
}

extern "C" int tts_render_bwd(const float* slots, const int32_t* count, int V, int H, int W, int K, const float* c_b,
                              const float* img, const float* den, const float* gimg, float* slot_grads,
                              float* gwb_partial, void* stream) {
  TTS_REQUIRE(V >= 1 && H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(K >= 1 && K <= KMAX, "K must be in [1, 256]");
  TTS_REQUIRE(aligned16(slots) && ((uintptr_t)slot_grads & 7u) == 0, "slots must be 16-byte and slot_grads 8-byte aligned");
  const int ntx = W / 16, T = ntx * (H / 16);
  const int threads = ((K + 31) / 32) * 32;
  dim3 grid(T, V);
  k_render_bwd<<<grid, threads, 0, as_stream(stream)>>>(slots, count, ntx, T, H, W, K, c_b, img, den, gimg, slot_grads,
                                                         gwb_partial);
  return check_launch("render_bwd");
}

extern "C" int tts_render_fwd_rv(const float* slots, const int32_t* count, int V, int H, int W, int K,
                                 const float* c_b, float* img, float* den, float* aux, void* stream) {
  TTS_REQUIRE(V >= 1 && H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(K >= 1 && K <= KMAX, "K must be in [1, 256]");
  TTS_REQUIRE(slots && count && c_b && img && den && aux, "null pointer");
  TTS_REQUIRE(aligned16(slots) && aligned16(aux), "slots and aux must be 16-byte aligned");
  const int ntx = W / 16, T = ntx * (H / 16);
  const size_t smem = (size_t)K * TTS_SLOT_FLOATS * sizeof(float);
  k_render_fwd_rv<<<dim3(T, V), RV_THREADS, smem, as_stream(stream)>>>(slots, count, ntx, T, H, W, K, c_b, img, den,
                                                                       reinterpret_cast<float4*>(aux));
  return check_launch("render_fwd_rv");
}

extern "C" int tts_render_bwd_rv(const float* slots, const int32_t* count, int V, int H, int W, int K,
                                 const float* c_b, const float* den, const float* aux, const float* gimg,
                                 float* slot_grads, float* gwb_partial, void* stream) {
  TTS_REQUIRE(V >= 1 && H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(K >= 1 && K <= KMAX, "K must be in [1, 256]");
  TTS_REQUIRE(slots && count && c_b && den && aux && gimg && slot_grads && gwb_partial, "null pointer");
  TTS_REQUIRE(aligned16(slots) && aligned16(aux) && ((uintptr_t)slot_grads & 7u) == 0,
              "slots and aux must be 16-byte and slot_grads 8-byte aligned");
  const int ntx = W / 16, T = ntx * (H / 16);
  const int threads = ((K + 31) / 32) * 32;
  k_render_bwd_rv<<<dim3(T, V), threads, 0, as_stream(stream)>>>(slots, count, ntx, T, H, W, K, c_b, den,
                                                                  reinterpret_cast<const float4*>(aux), gimg,
                                                                  slot_grads, gwb_partial);
  return check_launch("render_bwd_rv");
}

extern "C" int tts_pack_operands(const float* theta_u, const float* color_o, const float* o_col, int VT, int K,
                                 float* slots, void* stream) {
  TTS_REQUIRE(VT >= 0 && K >= 1, "bad sizes");
  const long long n = (long long)VT * K;
  if (n == 0) return TTS_OK;
  k_pack_operands<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(theta_u, color_o, o_col, VT, K, slots);
  return check_launch("pack_operands");
}

extern "C" int tts_unpack_slot_grads(const float* slot_grads, int VT, int K, float* gtheta_u, float* gcolor_o,
                                     float* go_col, void* stream) {
  TTS_REQUIRE(VT >= 0 && K >= 1, "bad sizes");
  const long long n = (long long)VT * K;
  if (n == 0) return TTS_OK;
  k_unpack_grads<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(slot_grads, VT, K, gtheta_u, gcolor_o,
                                                                               go_col);
  return check_launch("unpack_slot_grads");
}
