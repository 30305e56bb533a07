// Fused per-tile poly-splat + WSR forward and backward (one CTA per 16x16 tile per view).
//
// Forward (replaces _DevRenderBinned.forward, tools/m4_train_binned.py:156-166): the tile's
// slot rows (theta_u[6] | color_o[3] | o_col) are staged in shared memory by one bulk copy
// (cp.async.bulk, completion on an mbarrier); each thread owns RENDER_PPT pixels of one tile
// row and loops over the slots with the rows broadcast from shared memory:
//   u = theta . Phi(px, py) = (t0 px + (t2 py + t3)) px + ((t1 py + t4) py + t5)
//   w = max(u, 0)^2;  num += w color_o;  den += w o_col
// then C = (num + w_b c_b) / (den + w_b).  The [256 x K] weight matrix never leaves registers.
//
// Backward (replaces _DevRenderBinned.backward :169-186 / WSRPolySplatHot.backward,
// spike/backward.py:43-58): one thread per slot, looping over the tile's 256 pixels whose
// (gnum = gC/den, gden = -(gC.C)/den) are broadcast from shared memory; every per-slot sum
// (gcolor_o = w^T gnum, go_col = w^T gden, gtheta = Phi^T (2 relu(u) gw)) stays in the
// thread's registers, so no cross-thread reduction is needed.  gtheta is accumulated per row
// through the moments sum(gu), sum(gu px), sum(gu px^2).
#include "common.cuh"

namespace tts {

constexpr int RENDER_PPT = 2;                       // pixels per thread (same row, 8 apart)
constexpr int RENDER_THREADS = 256 / RENDER_PPT;    // 128
constexpr int KMAX = 256;

template <bool BF16>
__global__ void __launch_bounds__(RENDER_THREADS)
    k_render_fwd(const void* __restrict__ slots_, const int* __restrict__ count, int ntx, int T, int H, int W, int K,
                 const float* __restrict__ w_b_ptr, int w_b_is_raw, const float* __restrict__ c_b,
                 float* __restrict__ img, float* __restrict__ den_out) {
  __shared__ __align__(128) float s_rows[KMAX * TTS_SLOT_FLOATS];
  __shared__ __align__(8) uint64_t bar;
  const int t = blockIdx.x, v = blockIdx.y, tid = threadIdx.x;
  const int n = count[(long long)v * T + t];
  const long long row0 = ((long long)v * T + t) * K;
  bool ok = true;
  if (!BF16) {
    const float* src = static_cast<const float*>(slots_) + row0 * TTS_SLOT_FLOATS;
    if (tid == 0) {
      mbar_init(&bar, 1);
    }
    __syncthreads();
    if (n > 0) {
      if (tid == 0) {
        const uint32_t bytes = (uint32_t)n * TTS_SLOT_FLOATS * 4u;
        mbar_expect_tx(&bar, bytes);
        bulk_g2s(s_rows, src, bytes, &bar);
      }
      ok = mbar_wait_bounded(&bar, 0);
    }
  } else {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(slots_) + row0 * TTS_SLOT_FLOATS;
    for (int i = tid; i < n * TTS_SLOT_FLOATS; i += RENDER_THREADS) s_rows[i] = __bfloat162float(src[i]);
    __syncthreads();
  }
  if (!ok) return;   // status recorded; nothing of the tile is written

  const float wb = w_b_is_raw ? softplusf(*w_b_ptr) : *w_b_ptr;
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  const int ly = tid / (16 / RENDER_PPT);
  const int lx0 = tid % (16 / RENDER_PPT);
  const float py = (float)ly + 0.5f;
  float px[RENDER_PPT];
  float acc[RENDER_PPT][4];
#pragma unroll
  for (int i = 0; i < RENDER_PPT; i++) {
    px[i] = (float)(lx0 + i * (16 / RENDER_PPT)) + 0.5f;
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  }
  const float4* rows = reinterpret_cast<const float4*>(s_rows);
#pragma unroll 2
  for (int s = 0; s < n; ++s) {
    const float4 A = rows[3 * s + 0];   // t0 t1 t2 t3
    const float4 B = rows[3 * s + 1];   // t4 t5 cr cg
    const float4 C = rows[3 * s + 2];   // cb oc 0 0
    const float srow = fmaf(A.z, py, A.w);
    const float rrow = fmaf(fmaf(A.y, py, B.x), py, B.y);
#pragma unroll
    for (int i = 0; i < RENDER_PPT; i++) {
      const float u = fmaf(fmaf(A.x, px[i], srow), px[i], rrow);
      const float r = fmaxf(u, 0.f);
      const float w = r * r;
      acc[i][0] = fmaf(w, B.z, acc[i][0]);
      acc[i][1] = fmaf(w, B.w, acc[i][1]);
      acc[i][2] = fmaf(w, C.x, acc[i][2]);
      acc[i][3] = fmaf(w, C.y, acc[i][3]);
    }
  }
  const int tx = t % ntx, ty = t / ntx;
  const int gy = ty * 16 + ly;
#pragma unroll
  for (int i = 0; i < RENDER_PPT; i++) {
    const int gx = tx * 16 + lx0 + i * (16 / RENDER_PPT);
    const long long p = ((long long)v * H + gy) * W + gx;
    const float d = acc[i][3] + wb;
    img[3 * p + 0] = (acc[i][0] + wb * cb0) / d;
    img[3 * p + 1] = (acc[i][1] + wb * cb1) / d;
    img[3 * p + 2] = (acc[i][2] + wb * cb2) / d;
    den_out[p] = d;
  }
}

__global__ void __launch_bounds__(256)
    k_render_bwd(const float* __restrict__ slots, const int* __restrict__ count, int ntx, int T, int H, int W, int K,
                 const float* __restrict__ c_b, const float* __restrict__ img, const float* __restrict__ den,
                 const float* __restrict__ gimg, float* __restrict__ slot_grads, float* __restrict__ gwb_partial) {
  __shared__ __align__(16) float4 s_pix[256];
  __shared__ float s_red[32];
  const int t = blockIdx.x, v = blockIdx.y, tid = threadIdx.x;
  const int tx = t % ntx, ty = t / ntx;
  const int n = count[(long long)v * T + t];
  const float cb0 = c_b[0], cb1 = c_b[1], cb2 = c_b[2];
  // per-pixel upstream terms (tools/m4_train_binned.py:178-179, spike/backward.py:46-48)
  float wbp = 0.f;
  for (int p = tid; p < 256; p += blockDim.x) {
    const long long q = ((long long)v * H + ty * 16 + (p >> 4)) * W + tx * 16 + (p & 15);
    const float g0 = gimg[3 * q], g1 = gimg[3 * q + 1], g2 = gimg[3 * q + 2];
    const float c0 = img[3 * q], c1 = img[3 * q + 1], c2 = img[3 * q + 2];
    const float d = den[q];
    const float gn0 = g0 / d, gn1 = g1 / d, gn2 = g2 / d;
    const float gd = -(g0 * c0 + g1 * c1 + g2 * c2) / d;
    s_pix[p] = make_float4(gn0, gn1, gn2, gd);
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
  const int k = tid;
  if (k >= n) return;
  const long long o = ((long long)v * T + t) * K + k;
  const float4* row = reinterpret_cast<const float4*>(slots + o * TTS_SLOT_FLOATS);
  const float4 A = row[0], B = row[1], C = row[2];
  const float t0 = A.x, t1 = A.y, t2 = A.z, t3 = A.w, t4 = B.x, t5 = B.y;
  const float cr = B.z, cg = B.w, cbb = C.x, oc = C.y;
  float gc0 = 0.f, gc1 = 0.f, gc2 = 0.f, goc = 0.f;
  float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f, g4 = 0.f, g5 = 0.f;
  for (int ly = 0; ly < 16; ++ly) {
    const float py = (float)ly + 0.5f;
    const float srow = fmaf(t2, py, t3);
    const float rrow = fmaf(fmaf(t1, py, t4), py, t5);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int lx = 0; lx < 16; ++lx) {
      const float px = (float)lx + 0.5f;
      const float4 P = s_pix[ly * 16 + lx];
      const float u = fmaf(fmaf(t0, px, srow), px, rrow);
      const float r = fmaxf(u, 0.f);
      const float w = r * r;
      gc0 = fmaf(w, P.x, gc0);
      gc1 = fmaf(w, P.y, gc1);
      gc2 = fmaf(w, P.z, gc2);
      goc = fmaf(w, P.w, goc);
      const float gw = fmaf(P.x, cr, fmaf(P.y, cg, fmaf(P.z, cbb, P.w * oc)));
      const float gu = r * gw;
      a0 += gu;
      const float tpx = gu * px;
      a1 += tpx;
      a2 = fmaf(tpx, px, a2);
    }
    g0 += a2;
    g1 = fmaf(py * py, a0, g1);
    g2 = fmaf(py, a1, g2);
    g3 += a1;
    g4 = fmaf(py, a0, g4);
    g5 += a0;
  }
  // rows are 40 B: 8-byte aligned, so store as float2
  float2* out = reinterpret_cast<float2*>(slot_grads + o * TTS_SLOT_GRAD_FLOATS);
  out[0] = make_float2(2.f * g0, 2.f * g1);
  out[1] = make_float2(2.f * g2, 2.f * g3);
  out[2] = make_float2(2.f * g4, 2.f * g5);
  out[3] = make_float2(gc0, gc1);
  out[4] = make_float2(gc2, goc);
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
  if (slots_bf16)
    k_render_fwd<true><<<grid, RENDER_THREADS, 0, st>>>(slots, count, ntx, T, H, W, K, w_b, w_b_is_raw, c_b, img, den);
  else
    k_render_fwd<false><<<grid, RENDER_THREADS, 0, st>>>(slots, count, ntx, T, H, W, K, w_b, w_b_is_raw, c_b, img, den);
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
