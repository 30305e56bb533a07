// Thread-per-gaussian kernels: projection (geometry + SH colour + activations + home-cell
// count) and the parameter backward (slot->gaussian reduction + theta-build backward +
// geometry/SH/activation backward, summed over views).
#include "geom.cuh"

namespace tts {

__device__ int cell_coord_g(float m, int n) {
  const float v = floorf(__fdiv_rn(m, 16.0f));
  if (!(v >= 0.0f && v < 9.223372036854775808e18f)) return 0;
  return v >= (float)(n - 1) ? n - 1 : (int)v;
}

struct Loaded {
  float m[3], q[4], ls[3], op, dc[3];
};

__device__ __forceinline__ void load_params(const float* __restrict__ p, const ParamLayout& L, int g, Loaded& x) {
#pragma unroll
  for (int i = 0; i < 3; i++) {
    x.m[i] = p[L.means() + 3 * g + i];
    x.ls[i] = p[L.log_scales() + 3 * g + i];
    x.dc[i] = p[L.color_dc() + 3 * g + i];
  }
#pragma unroll
  for (int i = 0; i < 4; i++) x.q[i] = p[L.quats() + 4 * g + i];
  x.op = p[L.opacity() + g];
}

// SH colour pre-clamp value r + 0.5 per channel (spike/sh.py:55-72) or the DC colour
// 0.5 + C0*dc (spike/forward.py:69-71).
template <int DEG>
__device__ __forceinline__ void colour_pre(const float* __restrict__ p, const ParamLayout& L, int g, const Loaded& x,
                                           const float d[3], float pre[3]) {
  if (DEG == 0) {
#pragma unroll
    for (int c = 0; c < 3; c++) pre[c] = 0.5f + SH_C0 * x.dc[c];
    return;
  }
  float b[16];
  sh_basis(DEG, d[0], d[1], d[2], b);
  constexpr int NB = (DEG + 1) * (DEG + 1);
#pragma unroll
  for (int c = 0; c < 3; c++) {
    float r = b[0] * x.dc[c];
#pragma unroll
    for (int k = 1; k < NB; k++) r += b[k] * p[L.color_rest() + 45 * g + 3 * (k - 1) + c];
    pre[c] = r + 0.5f;
  }
}

template <int DEG>
__global__ void __launch_bounds__(128)
    k_project(const float* __restrict__ params, int G, const float* __restrict__ cams, int ntx, int nty, float blur,
              float near_plane, float* __restrict__ proj, float* __restrict__ mu2d, uint8_t* __restrict__ keep,
              int* __restrict__ cell_count, int2* __restrict__ cell_rank) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int v = blockIdx.y;
  const int T = ntx * nty;
  const ParamLayout L{G};
  int cell = -1;
  if (g < G) {
    const Cam cam = load_cam(cams, v);
    Loaded x;
    load_params(params, L, g, x);
    GeomFwd f;
    geom_forward(x.m, x.q, x.ls, cam, blur, near_plane, f);
    float d[3] = {0.f, 0.f, 0.f}, nrm;
    if (DEG > 0) view_dir(x.m, cam, d, nrm);
    float pre[3];
    colour_pre<DEG>(params, L, g, x, d, pre);
    const float o = sigmoidf(x.op);
    const float keo = f.keep ? o : 0.f;
    const long long o_ = (long long)v * G + g;
    float4* pr = reinterpret_cast<float4*>(proj + o_ * TTS_PROJ_FLOATS);
    pr[0] = make_float4(f.mux, f.muy, f.a, f.b);
    pr[1] = make_float4(f.c, keo * fmaxf(pre[0], 0.f), keo * fmaxf(pre[1], 0.f), keo * fmaxf(pre[2], 0.f));
    pr[2] = make_float4(keo, f.mcz, 0.f, 0.f);
    reinterpret_cast<float2*>(mu2d)[o_] = make_float2(f.mux, f.muy);
    keep[o_] = f.keep ? 1 : 0;
    if (f.keep) cell = cell_coord_g(f.muy, nty) * ntx + cell_coord_g(f.mux, ntx);
    else cell_rank[o_] = make_int2(-1, 0);
  }
  // warp-aggregated home-cell count (one atomic per distinct cell per warp)
  const unsigned mask = __ballot_sync(0xffffffffu, cell >= 0);
  if (cell >= 0) {
    const unsigned peers = __match_any_sync(mask, cell);
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(cell_count + (long long)v * T + cell, __popc(peers));
    base = __shfl_sync(peers, base, leader);
    cell_rank[(long long)v * G + g] = make_int2(cell, base + __popc(peers & ((1u << lane) - 1u)));
  }
}

// Per (gaussian, view): slot->gaussian gather over the stencil slots (ascending j,
// deterministic) with the theta-build backward (tools/operands_manual.py:65-80), geometry
// backward (tools/geom_bwd.py:67-152), activation backward (tools/operands_manual.py:103-110)
// and the view-direction part of the SH backward.  Writes 16 floats per (view, gaussian):
// gmeans[3], gquat[4], gscale[3], gopacity_raw, gcolour_pre[3] (the gradient reaching the
// SH sum, masked by the clamp), 0, 0.  The SH coefficient gradients need only gcolour_pre and
// the direction, so the per-view record stays small and the reduction recomputes the basis.
template <int DEG>
__global__ void __launch_bounds__(128)
    k_backward_view(const float* __restrict__ params, int G, const float* __restrict__ cams, int ntx, int nty, int S,
                    int K, float inv_k, float blur, float near_plane, const int* __restrict__ inv,
                    const float* __restrict__ slot_grads, float4* __restrict__ scratch) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int v = blockIdx.y;
  if (g >= G) return;
  const ParamLayout L{G};
  const int T = ntx * nty;
  float4* out = scratch + ((long long)v * G + g) * 4;
  const int* iv = inv + ((long long)v * G + g) * S;
  bool any = false;
  for (int j = 0; j < S; ++j) any |= iv[j] >= 0;
  if (!any) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    out[0] = z; out[1] = z; out[2] = z; out[3] = z;
    return;
  }
  Loaded x;
  load_params(params, L, g, x);
  const float o = sigmoidf(x.op);
  const Cam cam = load_cam(cams, v);
  GeomFwd f;
  geom_forward(x.m, x.q, x.ls, cam, blur, near_plane, f);
  float ga = 0.f, gb = 0.f, gc = 0.f, gmx = 0.f, gmy = 0.f, gcol[3] = {0.f, 0.f, 0.f}, goc = 0.f;
  for (int j = 0; j < S; ++j) {
    const int s = iv[j];
    if (s < 0) continue;
    const int t = s / K;
    const float mux = f.mux - (float)((t % ntx) * 16);
    const float muy = f.muy - (float)((t / ntx) * 16);
    // 40-byte rows are 8-byte aligned: read them as five float2
    const float2* sg = reinterpret_cast<const float2*>(slot_grads + ((long long)v * T * K + s) * TTS_SLOT_GRAD_FLOATS);
    const float2 a01 = sg[0], a23 = sg[1], a45 = sg[2], c01 = sg[3], c2o = sg[4];
    const float g0 = -a01.x * inv_k, g1 = -a01.y * inv_k, g2 = -a23.x * inv_k;
    const float g3 = -a23.y * inv_k, g4 = -a45.x * inv_k, g5 = -a45.y * inv_k;
    ga += g0 + g3 * (-2.f * mux) + g5 * mux * mux;
    gb += 2.f * g2 + g3 * (-2.f * muy) + g4 * (-2.f * mux) + g5 * (2.f * mux * muy);
    gc += g1 + g4 * (-2.f * muy) + g5 * muy * muy;
    gmx += g3 * (-2.f * f.a) + g4 * (-2.f * f.b) + g5 * (2.f * f.a * mux + 2.f * f.b * muy);
    gmy += g3 * (-2.f * f.b) + g4 * (-2.f * f.c) + g5 * (2.f * f.b * mux + 2.f * f.c * muy);
    gcol[0] += c01.x;
    gcol[1] += c01.y;
    gcol[2] += c2o.x;
    goc += c2o.y;
  }
  float gm[3] = {0.f, 0.f, 0.f}, gq[4] = {0.f, 0.f, 0.f, 0.f}, gs[3] = {0.f, 0.f, 0.f};
  geom_backward(f, cam, ga, gb, gc, gmx, gmy, gm, gq, gs);
  float d[3] = {0.f, 0.f, 0.f}, nrm = 1.f;
  if (DEG > 0) view_dir(x.m, cam, d, nrm);
  float pre[3];
  colour_pre<DEG>(params, L, g, x, d, pre);
  const float keepf = f.keep ? 1.f : 0.f;
  const float keo = keepf * o;
  const float gkeo = gcol[0] * fmaxf(pre[0], 0.f) + gcol[1] * fmaxf(pre[1], 0.f) + gcol[2] * fmaxf(pre[2], 0.f) + goc;
  const float gop = gkeo * keepf * o * (1.f - o);
  float gr[3];
#pragma unroll
  for (int c = 0; c < 3; c++) gr[c] = pre[c] >= 0.f ? gcol[c] * keo : 0.f;   // torch clamp passes at 0
  if (DEG > 0) {
    // direction gradient through the normalisation d = dirs / max(|dirs|, 1e-12)
    constexpr int NB = (DEG + 1) * (DEG + 1);
    float gd[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 1; k < NB; k++) {
      float dx, dy, dz;
      sh_basis_grad(k, d[0], d[1], d[2], dx, dy, dz);
      float w = 0.f;
#pragma unroll
      for (int c = 0; c < 3; c++) w += params[L.color_rest() + 45 * g + 3 * (k - 1) + c] * gr[c];
      gd[0] += w * dx;
      gd[1] += w * dy;
      gd[2] += w * dz;
    }
    if (nrm > 1e-12f) {
      const float dd = d[0] * gd[0] + d[1] * gd[1] + d[2] * gd[2];
#pragma unroll
      for (int i = 0; i < 3; i++) gm[i] += (gd[i] - d[i] * dd) / nrm;
    } else {
#pragma unroll
      for (int i = 0; i < 3; i++) gm[i] += gd[i] / 1e-12f;
    }
  }
  out[0] = make_float4(gm[0], gm[1], gm[2], gq[0]);
  out[1] = make_float4(gq[1], gq[2], gq[3], gs[0]);
  out[2] = make_float4(gs[1], gs[2], gop, gr[0]);
  out[3] = make_float4(gr[1], gr[2], 0.f, 0.f);
}

// Per gaussian: sum the per-view records in view order (deterministic), form the SH coefficient
// gradients basis_k(d_v) * gcolour_pre_v, add the reg_loss gradient (spike/mcmc.py:18-22) and
// write the parameter gradient.
template <int DEG>
__global__ void __launch_bounds__(128)
    k_backward_reduce(const float* __restrict__ params, int G, const float* __restrict__ cams, int V,
                      const float4* __restrict__ scratch, float lambda_o, float lambda_s, float* __restrict__ grads) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const ParamLayout L{G};
  constexpr int NB = (DEG + 1) * (DEG + 1);
  Loaded x;
  load_params(params, L, g, x);
  float gm[3] = {0.f, 0.f, 0.f}, gq[4] = {0.f, 0.f, 0.f, 0.f}, gs[3] = {0.f, 0.f, 0.f}, gop = 0.f;
  float gco[NB][3];
#pragma unroll
  for (int k = 0; k < NB; k++)
#pragma unroll
    for (int c = 0; c < 3; c++) gco[k][c] = 0.f;
  for (int v = 0; v < V; ++v) {
    const float4* r = scratch + ((long long)v * G + g) * 4;
    const float4 r0 = r[0], r1 = r[1], r2 = r[2], r3 = r[3];
    gm[0] += r0.x; gm[1] += r0.y; gm[2] += r0.z;
    gq[0] += r0.w; gq[1] += r1.x; gq[2] += r1.y; gq[3] += r1.z;
    gs[0] += r1.w; gs[1] += r2.x; gs[2] += r2.y;
    gop += r2.z;
    const float gr[3] = {r2.w, r3.x, r3.y};
    if (gr[0] == 0.f && gr[1] == 0.f && gr[2] == 0.f) continue;
    float d[3] = {0.f, 0.f, 0.f}, nrm;
    if (DEG > 0) {
      const Cam cam = load_cam(cams, v);
      view_dir(x.m, cam, d, nrm);
    }
    float b[16];
    sh_basis(DEG, d[0], d[1], d[2], b);
#pragma unroll
    for (int k = 0; k < NB; k++)
#pragma unroll
      for (int c = 0; c < 3; c++) gco[k][c] += b[k] * gr[c];
  }
  const float o = sigmoidf(x.op);
  gop += lambda_o / (float)G * o * (1.f - o);
#pragma unroll
  for (int i = 0; i < 3; i++) {
    const float s = expf(x.ls[i]);
    grads[L.means() + 3 * g + i] = gm[i];
    grads[L.log_scales() + 3 * g + i] = gs[i] * s + lambda_s / (3.f * (float)G) * s;
    grads[L.color_dc() + 3 * g + i] = gco[0][i];
  }
#pragma unroll
  for (int i = 0; i < 4; i++) grads[L.quats() + 4 * g + i] = gq[i];
  grads[L.opacity() + g] = gop;
  float* gr_rest = grads + L.color_rest() + 45 * g;
#pragma unroll
  for (int k = 1; k < 16; k++)
#pragma unroll
    for (int c = 0; c < 3; c++) gr_rest[3 * (k - 1) + c] = k < NB ? gco[k < NB ? k : 0][c] : 0.f;
}

// Deterministic sum of the per-tile w_b partials; grads[59G] = sum * softplus'(w_b_raw).
__global__ void __launch_bounds__(1024) k_wb_reduce(const float* __restrict__ part, int n, const float* __restrict__ params,
                                                     int G, float* __restrict__ grads) {
  __shared__ float red[1024];
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int i = threadIdx.x;
  for (; i + 3 * 1024 < n; i += 4 * 1024) {
    a0 += part[i];
    a1 += part[i + 1024];
    a2 += part[i + 2048];
    a3 += part[i + 3072];
  }
  for (; i < n; i += 1024) a0 += part[i];
  red[threadIdx.x] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  for (int s = blockDim.x >> 1; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const ParamLayout L{G};
    grads[L.w_b_raw()] = red[0] * softplus_grad(params[L.w_b_raw()]);
  }
}

}  // namespace tts

using namespace tts;

extern "C" int tts_project(const float* params, int G, int sh_degree, const float* cams, int V, int H, int W,
                           float blur, float near_plane, float* proj, float* mu2d, uint8_t* keep, int32_t* cell_count,
                           int32_t* cell_rank, void* stream) {
  TTS_REQUIRE(G >= 0 && V >= 1, "G must be >= 0 and V >= 1");
  TTS_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_degree must be in [0, 3]");
  TTS_REQUIRE(H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(aligned16(proj), "proj must be 16-byte aligned");
  if (G == 0) return TTS_OK;
  dim3 grid((G + 127) / 128, V);
  cudaStream_t st = as_stream(stream);
  const int ntx = W / 16, nty = H / 16;
  int2* cr = reinterpret_cast<int2*>(cell_rank);
  switch (sh_degree) {
    case 0: k_project<0><<<grid, 128, 0, st>>>(params, G, cams, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr); break;
    case 1: k_project<1><<<grid, 128, 0, st>>>(params, G, cams, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr); break;
    case 2: k_project<2><<<grid, 128, 0, st>>>(params, G, cams, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr); break;
    default: k_project<3><<<grid, 128, 0, st>>>(params, G, cams, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr); break;
  }
  return check_launch("project");
}

extern "C" size_t tts_backward_workspace_bytes(int G, int V) {
  return (G > 0 && V > 0) ? (size_t)V * G * 64 : 0;
}

extern "C" int tts_backward_params(const float* params, int G, int sh_degree, const float* cams, int V, int H, int W,
                                   int R, int K, float k_poly, float blur, float near_plane, const int32_t* inv,
                                   const float* slot_grads, const float* gwb_partial, float lambda_o, float lambda_s,
                                   float* grads, void* workspace, size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(G >= 1 && V >= 1, "G and V must be >= 1");
  TTS_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_degree must be in [0, 3]");
  TTS_REQUIRE(H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(R >= 0 && R <= 3 && K >= 1 && K <= 256, "R in [0,3] and K in [1,256]");
  TTS_REQUIRE(((uintptr_t)slot_grads & 7u) == 0, "slot_grads must be 8-byte aligned");
  TTS_REQUIRE(workspace && aligned16(workspace), "workspace must be a 16-byte aligned device buffer");
  if (workspace_bytes < tts_backward_workspace_bytes(G, V)) return fail(TTS_ERR_CAPACITY, "backward workspace too small");
  const int ntx = W / 16, nty = H / 16, S = (2 * R + 1) * (2 * R + 1);
  const float inv_k = (float)(1.0 / (double)k_poly);
  cudaStream_t st = as_stream(stream);
  float4* scr = static_cast<float4*>(workspace);
  dim3 gv((G + 127) / 128, V), g1((G + 127) / 128);
#define TTS_BWD(D)                                                                                               \
  k_backward_view<D><<<gv, 128, 0, st>>>(params, G, cams, ntx, nty, S, K, inv_k, blur, near_plane, inv, slot_grads, \
                                         scr);                                                                    \
  k_backward_reduce<D><<<g1, 128, 0, st>>>(params, G, cams, V, scr, lambda_o, lambda_s, grads);
  switch (sh_degree) {
    case 0: TTS_BWD(0) break;
    case 1: TTS_BWD(1) break;
    case 2: TTS_BWD(2) break;
    default: TTS_BWD(3) break;
  }
#undef TTS_BWD
  if (int rc = check_launch("backward_params")) return rc;
  k_wb_reduce<<<1, 1024, 0, st>>>(gwb_partial, V * ntx * nty, params, G, grads);
  return check_launch("wb_reduce");
}
