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

// ---- lanes-per-gaussian layout ---------------------------------------------------------------
// A block of 128 threads covers GPB = 128 / LPG gaussians with LPG consecutive lanes each; lane
// vl of a gaussian handles the views vl, vl + LPG, ...  The block's parameters (59 floats per
// gaussian) are staged once in shared memory with coalesced loads, so a gaussian's parameters
// are read from memory once for all views.
constexpr int GB_THREADS = 128;
constexpr int PSTRIDE = 59;   // odd row stride: lanes of different gaussians hit different banks

template <int GPB>
__device__ __forceinline__ void stage_params(const float* __restrict__ params, int G, int g0, float* s_p) {
  const ParamLayout L{G};
  const int ng = min(GPB, G - g0);
  const int offs[6] = {L.means(), L.log_scales(), L.quats(), L.opacity(), L.color_dc(), L.color_rest()};
  const int width[6] = {3, 3, 4, 1, 3, 45};
  const int col[6] = {0, 3, 6, 10, 11, 14};
#pragma unroll
  for (int f = 0; f < 6; ++f) {
    const int w = width[f], n = ng * w;
    const float* src = params + offs[f] + (long long)g0 * w;
    for (int i = threadIdx.x; i < n; i += GB_THREADS) {
      const int gg = i / w, c = i - gg * w;
      s_p[gg * PSTRIDE + col[f] + c] = __ldg(src + i);
    }
  }
}

// The inverse of stage_params: staged rows -> the flat layout, coalesced per field.
template <int GPB>
__device__ __forceinline__ void unstage_rows(const float* s_p, int G, int g0, float* __restrict__ dst) {
  const ParamLayout L{G};
  const int ng = min(GPB, G - g0);
  const int offs[6] = {L.means(), L.log_scales(), L.quats(), L.opacity(), L.color_dc(), L.color_rest()};
  const int width[6] = {3, 3, 4, 1, 3, 45};
  const int col[6] = {0, 3, 6, 10, 11, 14};
#pragma unroll
  for (int f = 0; f < 6; ++f) {
    const int w = width[f], n = ng * w;
    float* out = dst + offs[f] + (long long)g0 * w;
    for (int i = threadIdx.x; i < n; i += GB_THREADS) {
      const int gg = i / w, c = i - gg * w;
      out[i] = s_p[gg * PSTRIDE + col[f] + c];
    }
  }
}

// The cameras of the first CAM_STAGED views are staged in shared memory with the parameters
// (one coalesced load per block instead of a dependent camera read per lane after the staging
// barrier); later views read theirs from global memory.
constexpr int CAM_STAGED = 16;
__device__ __forceinline__ void stage_cams(const float* __restrict__ cams, int V, float* s_cam) {
  const int n = min(V, CAM_STAGED) * TTS_CAM_FLOATS;
  for (int i = threadIdx.x; i < n; i += GB_THREADS) s_cam[i] = __ldg(cams + i);
}
__device__ __forceinline__ Cam cam_at(const float* __restrict__ cams, const float* s_cam, int v) {
  if (v >= CAM_STAGED) return load_cam(cams, v);
  const float* p = s_cam + v * TTS_CAM_FLOATS;
  Cam c;
#pragma unroll
  for (int i = 0; i < 9; i++) c.R[i] = p[i];
#pragma unroll
  for (int i = 0; i < 3; i++) c.t[i] = p[9 + i];
  c.fx = p[12]; c.fy = p[13]; c.cx = p[14]; c.cy = p[15];
#pragma unroll
  for (int i = 0; i < 3; i++) c.c[i] = p[16 + i];
  return c;
}

__device__ __forceinline__ void load_staged(const float* s, Loaded& x) {
#pragma unroll
  for (int i = 0; i < 3; i++) {
    x.m[i] = s[i];
    x.ls[i] = s[3 + i];
    x.dc[i] = s[11 + i];
  }
#pragma unroll
  for (int i = 0; i < 4; i++) x.q[i] = s[6 + i];
  x.op = s[10];
}

// SH colour pre-clamp value r + 0.5 per channel (spike/sh.py:55-72) or the DC colour
// 0.5 + C0*dc (spike/forward.py:69-71); rest coefficients from the staged row.
template <int DEG>
__device__ __forceinline__ void colour_pre(const float* s, const Loaded& x, const float d[3], float pre[3]) {
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
    for (int k = 1; k < NB; k++) r += b[k] * s[14 + 3 * (k - 1) + c];
    pre[c] = r + 0.5f;
  }
}

// Arm B (spike/arms.py:34-37) scales the opacity by the depth weight
// rho = sigmoid(depth_beta * (depth_tau - z)) of the camera-space z (spike/geometry.py:43).
__device__ __forceinline__ float depth_weight(const float* bt, float z) { return sigmoidf(bt[0] * (bt[1] - z)); }

template <int DEG, int LPG, bool ARMB>
__global__ void __launch_bounds__(GB_THREADS, 6)
    k_project(const float* __restrict__ params, int G, const float* __restrict__ cams, int V, int ntx, int nty,
              float blur, float near_plane, float* __restrict__ proj, float* __restrict__ mu2d,
              uint8_t* __restrict__ keep, int* __restrict__ cell_count, int2* __restrict__ cell_rank,
              const float* __restrict__ depth_bt) {
  constexpr int GPB = GB_THREADS / LPG;
  __shared__ float s_p[GPB * PSTRIDE];
  __shared__ float s_cam[CAM_STAGED * TTS_CAM_FLOATS];
  const int g0 = blockIdx.x * GPB;
  const int gl = threadIdx.x / LPG, vl = threadIdx.x % LPG;
  const int g = g0 + gl;
  stage_cams(cams, V, s_cam);
  stage_params<GPB>(params, G, g0, s_p);
  __syncthreads();
  const int T = ntx * nty;
  const float* sp = s_p + gl * PSTRIDE;
  Loaded x;
  if (g < G) load_staged(sp, x);
  const float o = g < G ? sigmoidf(x.op) : 0.f;
  const int nit = (V + LPG - 1) / LPG;     // uniform trip count: the warp-wide cell count below
  for (int it = 0; it < nit; ++it) {
    const int v = vl + it * LPG;
    int key = -1;                          // v * T + home cell of a kept (gaussian, view)
    if (g < G && v < V) {
      const Cam cam = cam_at(cams, s_cam, v);
      GeomFwd f;
      geom_forward(x.m, x.q, x.ls, cam, blur, near_plane, f);
      float d[3] = {0.f, 0.f, 0.f}, nrm;
      if (DEG > 0) view_dir(x.m, cam, d, nrm);
      float pre[3];
      colour_pre<DEG>(sp, x, d, pre);
      const float keo = f.keep ? (ARMB ? o * depth_weight(depth_bt, f.mcz) : o) : 0.f;
      const long long o_ = (long long)v * G + g;
      float4* pr = reinterpret_cast<float4*>(proj + o_ * TTS_PROJ_FLOATS);
      pr[0] = make_float4(f.mux, f.muy, f.a, f.b);
      pr[1] = make_float4(f.c, keo * fmaxf(pre[0], 0.f), keo * fmaxf(pre[1], 0.f), keo * fmaxf(pre[2], 0.f));
      pr[2] = make_float4(keo, f.mcz, 0.f, 0.f);
      reinterpret_cast<float2*>(mu2d)[o_] = make_float2(f.mux, f.muy);
      keep[o_] = f.keep ? 1 : 0;
      if (f.keep) key = v * T + cell_coord_g(f.muy, nty) * ntx + cell_coord_g(f.mux, ntx);
      else cell_rank[o_] = make_int2(-1, 0);
    }
    // warp-aggregated home-cell count (one atomic per distinct (view, cell) per warp)
    const unsigned mask = __ballot_sync(0xffffffffu, key >= 0);
    if (key >= 0) {
      const unsigned peers = __match_any_sync(mask, key);
      const int lane = threadIdx.x & 31;
      const int leader = __ffs(peers) - 1;
      int base = 0;
      if (lane == leader) base = atomicAdd(cell_count + key, __popc(peers));
      base = __shfl_sync(peers, base, leader);
      cell_rank[(long long)v * G + g] = make_int2(key - v * T, base + __popc(peers & ((1u << lane) - 1u)));
    }
  }
}

// Sum over the LPG lanes of one gaussian (xor butterfly: every lane ends with the same bits).
template <int LPG>
__device__ __forceinline__ float lane_sum(float a) {
#pragma unroll
  for (int o = 1; o < LPG; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  return a;
}

// Slot->gaussian gather, one thread per (view, gaussian): the gaussian's (<= (2R+1)^2) slot
// gradients are summed in ascending stencil order (deterministic; build_inv/gather_reduce of
// tools/m9_scatter_oracle.py:20-42) through the theta-build backward (_theta_bwd,
// tools/operands_manual.py:65-80) into a 12-float record (ga, gb, gc, gmx | gmy, gcolour_o[3] |
// go_col, valid, 0, 0).  A slim kernel: many warps in flight to cover the random row reads.
__global__ void __launch_bounds__(256)
    k_slot_gather(const float* __restrict__ proj, int G, int V, int ntx, int T, int S, int K, float inv_k,
                  const int* __restrict__ inv, const float* __restrict__ slot_grads, float4* __restrict__ rec) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)V * G) return;
  const int v = (int)(i / G);
  const int* iv = inv + i * S;
  // the first nine stencil slots (all of them for R <= 1) are fetched together
  int sl[9];
  bool any = false;
#pragma unroll
  for (int j = 0; j < 9; ++j) {
    sl[j] = j < S ? __ldg(iv + j) : -1;
    any |= sl[j] >= 0;
  }
  if (S > 9)
    for (int j = 9; j < S; ++j) any |= __ldg(iv + j) >= 0;
  float4* out = rec + i * 3;
  if (!any) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    out[0] = z; out[1] = z; out[2] = z;
    return;
  }
  const float4 p0 = __ldg(reinterpret_cast<const float4*>(proj + i * TTS_PROJ_FLOATS));
  const float pc = __ldg(proj + i * TTS_PROJ_FLOATS + 4);
  const float fmux = p0.x, fmuy = p0.y, fa = p0.z, fb = p0.w, fc = pc;
  float ga = 0.f, gb = 0.f, gc = 0.f, gmx = 0.f, gmy = 0.f, gcol0 = 0.f, gcol1 = 0.f, gcol2 = 0.f, goc = 0.f;
  const float* vsg = slot_grads + (long long)v * T * K * TTS_SLOT_GRAD_FLOATS;
  auto gather = [&](int s) {
    const int t = s / K;
    const float mux = fmux - (float)((t % ntx) * 16);
    const float muy = fmuy - (float)((t / ntx) * 16);
    // 40-byte rows are 8-byte aligned: read them as five float2
    const float2* sg = reinterpret_cast<const float2*>(vsg + (long long)s * TTS_SLOT_GRAD_FLOATS);
    const float2 a01 = __ldg(sg), a23 = __ldg(sg + 1), a45 = __ldg(sg + 2), c01 = __ldg(sg + 3), c2o = __ldg(sg + 4);
    const float g0 = -a01.x * inv_k, g1 = -a01.y * inv_k, g2 = -a23.x * inv_k;
    const float g3 = -a23.y * inv_k, g4 = -a45.x * inv_k, g5 = -a45.y * inv_k;
    ga += g0 + g3 * (-2.f * mux) + g5 * mux * mux;
    gb += 2.f * g2 + g3 * (-2.f * muy) + g4 * (-2.f * mux) + g5 * (2.f * mux * muy);
    gc += g1 + g4 * (-2.f * muy) + g5 * muy * muy;
    gmx += g3 * (-2.f * fa) + g4 * (-2.f * fb) + g5 * (2.f * fa * mux + 2.f * fb * muy);
    gmy += g3 * (-2.f * fb) + g4 * (-2.f * fc) + g5 * (2.f * fb * mux + 2.f * fc * muy);
    gcol0 += c01.x;
    gcol1 += c01.y;
    gcol2 += c2o.x;
    goc += c2o.y;
  };
#pragma unroll
  for (int j = 0; j < 9; ++j)
    if (sl[j] >= 0) gather(sl[j]);
  for (int j = 9; j < S; ++j) {
    const int s = __ldg(iv + j);
    if (s >= 0) gather(s);
  }
  out[0] = make_float4(ga, gb, gc, gmx);
  out[1] = make_float4(gmy, gcol0, gcol1, gcol2);
  out[2] = make_float4(goc, 1.f, 0.f, 0.f);
}

// Parameter backward, one gaussian per LPG lanes, each lane over its views: from the gathered
// record, the geometry backward (tools/geom_bwd.py:67-152), activation backward
// (tools/operands_manual.py:103-110) and SH backward (coefficients and viewing direction); the
// lanes' geometry sums are combined by a butterfly, the colour-coefficient sums through a
// per-round shared-memory exchange of each view's SH basis and colour gradient (each lane sums
// the entries it writes), then the reg_loss gradient (spike/mcmc.py:18-22) is added and the
// gaussian's 59 gradients are written.
// Four blocks per SM (128 registers) when a gaussian has 4 or 8 lanes: the colour-coefficient
// sums live in shared memory, not in 48 registers per lane.  One or two lanes keep three blocks
// at SH degree 2 and 3 (four would spill 100-500 B per thread); degrees 0 and 1 fit four blocks
// without spills at any lane count (one view at 1M gaussians, SH 0: 0.318 -> 0.276 ms).
template <int DEG, int LPG, bool ARMB>
__global__ void __launch_bounds__(GB_THREADS, (LPG >= 4 || DEG <= 1) ? 4 : 3)
    k_backward(const float* __restrict__ params, int G, const float* __restrict__ cams, int V, float blur,
               float near_plane, const float4* __restrict__ rec, float lambda_o, float lambda_s,
               float* __restrict__ grads, const float* __restrict__ depth_bt, float2* __restrict__ bt_partial) {
  constexpr int GPB = GB_THREADS / LPG;
  constexpr int NB = (DEG + 1) * (DEG + 1);
  __shared__ float s_p[GPB * PSTRIDE];
  __shared__ float s_cam[CAM_STAGED * TTS_CAM_FLOATS];
  const int g0 = blockIdx.x * GPB;
  const int gl = threadIdx.x / LPG, vl = threadIdx.x % LPG;
  const int g = g0 + gl;
  // the first view's gathered record is requested before the parameter staging, so that its
  // latency overlaps it
  float4 r0 = make_float4(0.f, 0.f, 0.f, 0.f), r1 = r0, r2 = r0;
  if (g < G && vl < V) {
    const float4* r = rec + ((long long)vl * G + g) * 3;
    r0 = __ldg(r);
    r1 = __ldg(r + 1);
    r2 = __ldg(r + 2);
  }
  stage_cams(cams, V, s_cam);
  stage_params<GPB>(params, G, g0, s_p);
  __syncthreads();
  const ParamLayout L{G};
  const float* sp = s_p + gl * PSTRIDE;
  Loaded x;
  if (g < G) load_staged(sp, x);
  const float o = g < G ? sigmoidf(x.op) : 0.f;
  float gm[3] = {0.f, 0.f, 0.f}, gq[4] = {0.f, 0.f, 0.f, 0.f}, gs[3] = {0.f, 0.f, 0.f}, gop = 0.f;
  float2 gbt = make_float2(0.f, 0.f);       // arm B: d/d depth_beta, d/d depth_tau of this thread
  // colour-coefficient gradients: lane vl owns the entries e = 11 + 3k + c with e % LPG == vl (the
  // ones it writes out) and sums them over the views, in view order, from the per-view SH basis b
  // and colour gradient gr that every lane publishes in shared memory each round
  constexpr int NX = NB + 3, NOWN = (3 * NB + LPG - 1) / LPG;
  __shared__ float s_x[GPB * LPG * NX];
  float* xs = s_x + gl * LPG * NX;
  const int e0 = 11 + ((vl - 11) % LPG + LPG) % LPG;
  float gco[NOWN];
#pragma unroll
  for (int i = 0; i < NOWN; i++) gco[i] = 0.f;
  const int nr = (V + LPG - 1) / LPG;       // the same in every lane: the rounds are warp-uniform
  for (int rd = 0; rd < nr; ++rd) {
    const int v = rd * LPG + vl;
    float bx[NB], grx[3] = {0.f, 0.f, 0.f};  // zero: no contribution of this lane in this round
#pragma unroll
    for (int k = 0; k < NB; k++) bx[k] = 0.f;
    if (g < G && v < V) {
      if (rd > 0) {
        const float4* r = rec + ((long long)v * G + g) * 3;
        r0 = __ldg(r);
        r1 = __ldg(r + 1);
        r2 = __ldg(r + 2);
      }
      if (r2.y != 0.f) {               // else no valid slot in this view
        const float ga = r0.x, gb = r0.y, gc = r0.z, gmx = r0.w, gmy = r1.x;
        const float gcol[3] = {r1.y, r1.z, r1.w};
        const float goc = r2.x;
        const Cam cam = cam_at(cams, s_cam, v);
        GeomFwd f;
        geom_forward(x.m, x.q, x.ls, cam, blur, near_plane, f);
        geom_backward(f, cam, ga, gb, gc, gmx, gmy, gm, gq, gs);
        float d[3] = {0.f, 0.f, 0.f}, nrm = 1.f;
        if (DEG > 0) view_dir(x.m, cam, d, nrm);
        float pre[3];
        colour_pre<DEG>(sp, x, d, pre);
        const float keepf = f.keep ? 1.f : 0.f;
        const float rho = ARMB ? depth_weight(depth_bt, f.mcz) : 1.f;
        const float keo = keepf * o * rho;
        const float gkeo =
            gcol[0] * fmaxf(pre[0], 0.f) + gcol[1] * fmaxf(pre[1], 0.f) + gcol[2] * fmaxf(pre[2], 0.f) + goc;
        gop += gkeo * keepf * rho * o * (1.f - o);
        if (ARMB) {
          // keo = keep o rho, rho = sigmoid(beta (tau - z)): d rho = rho (1 - rho) (beta, tau - z, -beta)
          const float grho = gkeo * keepf * o * rho * (1.f - rho);
          gbt.x += grho * (depth_bt[1] - f.mcz);
          gbt.y += grho * depth_bt[0];
          const float gz = -grho * depth_bt[0];            // z = R_v[2] . means + t_v[2]
  #pragma unroll
          for (int i = 0; i < 3; i++) gm[i] += gz * cam.R[2 * 3 + i];
        }
        float gr[3];
  #pragma unroll
        for (int c = 0; c < 3; c++) gr[c] = pre[c] >= 0.f ? gcol[c] * keo : 0.f;   // torch clamp passes at 0
        float b[16];
        sh_basis(DEG, d[0], d[1], d[2], b);
  #pragma unroll
        for (int k = 0; k < NB; k++) bx[k] = b[k];
  #pragma unroll
        for (int c = 0; c < 3; c++) grx[c] = gr[c];
        if (DEG > 0) {
          // direction gradient through the normalisation d = dirs / max(|dirs|, 1e-12)
          float gd[3] = {0.f, 0.f, 0.f};
  #pragma unroll
          for (int k = 1; k < NB; k++) {
            float dx, dy, dz;
            sh_basis_grad(k, d[0], d[1], d[2], dx, dy, dz);
            float w = 0.f;
  #pragma unroll
            for (int c = 0; c < 3; c++) w += sp[14 + 3 * (k - 1) + c] * gr[c];
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
      }
    }
    float* mine = xs + vl * NX;
#pragma unroll
    for (int k = 0; k < NB; k++) mine[k] = bx[k];
#pragma unroll
    for (int c = 0; c < 3; c++) mine[NB + c] = grx[c];
    __syncwarp();
#pragma unroll
    for (int i = 0; i < NOWN; i++) {
      const int e = e0 + i * LPG;
      if (e < 11 + 3 * NB) {
        const int kk = (e - 11) / 3, c = (e - 11) % 3;
#pragma unroll
        for (int l = 0; l < LPG; l++) gco[i] += xs[l * NX + kk] * xs[l * NX + NB + c];
      }
    }
    __syncwarp();                        // the next round overwrites the exchange
  }
  // combine the lanes (all lanes of the warp take part: the shuffles are warp-wide)
#pragma unroll
  for (int i = 0; i < 3; i++) {
    gm[i] = lane_sum<LPG>(gm[i]);
    gs[i] = lane_sum<LPG>(gs[i]);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) gq[i] = lane_sum<LPG>(gq[i]);
  gop = lane_sum<LPG>(gop);
  // the gaussian's 59 gradients go to its staged row (lane vl fills the entries e with
  // e % LPG == vl), then the block writes the rows out field by field, coalesced
  __syncthreads();                 // every lane is done reading its staged parameters
  float* row = s_p + gl * PSTRIDE;
  auto put = [&](int e, float val) {
    if (g < G && e % LPG == vl) row[e] = val;
  };
#pragma unroll
  for (int i = 0; i < 3; i++) {
    const float s = expf(x.ls[i]);
    put(i, gm[i]);
    put(3 + i, gs[i] * s + lambda_s / (3.f * (float)G) * s);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) put(6 + i, gq[i]);
  put(10, gop + lambda_o / (float)G * o * (1.f - o));
#pragma unroll
  for (int i = 0; i < NOWN; i++) {
    const int e = e0 + i * LPG;
    if (e < 11 + 3 * NB) put(e, gco[i]);
  }
  for (int e = 11 + 3 * NB; e < 59; e++) put(e, 0.f);   // SH coefficients above the degree
  __syncthreads();
  unstage_rows<GPB>(s_p, G, g0, grads);
  if (ARMB) {
    // this block's (d beta, d tau): warp sums, then the warps in order (deterministic)
    __shared__ float2 s_bt[GB_THREADS / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gbt.x += __shfl_xor_sync(0xffffffffu, gbt.x, o);
      gbt.y += __shfl_xor_sync(0xffffffffu, gbt.y, o);
    }
    if ((threadIdx.x & 31) == 0) s_bt[threadIdx.x >> 5] = gbt;
    __syncthreads();
    if (threadIdx.x == 0) {
      float2 t = s_bt[0];
      for (int w = 1; w < GB_THREADS / 32; ++w) {
        t.x += s_bt[w].x;
        t.y += s_bt[w].y;
      }
      bt_partial[blockIdx.x] = t;
    }
  }
}

// Deterministic sum of the per-tile w_b partials; grads[59G] = sum * softplus'(w_b_raw).
__global__ void __launch_bounds__(1024) k_wb_reduce(const float* __restrict__ part, int n, const float* __restrict__ params,
                                                     int G, float* __restrict__ grads, const float2* __restrict__ bt_part,
                                                     int nbt, float* __restrict__ g_depth_bt) {
  __shared__ float red[32];
  if (bt_part && threadIdx.x == 0) {
    // arm B: the blocks' (d beta, d tau) in block order
    float2 t = make_float2(0.f, 0.f);
    for (int b = 0; b < nbt; ++b) {
      t.x += bt_part[b].x;
      t.y += bt_part[b].y;
    }
    g_depth_bt[0] = t.x;
    g_depth_bt[1] = t.y;
  }
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  int i = threadIdx.x;
  for (; i + 3 * 1024 < n; i += 4 * 1024) {
    a0 += part[i];
    a1 += part[i + 1024];
    a2 += part[i + 2048];
    a3 += part[i + 3072];
  }
  for (; i < n; i += 1024) a0 += part[i];
  // fixed order: each warp's xor butterfly, then the 32 warp sums in warp order
  float r = (a0 + a1) + (a2 + a3);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    const ParamLayout L{G};
    grads[L.w_b_raw()] = t * softplus_grad(params[L.w_b_raw()]);
  }
}


static int lanes_for(int V) { return V >= 8 ? 8 : V >= 4 ? 4 : V >= 2 ? 2 : 1; }

template <int DEG, int LPG>
static void launch_project(const float* params, int G, const float* cams, int V, int ntx, int nty, float blur,
                           float near_plane, float* proj, float* mu2d, uint8_t* keep, int* cc, int2* cr,
                           const float* depth_bt, cudaStream_t st) {
  constexpr int GPB = GB_THREADS / LPG;
  const unsigned nb = (G + GPB - 1) / GPB;
  if (depth_bt)
    k_project<DEG, LPG, true><<<nb, GB_THREADS, 0, st>>>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d,
                                                         keep, cc, cr, depth_bt);
  else
    k_project<DEG, LPG, false><<<nb, GB_THREADS, 0, st>>>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d,
                                                          keep, cc, cr, nullptr);
}

template <int DEG>
static void project_deg(int lpg, const float* params, int G, const float* cams, int V, int ntx, int nty, float blur,
                        float near_plane, float* proj, float* mu2d, uint8_t* keep, int* cc, int2* cr,
                        const float* bt, cudaStream_t st) {
  switch (lpg) {
    case 1: launch_project<DEG, 1>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cc, cr, bt, st); break;
    case 2: launch_project<DEG, 2>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cc, cr, bt, st); break;
    case 4: launch_project<DEG, 4>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cc, cr, bt, st); break;
    default: launch_project<DEG, 8>(params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cc, cr, bt, st); break;
  }
}

static size_t a256b(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace tts

using namespace tts;

extern "C" int tts_project(const float* params, int G, int sh_degree, const float* cams, int V, int H, int W,
                           float blur, float near_plane, float* proj, float* mu2d, uint8_t* keep, int32_t* cell_count,
                           int32_t* cell_rank, const float* depth_bt, void* stream) {
  TTS_REQUIRE(G >= 0 && V >= 1, "G must be >= 0 and V >= 1");
  TTS_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_degree must be in [0, 3]");
  TTS_REQUIRE(H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(aligned16(proj), "proj must be 16-byte aligned");
  TTS_REQUIRE((long long)V * (H / 16) * (W / 16) < (1LL << 31), "V * tiles must fit in 31 bits");
  TTS_REQUIRE(cell_count, "null cell_count");
  cudaStream_t st = as_stream(stream);
  const int ntx = W / 16, nty = H / 16, lpg = lanes_for(V);
  if (cudaMemsetAsync(cell_count, 0, (size_t)V * ntx * nty * sizeof(int32_t), st) != cudaSuccess)
    return check_launch("memset cell counts");
  if (G == 0) return TTS_OK;
  int2* cr = reinterpret_cast<int2*>(cell_rank);
  const float* bt = depth_bt;
  switch (sh_degree) {
    case 0: project_deg<0>(lpg, params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr, bt, st); break;
    case 1: project_deg<1>(lpg, params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr, bt, st); break;
    case 2: project_deg<2>(lpg, params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr, bt, st); break;
    default: project_deg<3>(lpg, params, G, cams, V, ntx, nty, blur, near_plane, proj, mu2d, keep, cell_count, cr, bt, st); break;
  }
  return check_launch("project");
}

// gathered records, then (arm B) one (d beta, d tau) partial per backward block (at most G of them)
extern "C" size_t tts_backward_workspace_bytes(int G, int V) {
  return (G > 0 && V > 0) ? a256b((size_t)V * G * 48) + a256b((size_t)G * 8) : 0;
}

extern "C" int tts_backward_params(const float* params, int G, int sh_degree, const float* cams, int V, int H, int W,
                                   int R, int K, float k_poly, float blur, float near_plane, const float* proj,
                                   const int32_t* inv, const float* slot_grads, const float* gwb_partial,
                                   float lambda_o, float lambda_s, float* grads, const float* depth_bt,
                                   float* g_depth_bt, void* workspace, size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(G >= 1 && V >= 1, "G and V must be >= 1");
  TTS_REQUIRE(sh_degree >= 0 && sh_degree <= 3, "sh_degree must be in [0, 3]");
  TTS_REQUIRE(H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(R >= 0 && R <= 3 && K >= 1 && K <= 256, "R in [0,3] and K in [1,256]");
  TTS_REQUIRE(params && cams && proj && inv && slot_grads && gwb_partial && grads, "null pointer");
  TTS_REQUIRE((depth_bt == nullptr) == (g_depth_bt == nullptr), "depth_bt and g_depth_bt go together (arm B)");
  TTS_REQUIRE(((uintptr_t)slot_grads & 7u) == 0, "slot_grads must be 8-byte aligned");
  TTS_REQUIRE(aligned16(proj), "proj must be 16-byte aligned");
  TTS_REQUIRE(workspace && aligned16(workspace), "workspace must be a 16-byte aligned device buffer");
  if (workspace_bytes < tts_backward_workspace_bytes(G, V)) return fail(TTS_ERR_CAPACITY, "backward workspace too small");
  const int ntx = W / 16, nty = H / 16, S = (2 * R + 1) * (2 * R + 1);
  const float inv_k = (float)(1.0 / (double)k_poly);
  cudaStream_t st = as_stream(stream);
  const int lpg = lanes_for(V);
  float4* rec = static_cast<float4*>(workspace);
  float2* btp = reinterpret_cast<float2*>(static_cast<char*>(workspace) + a256b((size_t)V * G * 48));
  const long long nvg = (long long)V * G;
  k_slot_gather<<<(unsigned)((nvg + 255) / 256), 256, 0, st>>>(proj, G, V, ntx, ntx * nty, S, K, inv_k, inv,
                                                              slot_grads, rec);
  if (int rc = check_launch("slot_gather")) return rc;
  int nblk = 0;
#define TTS_BWD(D, P)                                                                                              \
  nblk = (G + GB_THREADS / P - 1) / (GB_THREADS / P);                                                              \
  if (depth_bt)                                                                                                    \
    k_backward<D, P, true><<<nblk, GB_THREADS, 0, st>>>(params, G, cams, V, blur, near_plane, rec, lambda_o,       \
                                                        lambda_s, grads, depth_bt, btp);                           \
  else                                                                                                             \
    k_backward<D, P, false><<<nblk, GB_THREADS, 0, st>>>(params, G, cams, V, blur, near_plane, rec, lambda_o,      \
                                                         lambda_s, grads, nullptr, nullptr);
#define TTS_BWD_DEG(D)            \
  switch (lpg) {                  \
    case 1: TTS_BWD(D, 1) break;  \
    case 2: TTS_BWD(D, 2) break;  \
    case 4: TTS_BWD(D, 4) break;  \
    default: TTS_BWD(D, 8) break; \
  }
  switch (sh_degree) {
    case 0: TTS_BWD_DEG(0) break;
    case 1: TTS_BWD_DEG(1) break;
    case 2: TTS_BWD_DEG(2) break;
    default: TTS_BWD_DEG(3) break;
  }
#undef TTS_BWD_DEG
#undef TTS_BWD
  if (int rc = check_launch("backward_params")) return rc;
  k_wb_reduce<<<1, 1024, 0, st>>>(gwb_partial, V * ntx * nty, params, G, grads, depth_bt ? btp : nullptr, nblk,
                                  g_depth_bt);
  return check_launch("wb_reduce");
}
