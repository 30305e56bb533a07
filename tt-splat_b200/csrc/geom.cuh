// Per-gaussian geometry and SH colour, forward and backward (thread-per-gaussian helpers).
//
// Forward follows spike/geometry.py:10-57 in the per-component form of the reference's manual
// geometry tools/geom_bwd.py:26-64; backward restates tools/geom_bwd.py:67-152.  SH colour
// follows spike/sh.py:49-72; its backward is the autograd of that expression (coefficients
// and viewing direction).  The same inline functions serve the projection kernel and the
// backward kernel, so the backward recomputes bit-identical forward intermediates.
#pragma once
#include "common.cuh"

namespace tts {

constexpr float SH_C0 = 0.28209479177387814f;
constexpr float SH_C1 = 0.4886025119029199f;
__device__ __constant__ static const float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f,
                                                      0.31539156525252005f, -1.0925484305920792f,
                                                      0.5462742152960396f};
__device__ __constant__ static const float SH_C3[7] = {
    -0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f, 0.3731763325901154f,
    -0.4570457994644658f, 1.445305721320277f, -0.5900435899266435f};

struct GeomFwd {
  float w, x, y, z, n;          // normalised quaternion and its (clamped) norm
  float M[3][3];                // R_v * R(q)
  float s[3], s2[3];            // scales and squares
  float SC00, SC01, SC02, SC11, SC12, SC22;
  float mcx, mcy, mcz, zmask, zi;
  float J00, J02, J11, J12;
  float s00, s01, s11, dmask, deti;
  float mux, muy, a, b, c;
  bool keep;
};

__device__ __forceinline__ void geom_forward(const float m[3], const float q[4], const float ls[3],
                                             const Cam& cam, float blur, float near_plane,
                                             GeomFwd& f) {
  float nn = sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
  f.n = fmaxf(nn, 1e-12f);
  f.w = q[0] / f.n; f.x = q[1] / f.n; f.y = q[2] / f.n; f.z = q[3] / f.n;
  const float w = f.w, x = f.x, y = f.y, z = f.z;
  float R[3][3] = {{1.f - 2.f * (y * y + z * z), 2.f * (x * y - w * z), 2.f * (x * z + w * y)},
                   {2.f * (x * y + w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - w * x)},
                   {2.f * (x * z - w * y), 2.f * (y * z + w * x), 1.f - 2.f * (x * x + y * y)}};
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int k = 0; k < 3; k++)
      f.M[i][k] = cam.R[i * 3 + 0] * R[0][k] + cam.R[i * 3 + 1] * R[1][k] + cam.R[i * 3 + 2] * R[2][k];
#pragma unroll
  for (int k = 0; k < 3; k++) {
    f.s[k] = expf(ls[k]);
    f.s2[k] = f.s[k] * f.s[k];
  }
#define TTS_SC(i, l) (f.M[i][0] * f.M[l][0] * f.s2[0] + f.M[i][1] * f.M[l][1] * f.s2[1] + f.M[i][2] * f.M[l][2] * f.s2[2])
  f.SC00 = TTS_SC(0, 0); f.SC01 = TTS_SC(0, 1); f.SC02 = TTS_SC(0, 2);
  f.SC11 = TTS_SC(1, 1); f.SC12 = TTS_SC(1, 2); f.SC22 = TTS_SC(2, 2);
#undef TTS_SC
  f.mcx = cam.R[0] * m[0] + cam.R[1] * m[1] + cam.R[2] * m[2] + cam.t[0];
  f.mcy = cam.R[3] * m[0] + cam.R[4] * m[1] + cam.R[5] * m[2] + cam.t[1];
  f.mcz = cam.R[6] * m[0] + cam.R[7] * m[1] + cam.R[8] * m[2] + cam.t[2];
  f.keep = f.mcz > near_plane;
  f.zmask = f.keep ? 1.f : 0.f;
  const float zc = fmaxf(f.mcz, near_plane);
  f.zi = 1.f / zc;
  f.mux = cam.fx * f.mcx / zc + cam.cx;
  f.muy = cam.fy * f.mcy / zc + cam.cy;
  f.J00 = cam.fx * f.zi;
  f.J11 = cam.fy * f.zi;
  f.J02 = -cam.fx * f.mcx * f.zi * f.zi;
  f.J12 = -cam.fy * f.mcy * f.zi * f.zi;
  // Sigma2d = A A^T + blur I with A = J (R_v R) diag(s) (2x3).  Its entries are sums of squares
  // and products of A, and its determinant is taken in the Cauchy-Binet form
  //   det = sum of the squared 2x2 minors of A + blur (tr A A^T) + blur^2,
  // every term non-negative, so det >= blur^2 as in exact arithmetic.  The textbook
  // s00 s11 - s01^2 (spike/geometry.py:54) cancels to fp32 rounding noise for thin gaussians just
  // past the near plane (mean far off-screen, Sigma2d nearly rank one), where the 1e-12 clamp then
  // yields conics of ~1e20 whose tile-local polynomial overflows the render; the float64 value of
  // those conics is bounded by 1/blur, and this form stays within fp32 rounding of it.
  float A0[3], A1[3];
#pragma unroll
  for (int k = 0; k < 3; k++) {
    A0[k] = (f.J00 * f.M[0][k] + f.J02 * f.M[2][k]) * f.s[k];
    A1[k] = (f.J11 * f.M[1][k] + f.J12 * f.M[2][k]) * f.s[k];
  }
  const float p00 = A0[0] * A0[0] + A0[1] * A0[1] + A0[2] * A0[2];
  const float p11 = A1[0] * A1[0] + A1[1] * A1[1] + A1[2] * A1[2];
  f.s00 = p00 + blur;
  f.s11 = p11 + blur;
  f.s01 = A0[0] * A1[0] + A0[1] * A1[1] + A0[2] * A1[2];
  const float m01 = A0[0] * A1[1] - A0[1] * A1[0];
  const float m02 = A0[0] * A1[2] - A0[2] * A1[0];
  const float m12 = A0[1] * A1[2] - A0[2] * A1[1];
  const float det = (m01 * m01 + m02 * m02 + m12 * m12) + blur * (p00 + p11) + blur * blur;
  f.dmask = det > 1e-12f ? 1.f : 0.f;
  const float detc = fmaxf(det, 1e-12f);
  f.deti = 1.f / detc;
  f.a = f.s11 / detc;
  f.b = -f.s01 / detc;
  f.c = f.s00 / detc;
}

// tools/geom_bwd.py:67-152: (gconic, gmu2d) -> gmeans, gquat, gscale (added into the outputs).
__device__ __forceinline__ void geom_backward(const GeomFwd& f, const Cam& cam, float ga, float gb,
                                              float gc, float gmux, float gmuy, float gm[3],
                                              float gq[4], float gs[3]) {
  const float deti = f.deti;
  float gs11 = ga * deti, gs01 = -gb * deti, gs00 = gc * deti;
  const float gdeti = ga * f.s11 + (-gb) * f.s01 + gc * f.s00;
  const float gdet = -gdeti * deti * deti * f.dmask;
  gs00 += gdet * f.s11;
  gs11 += gdet * f.s00;
  gs01 += gdet * (-2.f * f.s01);
  const float J00 = f.J00, J02 = f.J02, J11 = f.J11, J12 = f.J12;
  const float gJ00 = gs00 * (2.f * J00 * f.SC00 + 2.f * J02 * f.SC02) + gs01 * (J11 * f.SC01 + J12 * f.SC02);
  const float gJ02 = gs00 * (2.f * J00 * f.SC02 + 2.f * J02 * f.SC22) + gs01 * (J11 * f.SC12 + J12 * f.SC22);
  const float gJ11 = gs11 * (2.f * J11 * f.SC11 + 2.f * J12 * f.SC12) + gs01 * (J00 * f.SC01 + J02 * f.SC12);
  const float gJ12 = gs11 * (2.f * J11 * f.SC12 + 2.f * J12 * f.SC22) + gs01 * (J00 * f.SC02 + J02 * f.SC22);
  const float gSC00 = gs00 * J00 * J00;
  const float gSC11 = gs11 * J11 * J11;
  const float gSC22 = gs00 * J02 * J02 + gs11 * J12 * J12 + gs01 * J02 * J12;
  const float gSC02 = gs00 * 2.f * J00 * J02 + gs01 * J00 * J12;
  const float gSC12 = gs11 * 2.f * J11 * J12 + gs01 * J02 * J11;
  const float gSC01 = gs01 * J00 * J11;
  const float fx = cam.fx, fy = cam.fy, zi = f.zi;
  const float gmcx = gmux * fx * zi + gJ02 * (-fx * zi * zi);
  const float gmcy = gmuy * fy * zi + gJ12 * (-fy * zi * zi);
  const float gzi = gmux * fx * f.mcx + gmuy * fy * f.mcy + gJ00 * fx + gJ11 * fy +
                    gJ02 * (-fx * f.mcx * 2.f * zi) + gJ12 * (-fy * f.mcy * 2.f * zi);
  const float gmcz = -gzi * zi * zi * f.zmask;
#pragma unroll
  for (int i = 0; i < 3; i++) gm[i] += gmcx * cam.R[0 * 3 + i] + gmcy * cam.R[1 * 3 + i] + gmcz * cam.R[2 * 3 + i];
  float gM[3][3], gs2[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int k = 0; k < 3; k++) gM[i][k] = 0.f;
  const float gdiag[3] = {gSC00, gSC11, gSC22};
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int k = 0; k < 3; k++) {
      gM[i][k] += gdiag[i] * 2.f * f.M[i][k] * f.s2[k];
      gs2[k] += gdiag[i] * f.M[i][k] * f.M[i][k];
    }
  const float goff[3] = {gSC01, gSC02, gSC12};
  const int oi[3] = {0, 0, 1}, ol[3] = {1, 2, 2};
#pragma unroll
  for (int e = 0; e < 3; e++)
#pragma unroll
    for (int k = 0; k < 3; k++) {
      gM[oi[e]][k] += goff[e] * f.M[ol[e]][k] * f.s2[k];
      gM[ol[e]][k] += goff[e] * f.M[oi[e]][k] * f.s2[k];
      gs2[k] += goff[e] * f.M[oi[e]][k] * f.M[ol[e]][k];
    }
#pragma unroll
  for (int k = 0; k < 3; k++) gs[k] += gs2[k] * 2.f * f.s[k];
  float gR[3][3];
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int k = 0; k < 3; k++)
      gR[i][k] = cam.R[0 * 3 + i] * gM[0][k] + cam.R[1 * 3 + i] * gM[1][k] + cam.R[2 * 3 + i] * gM[2][k];
  const float w = f.w, x = f.x, y = f.y, z = f.z;
  const float gw = gR[0][1] * (-2.f * z) + gR[0][2] * (2.f * y) + gR[1][0] * (2.f * z) +
                   gR[1][2] * (-2.f * x) + gR[2][0] * (-2.f * y) + gR[2][1] * (2.f * x);
  const float gx = gR[0][1] * (2.f * y) + gR[0][2] * (2.f * z) + gR[1][0] * (2.f * y) +
                   gR[1][1] * (-4.f * x) + gR[1][2] * (-2.f * w) + gR[2][0] * (2.f * z) +
                   gR[2][1] * (2.f * w) + gR[2][2] * (-4.f * x);
  const float gy = gR[0][0] * (-4.f * y) + gR[0][1] * (2.f * x) + gR[0][2] * (2.f * w) +
                   gR[1][0] * (2.f * x) + gR[1][2] * (2.f * z) + gR[2][0] * (-2.f * w) +
                   gR[2][1] * (2.f * z) + gR[2][2] * (-4.f * y);
  const float gz = gR[0][0] * (-4.f * z) + gR[0][1] * (-2.f * w) + gR[0][2] * (2.f * x) +
                   gR[1][0] * (2.f * w) + gR[1][1] * (-4.f * z) + gR[1][2] * (2.f * y) +
                   gR[2][0] * (2.f * x) + gR[2][1] * (2.f * y);
  const float dot = w * gw + x * gx + y * gy + z * gz;
  const float in = 1.f / f.n;
  gq[0] += (gw - w * dot) * in;
  gq[1] += (gx - x * dot) * in;
  gq[2] += (gy - y * dot) * in;
  gq[3] += (gz - z * dot) * in;
}

// SH basis (spike/sh.py:57-71 coefficient order) for a unit direction.
__device__ __forceinline__ void sh_basis(int deg, float x, float y, float z, float b[16]) {
  b[0] = SH_C0;
  if (deg >= 1) { b[1] = -SH_C1 * y; b[2] = SH_C1 * z; b[3] = -SH_C1 * x; }
  if (deg >= 2) {
    const float xx = x * x, yy = y * y, zz = z * z;
    b[4] = SH_C2[0] * x * y; b[5] = SH_C2[1] * y * z; b[6] = SH_C2[2] * (2.f * zz - xx - yy);
    b[7] = SH_C2[3] * x * z; b[8] = SH_C2[4] * (xx - yy);
  }
  if (deg >= 3) {
    const float xx = x * x, yy = y * y, zz = z * z;
    b[9] = SH_C3[0] * y * (3.f * xx - yy); b[10] = SH_C3[1] * x * y * z;
    b[11] = SH_C3[2] * y * (4.f * zz - xx - yy); b[12] = SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy);
    b[13] = SH_C3[4] * x * (4.f * zz - xx - yy); b[14] = SH_C3[5] * z * (xx - yy);
    b[15] = SH_C3[6] * x * (xx - 3.f * yy);
  }
}

// d basis_k / d(x, y, z) for k >= 1 (polynomial derivatives of sh_basis).
__device__ __forceinline__ void sh_basis_grad(int k, float x, float y, float z, float& dx, float& dy,
                                              float& dz) {
  const float xx = x * x, yy = y * y, zz = z * z;
  switch (k) {
    case 1: dx = 0.f; dy = -SH_C1; dz = 0.f; break;
    case 2: dx = 0.f; dy = 0.f; dz = SH_C1; break;
    case 3: dx = -SH_C1; dy = 0.f; dz = 0.f; break;
    case 4: dx = SH_C2[0] * y; dy = SH_C2[0] * x; dz = 0.f; break;
    case 5: dx = 0.f; dy = SH_C2[1] * z; dz = SH_C2[1] * y; break;
    case 6: dx = -2.f * SH_C2[2] * x; dy = -2.f * SH_C2[2] * y; dz = 4.f * SH_C2[2] * z; break;
    case 7: dx = SH_C2[3] * z; dy = 0.f; dz = SH_C2[3] * x; break;
    case 8: dx = 2.f * SH_C2[4] * x; dy = -2.f * SH_C2[4] * y; dz = 0.f; break;
    case 9: dx = 6.f * SH_C3[0] * x * y; dy = SH_C3[0] * (3.f * xx - 3.f * yy); dz = 0.f; break;
    case 10: dx = SH_C3[1] * y * z; dy = SH_C3[1] * x * z; dz = SH_C3[1] * x * y; break;
    case 11: dx = -2.f * SH_C3[2] * x * y; dy = SH_C3[2] * (4.f * zz - xx - 3.f * yy); dz = 8.f * SH_C3[2] * y * z; break;
    case 12: dx = -6.f * SH_C3[3] * x * z; dy = -6.f * SH_C3[3] * y * z; dz = SH_C3[3] * (6.f * zz - 3.f * xx - 3.f * yy); break;
    case 13: dx = SH_C3[4] * (4.f * zz - 3.f * xx - yy); dy = -2.f * SH_C3[4] * x * y; dz = 8.f * SH_C3[4] * x * z; break;
    case 14: dx = 2.f * SH_C3[5] * x * z; dy = -2.f * SH_C3[5] * y * z; dz = SH_C3[5] * (xx - yy); break;
    case 15: dx = SH_C3[6] * (3.f * xx - 3.f * yy); dy = -6.f * SH_C3[6] * x * y; dz = 0.f; break;
    default: dx = dy = dz = 0.f;
  }
}

// Normalised viewing direction means - centre (spike/render.py:25, spike/sh.py:55).
__device__ __forceinline__ void view_dir(const float m[3], const Cam& cam, float d[3], float& nrm) {
  const float dx = m[0] - cam.c[0], dy = m[1] - cam.c[1], dz = m[2] - cam.c[2];
  nrm = sqrtf(dx * dx + dy * dy + dz * dz);
  const float nc = fmaxf(nrm, 1e-12f);
  d[0] = dx / nc; d[1] = dy / nc; d[2] = dz / nc;
}

}  // namespace tts
