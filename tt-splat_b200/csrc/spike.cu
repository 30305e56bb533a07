// The reference's composable spike API on the device: the small differentiable building blocks of
// spike/geometry.py (quat_to_rotmat, cov3d, project_ewa), spike/sh.py (eval_sh_color) and
// spike/forward.py (quad_form, theta_from_conic, phi, the tile-local GEMM form of Q,
// poly_splat_wgeo, color_from_dc), each as a forward and a backward kernel, in fp32 or fp64.
//
// The training and rendering hot path fuses these steps (k_project, k_backward, the tile
// kernels); these entry points serve callers that compose the reference's functions by hand,
// such as its dense render (spike/render.py:14-49) and its tests.  Element-wise steps are a
// thread per element (grid-stride).  Reductions over the pixels of a [P,G] gradient run in two
// deterministic passes: per-chunk partials in a caller workspace, then a fixed-order sum.
// Camera intrinsics and poses are constants here (the reference never differentiates them).
#include "common.cuh"

namespace tts {
namespace {

constexpr int SP_THREADS = 256;
constexpr int SP_MAX_BLOCKS = 148 * 16;
constexpr int SP_REDUCE_BLOCKS = 148 * 8;   // target blocks of a partials pass
constexpr int SP_MAX_CHUNKS = 256;          // pixel chunks of a partials pass
constexpr int SP_MAX_ACC = 6;               // accumulators per gaussian in a partials pass

__device__ __forceinline__ float tsqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double tsqrt(double x) { return sqrt(x); }
template <typename T>
__device__ __forceinline__ T tmax(T a, T b) {
  return a > b ? a : b;
}

unsigned grid_for(long long n) {
  long long b = (n + SP_THREADS - 1) / SP_THREADS;
  return (unsigned)(b < 1 ? 1 : (b > SP_MAX_BLOCKS ? SP_MAX_BLOCKS : b));
}

// Individually rounded arithmetic (no FMA contraction): the reference's expressions evaluated
// in its op order, as torch's CPU kernels do.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }

#define SP_LOOP(i, n) \
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (n); i += (long long)gridDim.x * blockDim.x)

// ---- quaternion -> rotation (spike/geometry.py:10-19) -----------------------------------------
// q / max(|q|, 1e-12), then the rotation matrix of the unit quaternion (w, x, y, z).  `flows` is
// whether the norm passed the clamp (the clamp's gradient is zero below its bound).
template <typename T>
__device__ __forceinline__ void quat_unit(const T* q, T u[4], T& n, bool& flows) {
  const T s = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
  const T nrm = tsqrt(s);
  flows = nrm >= T(1e-12);
  n = flows ? nrm : T(1e-12);
#pragma unroll
  for (int i = 0; i < 4; ++i) u[i] = q[i] / n;
}

template <typename T>
__device__ __forceinline__ void rot_of(const T u[4], T R[9]) {
  const T w = u[0], x = u[1], y = u[2], z = u[3];
  R[0] = T(1) - T(2) * (y * y + z * z); R[1] = T(2) * (x * y - w * z); R[2] = T(2) * (x * z + w * y);
  R[3] = T(2) * (x * y + w * z); R[4] = T(1) - T(2) * (x * x + z * z); R[5] = T(2) * (y * z - w * x);
  R[6] = T(2) * (x * z - w * y); R[7] = T(2) * (y * z + w * x); R[8] = T(1) - T(2) * (x * x + y * y);
}

template <typename T>
__global__ void __launch_bounds__(SP_THREADS) k_quat_rotmat(const T* __restrict__ q, long long n, T* __restrict__ R) {
  SP_LOOP(i, n) {
    T u[4], nrm, r[9];
    bool flows;
    quat_unit(q + 4 * i, u, nrm, flows);
    rot_of(u, r);
#pragma unroll
    for (int k = 0; k < 9; ++k) R[9 * i + k] = r[k];
  }
}

// dR/du contracted with gR, then through the normalisation: (g - u (u.g)) / |q| when the norm
// is above the clamp, g / 1e-12 below it.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_quat_rotmat_bwd(const T* __restrict__ q, const T* __restrict__ gR, long long n, T* __restrict__ gq) {
  SP_LOOP(i, n) {
    T u[4], nrm;
    bool flows;
    quat_unit(q + 4 * i, u, nrm, flows);
    const T* g = gR + 9 * i;
    const T w = u[0], x = u[1], y = u[2], z = u[3];
    T gu[4];
    gu[0] = T(2) * (-z * g[1] + y * g[2] + z * g[3] - x * g[5] - y * g[6] + x * g[7]);
    gu[1] = T(2) * (y * g[1] + z * g[2] + y * g[3] - T(2) * x * g[4] - w * g[5] + z * g[6] + w * g[7] - T(2) * x * g[8]);
    gu[2] = T(2) * (-T(2) * y * g[0] + x * g[1] + w * g[2] + x * g[3] + z * g[5] - w * g[6] + z * g[7] - T(2) * y * g[8]);
    gu[3] = T(2) * (-T(2) * z * g[0] - w * g[1] + x * g[2] + w * g[3] - T(2) * z * g[4] + y * g[5] + x * g[6] + y * g[7]);
    const T dot = flows ? (u[0] * gu[0] + u[1] * gu[1] + u[2] * gu[2] + u[3] * gu[3]) : T(0);
#pragma unroll
    for (int k = 0; k < 4; ++k) gq[4 * i + k] = (gu[k] - u[k] * dot) / nrm;
  }
}

// ---- 3-D covariance R diag(s^2) R^T (spike/geometry.py:22-25) -------------------------------
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_cov3d(const T* __restrict__ s, const T* __restrict__ R, long long n, T* __restrict__ cov) {
  SP_LOOP(i, n) {
    const T* r = R + 9 * i;
    const T s2[3] = {s[3 * i] * s[3 * i], s[3 * i + 1] * s[3 * i + 1], s[3 * i + 2] * s[3 * i + 2]};
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        cov[9 * i + 3 * a + b] = r[3 * a] * s2[0] * r[3 * b] + r[3 * a + 1] * s2[1] * r[3 * b + 1] +
                                 r[3 * a + 2] * s2[2] * r[3 * b + 2];
  }
}

template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_cov3d_bwd(const T* __restrict__ s, const T* __restrict__ R, const T* __restrict__ gcov, long long n,
                T* __restrict__ gs, T* __restrict__ gR) {
  SP_LOOP(i, n) {
    const T* r = R + 9 * i;
    const T* g = gcov + 9 * i;
    T s2[3], gs2[3] = {T(0), T(0), T(0)}, gr[9];
#pragma unroll
    for (int k = 0; k < 3; ++k) s2[k] = s[3 * i + k] * s[3 * i + k];
#pragma unroll
    for (int e = 0; e < 9; ++e) gr[e] = T(0);
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) {
        const T gab = g[3 * a + b];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          gr[3 * a + k] += gab * s2[k] * r[3 * b + k];
          gr[3 * b + k] += gab * r[3 * a + k] * s2[k];
          gs2[k] += gab * r[3 * a + k] * r[3 * b + k];
        }
      }
#pragma unroll
    for (int k = 0; k < 3; ++k) gs[3 * i + k] = T(2) * s[3 * i + k] * gs2[k];
#pragma unroll
    for (int e = 0; e < 9; ++e) gR[9 * i + e] = gr[e];
  }
}

// ---- EWA projection (spike/geometry.py:28-57) ---------------------------------------------------
template <typename T>
struct PinholeT {
  T R[9], t[3], fx, fy, cx, cy;
};

template <typename T>
struct EwaFwd {
  T mc[3], z, Sc[9], J[6], S00, S01, S11, det;
  bool z_flows, det_flows;
};

// mu_cam = R_v m + t_v; z = max(depth, near); mu2d = f mu_cam / z + c; Sigma_cam = R_v S R_v^T;
// J = d(mu2d)/d(mu_cam); Sigma2d = J Sigma_cam J^T + blur I; conic = its inverse (det >= 1e-12).
template <typename T>
__device__ __forceinline__ void ewa_forward(const T* m, const T* S, const PinholeT<T>& c, T blur, T near_plane,
                                            EwaFwd<T>& f) {
#pragma unroll
  for (int a = 0; a < 3; ++a) f.mc[a] = c.R[3 * a] * m[0] + c.R[3 * a + 1] * m[1] + c.R[3 * a + 2] * m[2] + c.t[a];
  f.z_flows = f.mc[2] >= near_plane;
  f.z = tmax(f.mc[2], near_plane);
  T RS[9];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int k = 0; k < 3; ++k) RS[3 * a + k] = c.R[3 * a] * S[k] + c.R[3 * a + 1] * S[3 + k] + c.R[3 * a + 2] * S[6 + k];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int l = 0; l < 3; ++l)
      f.Sc[3 * a + l] = RS[3 * a] * c.R[3 * l] + RS[3 * a + 1] * c.R[3 * l + 1] + RS[3 * a + 2] * c.R[3 * l + 2];
  const T z = f.z;
  f.J[0] = c.fx / z; f.J[1] = T(0); f.J[2] = -c.fx * f.mc[0] / (z * z);
  f.J[3] = T(0); f.J[4] = c.fy / z; f.J[5] = -c.fy * f.mc[1] / (z * z);
  T JS[6];   // J Sigma_cam [2,3]
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int k = 0; k < 3; ++k)
      JS[3 * a + k] = f.J[3 * a] * f.Sc[k] + f.J[3 * a + 1] * f.Sc[3 + k] + f.J[3 * a + 2] * f.Sc[6 + k];
  f.S00 = JS[0] * f.J[0] + JS[1] * f.J[1] + JS[2] * f.J[2] + blur;
  f.S01 = JS[0] * f.J[3] + JS[1] * f.J[4] + JS[2] * f.J[5];
  f.S11 = JS[3] * f.J[3] + JS[4] * f.J[4] + JS[5] * f.J[5] + blur;
  const T d = f.S00 * f.S11 - f.S01 * f.S01;
  f.det_flows = d >= T(1e-12);
  f.det = tmax(d, T(1e-12));
}

template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_project_ewa(const T* __restrict__ means, const T* __restrict__ cov, long long G, PinholeT<T> c, T blur,
                  T near_plane, T* __restrict__ mu2d, T* __restrict__ conic, T* __restrict__ depth,
                  uint8_t* __restrict__ keep) {
  SP_LOOP(g, G) {
    EwaFwd<T> f;
    ewa_forward(means + 3 * g, cov + 9 * g, c, blur, near_plane, f);
    mu2d[2 * g] = c.fx * f.mc[0] / f.z + c.cx;
    mu2d[2 * g + 1] = c.fy * f.mc[1] / f.z + c.cy;
    conic[3 * g] = f.S11 / f.det;
    conic[3 * g + 1] = -f.S01 / f.det;
    conic[3 * g + 2] = f.S00 / f.det;
    depth[g] = f.mc[2];
    keep[g] = f.mc[2] > near_plane ? 1 : 0;
  }
}

// The autograd of the forward above: (gmu2d, gconic, gdepth; each may be NULL = zero) ->
// gmeans[G,3], gcov[G,3,3].  Sigma2d's (1,0) entry is unused by the conic, so gSigma2d is upper
// triangular; gJ = gS (Sigma_cam J^T)^T + gS^T (J Sigma_cam), gSigma_cam = J^T gS J,
// gcov = R_v^T gSigma_cam R_v.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_project_ewa_bwd(const T* __restrict__ means, const T* __restrict__ cov, long long G, PinholeT<T> c, T blur,
                      T near_plane, const T* __restrict__ gmu2d, const T* __restrict__ gconic,
                      const T* __restrict__ gdepth, T* __restrict__ gmeans, T* __restrict__ gcov) {
  SP_LOOP(g, G) {
    EwaFwd<T> f;
    ewa_forward(means + 3 * g, cov + 9 * g, c, blur, near_plane, f);
    const T ga = gconic ? gconic[3 * g] : T(0), gb = gconic ? gconic[3 * g + 1] : T(0);
    const T gc = gconic ? gconic[3 * g + 2] : T(0);
    const T gm0 = gmu2d ? gmu2d[2 * g] : T(0), gm1 = gmu2d ? gmu2d[2 * g + 1] : T(0);
    const T det = f.det;
    T gS00 = gc / det, gS11 = ga / det, gS01 = -gb / det;
    if (f.det_flows) {
      const T gdet = -(ga * f.S11 - gb * f.S01 + gc * f.S00) / (det * det);
      gS00 += gdet * f.S11;
      gS11 += gdet * f.S00;
      gS01 += gdet * (T(-2) * f.S01);
    }
    const T gS[4] = {gS00, gS01, T(0), gS11};   // [i][l], row-major 2x2
    T A[6], B[6];   // A = Sigma_cam J^T [3,2], B = J Sigma_cam [2,3]
#pragma unroll
    for (int b = 0; b < 3; ++b)
#pragma unroll
      for (int l = 0; l < 2; ++l)
        A[2 * b + l] = f.Sc[3 * b] * f.J[3 * l] + f.Sc[3 * b + 1] * f.J[3 * l + 1] + f.Sc[3 * b + 2] * f.J[3 * l + 2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        B[3 * i + b] = f.J[3 * i] * f.Sc[b] + f.J[3 * i + 1] * f.Sc[3 + b] + f.J[3 * i + 2] * f.Sc[6 + b];
    T gJ[6];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        gJ[3 * a + b] = gS[2 * a] * A[2 * b] + gS[2 * a + 1] * A[2 * b + 1] + gS[a] * B[b] + gS[2 + a] * B[3 + b];
    T gSc[9];   // J^T gS J
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        T acc = T(0);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int l = 0; l < 2; ++l) acc += gS[2 * i + l] * f.J[3 * i + j] * f.J[3 * l + k];
        gSc[3 * j + k] = acc;
      }
    // gcov = R^T gSc R
    T tmp[9];
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int l = 0; l < 3; ++l)
        tmp[3 * j + l] = c.R[j] * gSc[l] + c.R[3 + j] * gSc[3 + l] + c.R[6 + j] * gSc[6 + l];
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int k = 0; k < 3; ++k)
        gcov[9 * g + 3 * j + k] = tmp[3 * j] * c.R[k] + tmp[3 * j + 1] * c.R[3 + k] + tmp[3 * j + 2] * c.R[6 + k];
    const T z = f.z, z2 = z * z, z3 = z2 * z;
    const T gz = gJ[0] * (-c.fx / z2) + gJ[2] * (T(2) * c.fx * f.mc[0] / z3) + gJ[4] * (-c.fy / z2) +
                 gJ[5] * (T(2) * c.fy * f.mc[1] / z3) + gm0 * (-c.fx * f.mc[0] / z2) + gm1 * (-c.fy * f.mc[1] / z2);
    const T gmc0 = gJ[2] * (-c.fx / z2) + gm0 * c.fx / z;
    const T gmc1 = gJ[5] * (-c.fy / z2) + gm1 * c.fy / z;
    const T gmc2 = (gdepth ? gdepth[g] : T(0)) + (f.z_flows ? gz : T(0));
#pragma unroll
    for (int k = 0; k < 3; ++k) gmeans[3 * g + k] = c.R[k] * gmc0 + c.R[3 + k] * gmc1 + c.R[6 + k] * gmc2;
  }
}

// ---- real SH, degrees 0-3 (spike/sh.py:49-72) ---------------------------------------------------
template <typename T>
__device__ __forceinline__ void sh_basis_t(int deg, T x, T y, T z, T b[16]) {
  const T C0 = T(0.28209479177387814), C1 = T(0.4886025119029199);
  b[0] = C0;
  if (deg >= 1) { b[1] = -C1 * y; b[2] = C1 * z; b[3] = -C1 * x; }
  if (deg >= 2) {
    const T xx = x * x, yy = y * y, zz = z * z;
    b[4] = T(1.0925484305920792) * x * y; b[5] = T(-1.0925484305920792) * y * z;
    b[6] = T(0.31539156525252005) * (T(2) * zz - xx - yy); b[7] = T(-1.0925484305920792) * x * z;
    b[8] = T(0.5462742152960396) * (xx - yy);
  }
  if (deg >= 3) {
    const T xx = x * x, yy = y * y, zz = z * z;
    b[9] = T(-0.5900435899266435) * y * (T(3) * xx - yy); b[10] = T(2.890611442640554) * x * y * z;
    b[11] = T(-0.4570457994644658) * y * (T(4) * zz - xx - yy);
    b[12] = T(0.3731763325901154) * z * (T(2) * zz - T(3) * xx - T(3) * yy);
    b[13] = T(-0.4570457994644658) * x * (T(4) * zz - xx - yy); b[14] = T(1.445305721320277) * z * (xx - yy);
    b[15] = T(-0.5900435899266435) * x * (xx - T(3) * yy);
  }
}

// Gradient of sum_k w_k basis_k(x, y, z) with respect to (x, y, z).
template <typename T>
__device__ __forceinline__ void sh_basis_vjp(int deg, T x, T y, T z, const T w[16], T& dx, T& dy, T& dz) {
  const T C1 = T(0.4886025119029199);
  dx = dy = dz = T(0);
  if (deg >= 1) { dy -= C1 * w[1]; dz += C1 * w[2]; dx -= C1 * w[3]; }
  if (deg >= 2) {
    const T a = T(1.0925484305920792), b6 = T(0.31539156525252005), b8 = T(0.5462742152960396);
    dx += a * y * w[4]; dy += a * x * w[4];
    dy -= a * z * w[5]; dz -= a * y * w[5];
    dx -= T(2) * b6 * x * w[6]; dy -= T(2) * b6 * y * w[6]; dz += T(4) * b6 * z * w[6];
    dx -= a * z * w[7]; dz -= a * x * w[7];
    dx += T(2) * b8 * x * w[8]; dy -= T(2) * b8 * y * w[8];
  }
  if (deg >= 3) {
    const T xx = x * x, yy = y * y, zz = z * z;
    const T c9 = T(-0.5900435899266435), c10 = T(2.890611442640554), c11 = T(-0.4570457994644658);
    const T c12 = T(0.3731763325901154), c14 = T(1.445305721320277);
    dx += T(6) * c9 * x * y * w[9]; dy += c9 * (T(3) * xx - T(3) * yy) * w[9];
    dx += c10 * y * z * w[10]; dy += c10 * x * z * w[10]; dz += c10 * x * y * w[10];
    dx += T(-2) * c11 * x * y * w[11]; dy += c11 * (T(4) * zz - xx - T(3) * yy) * w[11]; dz += T(8) * c11 * y * z * w[11];
    dx += T(-6) * c12 * x * z * w[12]; dy += T(-6) * c12 * y * z * w[12];
    dz += c12 * (T(6) * zz - T(3) * xx - T(3) * yy) * w[12];
    dx += c11 * (T(4) * zz - T(3) * xx - yy) * w[13]; dy += T(-2) * c11 * x * y * w[13]; dz += T(8) * c11 * x * z * w[13];
    dx += T(2) * c14 * x * z * w[14]; dy += T(-2) * c14 * y * z * w[14]; dz += c14 * (xx - yy) * w[14];
    dx += c9 * (T(3) * xx - T(3) * yy) * w[15]; dy += T(-6) * c9 * x * y * w[15];
  }
}

template <typename T>
__device__ __forceinline__ void unit_dir(const T* d, T u[3], T& n, bool& flows) {
  const T nrm = tsqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  flows = nrm >= T(1e-12);
  n = flows ? nrm : T(1e-12);
  u[0] = d[0] / n; u[1] = d[1] / n; u[2] = d[2] / n;
}

// out[g, ch] = sum_k basis_k(dir_g) coeffs[g, k, ch] over k < (deg+1)^2; colour mode adds 0.5 and
// clamps at 0 (eval_sh_color), raw mode returns the sum (the scalar SH of spike/sh.py:20-30).
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_eval_sh(int deg, const T* __restrict__ coeffs, int nc, int nch, const T* __restrict__ dirs, long long G,
              int raw, T* __restrict__ out) {
  const int nb = (deg + 1) * (deg + 1);
  SP_LOOP(g, G) {
    T u[3], n, b[16];
    bool flows;
    unit_dir(dirs + 3 * g, u, n, flows);
    sh_basis_t(deg, u[0], u[1], u[2], b);
    const T* cg = coeffs + (long long)g * nc * nch;
    for (int ch = 0; ch < nch; ++ch) {
      T r = T(0);
      for (int k = 0; k < nb; ++k) r += b[k] * cg[k * nch + ch];
      out[(long long)g * nch + ch] = raw ? r : tmax(r + T(0.5), T(0));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_eval_sh_bwd(int deg, const T* __restrict__ coeffs, int nc, int nch, const T* __restrict__ dirs, long long G,
                  int raw, const T* __restrict__ gout, T* __restrict__ gcoeffs, T* __restrict__ gdirs) {
  const int nb = (deg + 1) * (deg + 1);
  SP_LOOP(g, G) {
    T u[3], n, b[16], w[16];
    bool flows;
    unit_dir(dirs + 3 * g, u, n, flows);
    sh_basis_t(deg, u[0], u[1], u[2], b);
    const T* cg = coeffs + (long long)g * nc * nch;
    T* gc = gcoeffs + (long long)g * nc * nch;
    for (int k = 0; k < 16; ++k) w[k] = T(0);
    for (int ch = 0; ch < nch; ++ch) {
      T gr = gout[(long long)g * nch + ch];
      if (!raw) {
        T r = T(0);
        for (int k = 0; k < nb; ++k) r += b[k] * cg[k * nch + ch];
        if (!(r + T(0.5) >= T(0))) gr = T(0);      // clamp(min=0) passes the gradient where x >= 0
      }
      for (int k = 0; k < nb; ++k) {
        gc[k * nch + ch] = b[k] * gr;
        w[k] += cg[k * nch + ch] * gr;
      }
      for (int k = nb; k < nc; ++k) gc[k * nch + ch] = T(0);
    }
    T du[3];
    sh_basis_vjp(deg, u[0], u[1], u[2], w, du[0], du[1], du[2]);
    const T dot = flows ? (u[0] * du[0] + u[1] * du[1] + u[2] * du[2]) : T(0);
#pragma unroll
    for (int k = 0; k < 3; ++k) gdirs[3 * g + k] = (du[k] - u[k] * dot) / n;
  }
}

// ---- colour from the DC coefficient (spike/forward.py:69-71) ---------------------------------
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_color_dc(const T* __restrict__ dc, long long n, const T* __restrict__ gout, T* __restrict__ out) {
  const T C0 = T(0.28209479177387814);
  SP_LOOP(i, n) {
    const T pre = T(0.5) + C0 * dc[i];
    out[i] = gout ? (pre >= T(0) ? C0 * gout[i] : T(0)) : tmax(pre, T(0));
  }
}

// ---- monomial basis Phi = [px^2, py^2, px py, px, py, 1] (spike/forward.py:42-44) -------------
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_phi(const T* __restrict__ px, const T* __restrict__ py, long long P, T* __restrict__ Phi) {
  SP_LOOP(p, P) {
    const T x = px[p], y = py[p];
    T* o = Phi + 6 * p;
    o[0] = x * x; o[1] = y * y; o[2] = x * y; o[3] = x; o[4] = y; o[5] = T(1);
  }
}

template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_phi_bwd(const T* __restrict__ px, const T* __restrict__ py, const T* __restrict__ gPhi, long long P,
              T* __restrict__ gpx, T* __restrict__ gpy) {
  SP_LOOP(p, P) {
    const T x = px[p], y = py[p];
    const T* g = gPhi + 6 * p;
    gpx[p] = T(2) * x * g[0] + y * g[2] + g[3];
    gpy[p] = T(2) * y * g[1] + x * g[2] + g[4];
  }
}

// ---- theta from the conic (spike/forward.py:23-39; gathered order tools/m4_train_binned.py:130-143)
// theta_Q = [a, c, 2b, -2(a mx + b my), -2(b mx + c my), a mx^2 + 2 b mx my + c my^2] over
// Phi, theta_u = (-1/k) theta_Q + [0,0,0,0,0,1].  The mean is taken relative to
// origins[i / per] when origins is given.  layout 0 writes [n,6]; layout 1 writes theta_u as
// [n/per, 6, per] (the [T,6,K] operand of the binned render) in the op order of
// theta_u_gathered, bit-identical to the slot rows of the binning kernel.  1/k is formed in
// double and rounded to T, as the reference's Python scalar is.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_theta(const T* __restrict__ conic, const T* __restrict__ mu, const T* __restrict__ origins, long long per,
            long long n, double k, int layout, T* __restrict__ thQ, T* __restrict__ thU) {
  const T two = T(2);
  SP_LOOP(i, n) {
    const T a = conic[3 * i], b = conic[3 * i + 1], c = conic[3 * i + 2];
    T mx = mu[2 * i], my = mu[2 * i + 1];
    if (origins) {
      mx = sub_rn(mx, origins[2 * (i / per)]);
      my = sub_rn(my, origins[2 * (i / per) + 1]);
    }
    if (layout == 1) {
      const T ik = (T)(1.0 / k);
      const T Q = add_rn(add_rn(mul_rn(mul_rn(a, mx), mx), mul_rn(mul_rn(mul_rn(two, b), mx), my)),
                         mul_rn(mul_rn(c, my), my));
      const T th[6] = {mul_rn(-a, ik), mul_rn(-c, ik), mul_rn(mul_rn(T(-2), b), ik),
                       mul_rn(mul_rn(two, add_rn(mul_rn(a, mx), mul_rn(b, my))), ik),
                       mul_rn(mul_rn(two, add_rn(mul_rn(b, mx), mul_rn(c, my))), ik), sub_rn(T(1), mul_rn(Q, ik))};
      const long long t = i / per, s = i % per;
#pragma unroll
      for (int e = 0; e < 6; ++e) thU[(t * 6 + e) * per + s] = th[e];
      continue;
    }
    const T q[6] = {a, c, mul_rn(two, b), mul_rn(T(-2), add_rn(mul_rn(a, mx), mul_rn(b, my))),
                    mul_rn(T(-2), add_rn(mul_rn(b, mx), mul_rn(c, my))),
                    add_rn(add_rn(mul_rn(mul_rn(a, mx), mx), mul_rn(mul_rn(mul_rn(two, b), mx), my)),
                           mul_rn(mul_rn(c, my), my))};
    const T nk = (T)(-1.0 / k);
#pragma unroll
    for (int e = 0; e < 6; ++e) {
      if (thQ) thQ[6 * i + e] = q[e];
      if (thU) thU[6 * i + e] = add_rn(mul_rn(nk, q[e]), e == 5 ? T(1) : T(0));
    }
  }
}

// (gtheta_Q, gtheta_u; either may be NULL) -> gconic[n,3], gmu[n,2] (layout 0 only).
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_theta_bwd(const T* __restrict__ conic, const T* __restrict__ mu, const T* __restrict__ origins, long long per,
                long long n, double k, const T* __restrict__ gQ, const T* __restrict__ gU, T* __restrict__ gconic,
                T* __restrict__ gmu) {
  SP_LOOP(i, n) {
    const T a = conic[3 * i], b = conic[3 * i + 1], c = conic[3 * i + 2];
    T mx = mu[2 * i], my = mu[2 * i + 1];
    if (origins) {
      mx -= origins[2 * (i / per)];
      my -= origins[2 * (i / per) + 1];
    }
    T g[6];
    const T nk = (T)(-1.0 / k);
#pragma unroll
    for (int e = 0; e < 6; ++e) g[e] = (gQ ? gQ[6 * i + e] : T(0)) + (gU ? nk * gU[6 * i + e] : T(0));
    gconic[3 * i] = g[0] + g[3] * (T(-2) * mx) + g[5] * (mx * mx);
    gconic[3 * i + 1] = T(2) * g[2] + g[3] * (T(-2) * my) + g[4] * (T(-2) * mx) + g[5] * (T(2) * mx * my);
    gconic[3 * i + 2] = g[1] + g[4] * (T(-2) * my) + g[5] * (my * my);
    gmu[2 * i] = g[3] * (T(-2) * a) + g[4] * (T(-2) * b) + g[5] * (T(2) * a * mx + T(2) * b * my);
    gmu[2 * i + 1] = g[3] * (T(-2) * b) + g[4] * (T(-2) * c) + g[5] * (T(2) * b * mx + T(2) * c * my);
  }
}

// ---- dense [P,G] products ---------------------------------------------------------------------
// quad_form (spike/forward.py:13-20): Q[p,g] = a dx^2 + 2 b dx dy + c dy^2, d = pixel - mean.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_quad_form(const T* __restrict__ px, const T* __restrict__ py, const T* __restrict__ mu,
                const T* __restrict__ conic, long long P, long long G, T* __restrict__ Q) {
  SP_LOOP(i, P * G) {
    const long long p = i / G, g = i % G;
    const T dx = px[p] - mu[2 * g], dy = py[p] - mu[2 * g + 1];
    Q[i] = conic[3 * g] * dx * dx + T(2) * conic[3 * g + 1] * dx * dy + conic[3 * g + 2] * dy * dy;
  }
}

// Q = Phi theta^T ([P,6] x [G,6]^T), the GEMM form of spike/forward.py:47-58.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_phi_theta(const T* __restrict__ Phi, const T* __restrict__ th, long long P, long long G, T* __restrict__ Q) {
  SP_LOOP(i, P * G) {
    const long long p = i / G, g = i % G;
    const T* f = Phi + 6 * p;
    const T* t = th + 6 * g;
    Q[i] = f[0] * t[0] + f[1] * t[1] + f[2] * t[2] + f[3] * t[3] + f[4] * t[4] + f[5] * t[5];
  }
}

// poly_splat_wgeo (spike/forward.py:61-66): w = max(0, 1 - Q/k)^2 * keep[g]; with gout, the
// gradient dL/dQ instead.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_poly(const T* __restrict__ Q, long long P, long long G, T k, const uint8_t* __restrict__ keep,
           const T* __restrict__ gout, T* __restrict__ out) {
  SP_LOOP(i, P * G) {
    const T u = tmax(T(1) - Q[i] / k, T(0));
    const T kp = keep ? (keep[i % G] ? T(1) : T(0)) : T(1);
    out[i] = gout ? gout[i] * kp * (T(2) * u) * (T(-1) / k) : u * u * kp;
  }
}

// Column partials of a [P,G] gradient: chunk y of the pixels, gaussian g -> NACC sums.
//   mode 0 (quad_form): ga, gb, gc, gmux, gmuy;   mode 1 (Phi theta^T): gtheta[6].
template <typename T, int MODE>
__global__ void __launch_bounds__(SP_THREADS)
    k_cols_partial(const T* __restrict__ gQ, const T* __restrict__ a0, const T* __restrict__ a1,
                   const T* __restrict__ mu, const T* __restrict__ conic, long long P, long long G, long long chunk,
                   T* __restrict__ part) {
  const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const long long p0 = (long long)blockIdx.y * chunk, p1 = p0 + chunk < P ? p0 + chunk : P;
  T acc[SP_MAX_ACC];
#pragma unroll
  for (int e = 0; e < SP_MAX_ACC; ++e) acc[e] = T(0);
  if (MODE == 0) {
    const T mx = mu[2 * g], my = mu[2 * g + 1], a = conic[3 * g], b = conic[3 * g + 1], c = conic[3 * g + 2];
    for (long long p = p0; p < p1; ++p) {
      const T gq = gQ[p * G + g];
      const T dx = a0[p] - mx, dy = a1[p] - my;
      acc[0] += gq * dx * dx;
      acc[1] += T(2) * gq * dx * dy;
      acc[2] += gq * dy * dy;
      acc[3] -= gq * (T(2) * a * dx + T(2) * b * dy);
      acc[4] -= gq * (T(2) * b * dx + T(2) * c * dy);
    }
  } else {
    for (long long p = p0; p < p1; ++p) {
      const T gq = gQ[p * G + g];
      const T* f = a0 + 6 * p;
#pragma unroll
      for (int e = 0; e < 6; ++e) acc[e] += gq * f[e];
    }
  }
#pragma unroll
  for (int e = 0; e < SP_MAX_ACC; ++e) part[((long long)blockIdx.y * G + g) * SP_MAX_ACC + e] = acc[e];
}

// Sum the chunks in chunk order; mode 0 splits into gconic[G,3] / gmu[G,2], mode 1 writes [G,6].
template <typename T, int MODE>
__global__ void __launch_bounds__(SP_THREADS)
    k_cols_sum(const T* __restrict__ part, int chunks, long long G, T* __restrict__ o0, T* __restrict__ o1) {
  SP_LOOP(g, G) {
    T acc[SP_MAX_ACC];
#pragma unroll
    for (int e = 0; e < SP_MAX_ACC; ++e) acc[e] = T(0);
    for (int y = 0; y < chunks; ++y)
#pragma unroll
      for (int e = 0; e < SP_MAX_ACC; ++e) acc[e] += part[((long long)y * G + g) * SP_MAX_ACC + e];
    if (MODE == 0) {
      o0[3 * g] = acc[0]; o0[3 * g + 1] = acc[1]; o0[3 * g + 2] = acc[2];
      o1[2 * g] = acc[3]; o1[2 * g + 1] = acc[4];
    } else {
#pragma unroll
      for (int e = 0; e < 6; ++e) o0[6 * g + e] = acc[e];
    }
  }
}

// gPhi[p,:] = sum_g gQ[p,g] theta[g,:]: a warp per pixel row, lanes over g, fixed-order butterfly.
template <typename T>
__global__ void __launch_bounds__(SP_THREADS)
    k_rows_phi(const T* __restrict__ gQ, const T* __restrict__ th, long long P, long long G, T* __restrict__ gPhi) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < P; p += warps) {
    T acc[6] = {T(0), T(0), T(0), T(0), T(0), T(0)};
    for (long long g = lane; g < G; g += 32) {
      const T gq = gQ[p * G + g];
#pragma unroll
      for (int e = 0; e < 6; ++e) acc[e] += gq * th[6 * g + e];
    }
#pragma unroll
    for (int e = 0; e < 6; ++e)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    if (lane == 0)
#pragma unroll
      for (int e = 0; e < 6; ++e) gPhi[6 * p + e] = acc[e];
  }
}

// Pixel chunks for a partials pass over G gaussians: enough blocks to fill the GPU, at most
// SP_MAX_CHUNKS.
int chunks_for(long long P, long long G) {
  const long long gb = (G + SP_THREADS - 1) / SP_THREADS;
  long long ch = (SP_REDUCE_BLOCKS + gb - 1) / gb;
  if (ch > SP_MAX_CHUNKS) ch = SP_MAX_CHUNKS;
  if (ch > P) ch = P;
  return (int)(ch < 1 ? 1 : ch);
}

// ---- host dispatch ------------------------------------------------------------------------------
int dtype_size(int dtype) { return dtype == 0 ? 4 : dtype == 1 ? 8 : 0; }

#define SP_DISPATCH(dtype, ...)                  \
  do {                                           \
    if ((dtype) == 0) {                          \
      using T = float;                           \
      __VA_ARGS__;                               \
    } else {                                     \
      using T = double;                          \
      __VA_ARGS__;                               \
    }                                            \
  } while (0)

#define SP_CHECK_DTYPE(dtype) TTS_REQUIRE((dtype) == 0 || (dtype) == 1, "dtype must be 0 (float32) or 1 (float64)")

template <typename T>
PinholeT<T> pinhole_of(const double* cam16) {
  PinholeT<T> c;
  for (int i = 0; i < 9; ++i) c.R[i] = (T)cam16[i];
  for (int i = 0; i < 3; ++i) c.t[i] = (T)cam16[9 + i];
  c.fx = (T)cam16[12]; c.fy = (T)cam16[13]; c.cx = (T)cam16[14]; c.cy = (T)cam16[15];
  return c;
}

}  // namespace
}  // namespace tts

using namespace tts;

extern "C" size_t tts_spike_workspace_bytes(long long P, long long G, int dtype) {
  if (P < 1 || G < 1 || dtype_size(dtype) == 0) return 0;
  return (size_t)chunks_for(P, G) * (size_t)G * SP_MAX_ACC * (size_t)dtype_size(dtype);
}

extern "C" int tts_quat_to_rotmat(const void* q, long long n, void* R, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(n >= 0 && (n == 0 || (q && R)), "bad quat_to_rotmat arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_quat_rotmat<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(q), n, static_cast<T*>(R))));
  return check_launch("quat_to_rotmat");
}

extern "C" int tts_quat_to_rotmat_bwd(const void* q, const void* gR, long long n, void* gq, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(n >= 0 && (n == 0 || (q && gR && gq)), "bad quat_to_rotmat_bwd arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_quat_rotmat_bwd<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(q), static_cast<const T*>(gR), n, static_cast<T*>(gq))));
  return check_launch("quat_to_rotmat_bwd");
}

extern "C" int tts_cov3d(const void* scales, const void* R, long long n, void* cov, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(n >= 0 && (n == 0 || (scales && R && cov)), "bad cov3d arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_cov3d<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(scales), static_cast<const T*>(R), n, static_cast<T*>(cov))));
  return check_launch("cov3d");
}

extern "C" int tts_cov3d_bwd(const void* scales, const void* R, const void* gcov, long long n, void* gscales,
                             void* gR, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(n >= 0 && (n == 0 || (scales && R && gcov && gscales && gR)), "bad cov3d_bwd arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_cov3d_bwd<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(scales), static_cast<const T*>(R), static_cast<const T*>(gcov), n,
                         static_cast<T*>(gscales), static_cast<T*>(gR))));
  return check_launch("cov3d_bwd");
}

extern "C" int tts_project_ewa(const void* means, const void* cov, long long G, const double* cam16, double blur,
                               double near_plane, void* mu2d, void* conic, void* depth, uint8_t* keep, int dtype,
                               void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(cam16, "null camera");
  TTS_REQUIRE(G >= 0 && (G == 0 || (means && cov && mu2d && conic && depth && keep)), "bad project_ewa arguments");
  if (G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_project_ewa<T><<<grid_for(G), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(means), static_cast<const T*>(cov), G, pinhole_of<T>(cam16), (T)blur,
                         (T)near_plane, static_cast<T*>(mu2d), static_cast<T*>(conic), static_cast<T*>(depth), keep)));
  return check_launch("project_ewa");
}

extern "C" int tts_project_ewa_bwd(const void* means, const void* cov, long long G, const double* cam16, double blur,
                                   double near_plane, const void* gmu2d, const void* gconic, const void* gdepth,
                                   void* gmeans, void* gcov, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(cam16, "null camera");
  TTS_REQUIRE(G >= 0 && (G == 0 || (means && cov && gmeans && gcov)), "bad project_ewa_bwd arguments");
  if (G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_project_ewa_bwd<T><<<grid_for(G), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(means), static_cast<const T*>(cov), G, pinhole_of<T>(cam16), (T)blur,
                         (T)near_plane, static_cast<const T*>(gmu2d), static_cast<const T*>(gconic),
                         static_cast<const T*>(gdepth), static_cast<T*>(gmeans), static_cast<T*>(gcov))));
  return check_launch("project_ewa_bwd");
}

extern "C" int tts_eval_sh(int deg, const void* coeffs, int nc, int nch, const void* dirs, long long G, int raw,
                           void* out, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(deg >= 0 && deg <= 3, "SH degree must be 0..3");
  TTS_REQUIRE(nc >= (deg + 1) * (deg + 1) && nch >= 1, "too few SH coefficients for the degree");
  TTS_REQUIRE(G >= 0 && (G == 0 || (coeffs && dirs && out)), "bad eval_sh arguments");
  if (G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_eval_sh<T><<<grid_for(G), SP_THREADS, 0, as_stream(stream)>>>(
                         deg, static_cast<const T*>(coeffs), nc, nch, static_cast<const T*>(dirs), G, raw,
                         static_cast<T*>(out))));
  return check_launch("eval_sh");
}

extern "C" int tts_eval_sh_bwd(int deg, const void* coeffs, int nc, int nch, const void* dirs, long long G, int raw,
                               const void* gout, void* gcoeffs, void* gdirs, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(deg >= 0 && deg <= 3, "SH degree must be 0..3");
  TTS_REQUIRE(nc >= (deg + 1) * (deg + 1) && nch >= 1, "too few SH coefficients for the degree");
  TTS_REQUIRE(G >= 0 && (G == 0 || (coeffs && dirs && gout && gcoeffs && gdirs)), "bad eval_sh_bwd arguments");
  if (G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_eval_sh_bwd<T><<<grid_for(G), SP_THREADS, 0, as_stream(stream)>>>(
                         deg, static_cast<const T*>(coeffs), nc, nch, static_cast<const T*>(dirs), G, raw,
                         static_cast<const T*>(gout), static_cast<T*>(gcoeffs), static_cast<T*>(gdirs))));
  return check_launch("eval_sh_bwd");
}

extern "C" int tts_color_from_dc(const void* dc, long long n, const void* gout, void* out, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(n >= 0 && (n == 0 || (dc && out)), "bad color_from_dc arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_color_dc<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(dc), n, static_cast<const T*>(gout), static_cast<T*>(out))));
  return check_launch("color_from_dc");
}

extern "C" int tts_phi(const void* px, const void* py, long long P, void* Phi, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 0 && (P == 0 || (px && py && Phi)), "bad phi arguments");
  if (P == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_phi<T><<<grid_for(P), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(px), static_cast<const T*>(py), P, static_cast<T*>(Phi))));
  return check_launch("phi");
}

extern "C" int tts_phi_bwd(const void* px, const void* py, const void* gPhi, long long P, void* gpx, void* gpy,
                           int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 0 && (P == 0 || (px && py && gPhi && gpx && gpy)), "bad phi_bwd arguments");
  if (P == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_phi_bwd<T><<<grid_for(P), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(px), static_cast<const T*>(py), static_cast<const T*>(gPhi), P,
                         static_cast<T*>(gpx), static_cast<T*>(gpy))));
  return check_launch("phi_bwd");
}

extern "C" int tts_theta_from_conic(const void* conic, const void* mu, const void* origins, long long per, long long n,
                                    double k, int layout, void* theta_Q, void* theta_u, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(k != 0.0, "k must be non-zero");
  TTS_REQUIRE(layout == 0 || layout == 1, "layout must be 0 ([n,6]) or 1 ([n/per,6,per])");
  TTS_REQUIRE(per >= 1 && (layout == 0 || n % per == 0), "rows per origin must divide n");
  TTS_REQUIRE(layout == 0 || (theta_u && !theta_Q), "layout 1 writes theta_u only");
  TTS_REQUIRE(n >= 0 && (n == 0 || (conic && mu && (theta_Q || theta_u))), "bad theta_from_conic arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_theta<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(conic), static_cast<const T*>(mu), static_cast<const T*>(origins), per,
                         n, k, layout, static_cast<T*>(theta_Q), static_cast<T*>(theta_u))));
  return check_launch("theta_from_conic");
}

extern "C" int tts_theta_from_conic_bwd(const void* conic, const void* mu, const void* origins, long long per,
                                        long long n, double k, const void* gtheta_Q, const void* gtheta_u,
                                        void* gconic, void* gmu, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(k != 0.0 && per >= 1, "bad theta_from_conic_bwd arguments");
  TTS_REQUIRE(n >= 0 && (n == 0 || (conic && mu && gconic && gmu)), "bad theta_from_conic_bwd arguments");
  if (n == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_theta_bwd<T><<<grid_for(n), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(conic), static_cast<const T*>(mu), static_cast<const T*>(origins), per,
                         n, k, static_cast<const T*>(gtheta_Q), static_cast<const T*>(gtheta_u),
                         static_cast<T*>(gconic), static_cast<T*>(gmu))));
  return check_launch("theta_from_conic_bwd");
}

extern "C" int tts_quad_form(const void* px, const void* py, const void* mu2d, const void* conic, long long P,
                             long long G, void* Q, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 0 && G >= 0 && (P * G == 0 || (px && py && mu2d && conic && Q)), "bad quad_form arguments");
  if (P * G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_quad_form<T><<<grid_for(P * G), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(px), static_cast<const T*>(py), static_cast<const T*>(mu2d),
                         static_cast<const T*>(conic), P, G, static_cast<T*>(Q))));
  return check_launch("quad_form");
}

extern "C" int tts_quad_form_bwd(const void* px, const void* py, const void* mu2d, const void* conic, const void* gQ,
                                 long long P, long long G, void* gmu2d, void* gconic, void* workspace,
                                 size_t workspace_bytes, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 1 && G >= 1 && px && py && mu2d && conic && gQ && gmu2d && gconic, "bad quad_form_bwd arguments");
  TTS_REQUIRE(workspace && workspace_bytes >= tts_spike_workspace_bytes(P, G, dtype),
              "workspace smaller than tts_spike_workspace_bytes");
  const int ch = chunks_for(P, G);
  const long long chunk = (P + ch - 1) / ch;
  const dim3 grid((unsigned)((G + SP_THREADS - 1) / SP_THREADS), (unsigned)ch);
  cudaStream_t st = as_stream(stream);
  SP_DISPATCH(dtype, ({
                k_cols_partial<T, 0><<<grid, SP_THREADS, 0, st>>>(
                    static_cast<const T*>(gQ), static_cast<const T*>(px), static_cast<const T*>(py),
                    static_cast<const T*>(mu2d), static_cast<const T*>(conic), P, G, chunk, static_cast<T*>(workspace));
                k_cols_sum<T, 0><<<grid_for(G), SP_THREADS, 0, st>>>(static_cast<const T*>(workspace), ch, G,
                                                                      static_cast<T*>(gconic), static_cast<T*>(gmu2d));
              }));
  return check_launch("quad_form_bwd");
}

extern "C" int tts_phi_theta(const void* Phi, const void* theta, long long P, long long G, void* Q, int dtype,
                             void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 0 && G >= 0 && (P * G == 0 || (Phi && theta && Q)), "bad phi_theta arguments");
  if (P * G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_phi_theta<T><<<grid_for(P * G), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(Phi), static_cast<const T*>(theta), P, G, static_cast<T*>(Q))));
  return check_launch("phi_theta");
}

extern "C" int tts_phi_theta_bwd(const void* Phi, const void* theta, const void* gQ, long long P, long long G,
                                 void* gPhi, void* gtheta, void* workspace, size_t workspace_bytes, int dtype,
                                 void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(P >= 1 && G >= 1 && Phi && theta && gQ && (gPhi || gtheta), "bad phi_theta_bwd arguments");
  cudaStream_t st = as_stream(stream);
  if (gtheta) {
    TTS_REQUIRE(workspace && workspace_bytes >= tts_spike_workspace_bytes(P, G, dtype),
                "workspace smaller than tts_spike_workspace_bytes");
    const int ch = chunks_for(P, G);
    const long long chunk = (P + ch - 1) / ch;
    const dim3 grid((unsigned)((G + SP_THREADS - 1) / SP_THREADS), (unsigned)ch);
    SP_DISPATCH(dtype, ({
                  k_cols_partial<T, 1><<<grid, SP_THREADS, 0, st>>>(static_cast<const T*>(gQ),
                                                                     static_cast<const T*>(Phi), nullptr, nullptr,
                                                                     nullptr, P, G, chunk, static_cast<T*>(workspace));
                  k_cols_sum<T, 1><<<grid_for(G), SP_THREADS, 0, st>>>(static_cast<const T*>(workspace), ch, G,
                                                                        static_cast<T*>(gtheta), nullptr);
                }));
    if (int rc = check_launch("phi_theta_bwd theta")) return rc;
  }
  if (gPhi) {
    long long blocks = (P + (SP_THREADS / 32) - 1) / (SP_THREADS / 32);
    if (blocks > SP_MAX_BLOCKS) blocks = SP_MAX_BLOCKS;
    SP_DISPATCH(dtype, (k_rows_phi<T><<<(unsigned)blocks, SP_THREADS, 0, st>>>(
                           static_cast<const T*>(gQ), static_cast<const T*>(theta), P, G, static_cast<T*>(gPhi))));
  }
  return check_launch("phi_theta_bwd");
}

extern "C" int tts_poly_splat_wgeo(const void* Q, long long P, long long G, double k, const uint8_t* keep,
                                   const void* gout, void* out, int dtype, void* stream) {
  SP_CHECK_DTYPE(dtype);
  TTS_REQUIRE(k != 0.0, "k must be non-zero");
  TTS_REQUIRE(P >= 0 && G >= 0 && (P * G == 0 || (Q && out)), "bad poly_splat_wgeo arguments");
  if (P * G == 0) return TTS_OK;
  SP_DISPATCH(dtype, (k_poly<T><<<grid_for(P * G), SP_THREADS, 0, as_stream(stream)>>>(
                         static_cast<const T*>(Q), P, G, (T)k, keep, static_cast<const T*>(gout), static_cast<T*>(out))));
  return check_launch("poly_splat_wgeo");
}
