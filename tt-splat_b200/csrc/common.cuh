// Shared device helpers for the tt-splat B200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <atomic>
#include <string>

#include "../../include/ttsplat_b200.h"

namespace tts {

// ---- host-side error plumbing ------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

#define TTS_REQUIRE(cond, msg)                                   \
  do {                                                           \
    if (!(cond)) return ::tts::fail(TTS_ERR_INVALID, (msg));     \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Runs `set` once per device of this process (kernel attributes such as the dynamic shared memory
// limit belong to the device context they were set in).
template <class F>
inline void once_per_device(std::atomic<unsigned long long>& done, F set) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(done.load() & bit)) {
    set();
    done.fetch_or(bit);
  }
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device status word (bounded waits that gave up record here instead of trapping).
extern __device__ int g_status;
constexpr int STATUS_MBAR_TIMEOUT = 1;

// ---- flat parameter layout (spike/model.py:28-47) ------------------------------------------
struct ParamLayout {
  int G;
  __host__ __device__ int means() const { return 0; }
  __host__ __device__ int log_scales() const { return 3 * G; }
  __host__ __device__ int quats() const { return 6 * G; }
  __host__ __device__ int opacity() const { return 10 * G; }
  __host__ __device__ int color_dc() const { return 11 * G; }
  __host__ __device__ int color_rest() const { return 14 * G; }
  __host__ __device__ int w_b_raw() const { return 59 * G; }
  __host__ __device__ long long total() const { return 59LL * G + 1; }
};

struct Cam {
  float R[9], t[3], fx, fy, cx, cy, c[3];
};

__device__ __forceinline__ Cam load_cam(const float* cams, int v) {
  Cam c;
  const float* p = cams + v * TTS_CAM_FLOATS;
#pragma unroll
  for (int i = 0; i < 9; i++) c.R[i] = __ldg(p + i);
#pragma unroll
  for (int i = 0; i < 3; i++) c.t[i] = __ldg(p + 9 + i);
  c.fx = __ldg(p + 12); c.fy = __ldg(p + 13); c.cx = __ldg(p + 14); c.cy = __ldg(p + 15);
#pragma unroll
  for (int i = 0; i < 3; i++) c.c[i] = __ldg(p + 16 + i);
  return c;
}

// torch.nn.functional.softplus(beta=1, threshold=20) and its derivative.
__device__ __forceinline__ float softplusf(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) {
  if (x > 20.f) return 1.f;
  float z = expf(x);
  return z / (z + 1.f);
}
__device__ __forceinline__ float sigmoidf(float x) { return 1.f / (1.f + expf(-x)); }

// ---- bounded mbarrier + bulk copy (1-D TMA, one destination CTA) -------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` with an iteration limit; on timeout record the status and report
// false.  try_wait itself suspends for a hardware-defined interval, so the limit is ~seconds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (int it = 0; it < (1 << 22); ++it)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_status, STATUS_MBAR_TIMEOUT);
  // A CTA must not exit while its bulk copy may still write into its shared memory (the next
  // CTA on the SM would receive that memory): wait once more, again with a limit, for the copy
  // in flight before the caller abandons the tile.
  for (int it = 0; it < (1 << 22); ++it)
    if (mbar_try_wait(bar, parity)) break;
  return false;
}

// ---- Philox4x32-10 (Salmon et al., SC'11 "Parallel random numbers: as easy as 1, 2, 3") ----
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox4x32_10(U4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    U4 n;
    n.x = hi1 ^ ctr.y ^ k0;
    n.y = lo1;
    n.z = hi0 ^ ctr.w ^ k1;
    n.w = lo0;
    ctr = n;
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}
// x / 255 for a byte x, correctly rounded (the [0, 1] float of an 8-bit pixel, equal to numpy's
// float32(x) / float32(255)): the product with fp32(1/255) and one Newton-style correction through
// the exact fma residual, which an exhaustive check over the 256 bytes shows to round correctly
// (the product alone is off by one ulp for 126 of them).
__device__ __forceinline__ float unit_from_byte(unsigned x) {
  const float xf = (float)x, r = 1.0f / 255.0f;
  const float q = __fmul_rn(xf, r);
  const float e = __fmaf_rn(-q, 255.0f, xf);
  return __fmaf_rn(e, r, q);
}

// Uniform in (0, 1] from 32 random bits (never 0, so log() is finite).
__device__ __forceinline__ float u01(uint32_t b) { return (float)(b >> 8) * (1.0f / 16777216.0f) + (0.5f / 16777216.0f); }
// Uniform in [0, 1).
__device__ __forceinline__ float u01_open(uint32_t b) { return (float)(b >> 8) * (1.0f / 16777216.0f); }
// Box-Muller: two standard normals from two uniforms.
__device__ __forceinline__ void box_muller(uint32_t a, uint32_t b, float& n0, float& n1) {
  float r = sqrtf(-2.0f * logf(u01(a)));
  float s, c;
  sincospif(2.0f * u01_open(b), &s, &c);
  n0 = r * c;
  n1 = r * s;
}

// Whether a slot's weight max(u, 0)^2 is exactly zero at every pixel centre of the tile, so that
// the tile kernels may skip it without changing a bit.  u = theta . Phi is a concave quadratic for
// the positive-definite conics of the projection; the region u > -m, with m = 1e-6 x the sum of
// the terms' magnitudes over the tile (far above the rounding of the kernels' fp32 evaluation of u,
// at most ~3e-7 of that sum), is an ellipse, and when its bounding box misses the box of pixel
// centres [0.5, 15.5]^2 every evaluated u there is negative.  Evaluated in double; anything else
// (a degenerate or non-finite row) counts as live.
__device__ __forceinline__ bool slot_dead(float t0, float t1, float t2, float t3, float t4, float t5) {
  const double A = t0, B = t1, C = t2, D = t3, E = t4, F = t5;
  const double det = 4.0 * A * B - C * C;
  if (!(A < 0.0 && B < 0.0 && det > 0.0)) return false;
  // the peak (xs, ys) = (XN, YN) / det and everything below scaled by det > 0 (no division)
  const double XN = C * E - 2.0 * B * D, YN = C * D - 2.0 * A * E;
  const double M = (fabs(A) + fabs(B) + fabs(C)) * 240.25 + (fabs(D) + fabs(E)) * 15.5 + fabs(F);
  const double umd = (F + 1e-6 * M) * det + 0.5 * (D * XN + E * YN);   // (peak of u above -m) * det
  if (!(umd > 0.0)) return umd <= 0.0;
  const double rx = -4.0 * B * umd, ry = -4.0 * A * umd;   // squared half-extents * det^2
  const double lo = 0.5 * det, hi = 15.5 * det;
  return (XN < lo && (lo - XN) * (lo - XN) > rx) || (XN > hi && (XN - hi) * (XN - hi) > rx) ||
         (YN < lo && (lo - YN) * (lo - YN) > ry) || (YN > hi && (YN - hi) * (YN - hi) > ry);
}

// ---- packed FP32 pairs (sm_100a .f32x2 arithmetic: two IEEE fp32 lanes per instruction) ----
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 mk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void split2(f32x2 a, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a));
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a * b + c, 0) per lane where the exact result is at most 1: the fused multiply-add
// saturated to [0, 1] (fma.rn.sat.f32 on each lane; the packed form has no .sat), two issue
// slots instead of a packed FMA and two max operations.
__device__ __forceinline__ f32x2 fma_sat2(f32x2 a, f32x2 b, float c) {
  float alo, ahi, blo, bhi, lo, hi;
  split2(a, alo, ahi);
  split2(b, blo, bhi);
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(lo) : "f"(alo), "f"(blo), "f"(c));
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(hi) : "f"(ahi), "f"(bhi), "f"(c));
  return mk2(lo, hi);
}
__device__ __forceinline__ f32x2 relu2(f32x2 a) {
  float lo, hi;
  split2(a, lo, hi);
  return mk2(fmaxf(lo, 0.f), fmaxf(hi, 0.f));
}
__device__ __forceinline__ float hsum2(f32x2 a) {
  float lo, hi;
  split2(a, lo, hi);
  return lo + hi;
}

}  // namespace tts
