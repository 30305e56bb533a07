// 3DGS-MCMC relocation on the device (replaces relocate + reset_adam_state, spike/mcmc.py:41-87).
//
//   1. threshold: dead_thr, or the torch.quantile of the opacities at dead_frac, found by an
//      exact MSB radix select (11/11/10-bit digits of the fp32 bit pattern, order-preserving
//      for the non-negative opacities) of the two bracketing order statistics;
//   2. per-block dead counts and alive opacity sums, one scan block, then the ascending dead
//      list and the inclusive opacity CDF over the alive set (float64);
//   3. one target per dead slot, drawn with replacement proportional to opacity (binary search
//      of a Philox uniform in the CDF) or injected; per-target occurrence counts n;
//   4. dead slots take the target's parameters (+ offset * N(0,1) on the means) and the split
//      opacity logit(o_t / (n_t + 1)); targets get the same split; Adam moments of every
//      touched gaussian are zeroed.  Steps run as separate stream-ordered kernels, so targets
//      are read before their opacity is rewritten.
#include "common.cuh"

namespace tts {

constexpr int RL_BLOCK = 1024;

struct RelocState {
  unsigned pval[2], pmask[2];
  int need[2];           // remaining rank (1-based) inside the current prefix
  float thr;
  int n_dead, n_alive;
  double total;
  int lo, hi;
  float weight;
};

__device__ __forceinline__ float opacity_of(const float* params, const ParamLayout& L, int g) {
  return sigmoidf(params[L.opacity() + g]);
}

__global__ void k_rl_init(RelocState* st, int G, float dead_thr, float dead_frac) {
  st->pval[0] = st->pval[1] = 0u;
  st->pmask[0] = st->pmask[1] = 0u;
  if (dead_frac > 0.f) {
    // torch.quantile: ranks = q * (n - 1) in the input dtype; below = long(ranks); above = ceil
    const float ranks = dead_frac * (float)(G - 1);
    st->lo = (int)ranks;
    st->hi = (int)ceilf(ranks);
    st->weight = ranks - (float)st->lo;
  } else {
    st->lo = st->hi = 0;
    st->weight = 0.f;
  }
  st->need[0] = st->lo + 1;
  st->need[1] = st->hi + 1;
  st->thr = dead_thr;
}

__global__ void __launch_bounds__(256) k_rl_hist(const float* __restrict__ params, int G, int shift, int bits,
                                                 const RelocState* __restrict__ st, int* __restrict__ hist) {
  __shared__ int sh[2][2048];
  const int nb = 1 << bits;
  for (int i = threadIdx.x; i < 2 * nb; i += blockDim.x) sh[i / nb][i % nb] = 0;
  __syncthreads();
  const ParamLayout L{G};
  const unsigned pv0 = st->pval[0], pm0 = st->pmask[0], pv1 = st->pval[1], pm1 = st->pmask[1];
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < G; g += gridDim.x * blockDim.x) {
    const unsigned b = __float_as_uint(opacity_of(params, L, g));
    const unsigned d = (b >> shift) & (unsigned)(nb - 1);
    if ((b & pm0) == pv0) atomicAdd(&sh[0][d], 1);
    if ((b & pm1) == pv1) atomicAdd(&sh[1][d], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * nb; i += blockDim.x) {
    const int c = sh[i / nb][i % nb];
    if (c) atomicAdd(hist + i, c);
  }
}

// Pick the bucket holding the needed rank for both selections: 256 threads scan 8 bins each.
__global__ void __launch_bounds__(256) k_rl_pick(RelocState* st, int* hist, int shift, int bits) {
  __shared__ int s_scan[8];
  const int nb = 1 << bits;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = nb / 256;      // 8 or 4 bins per thread
  for (int w = 0; w < 2; ++w) {
    const int need = st->need[w];   // read by every thread before the barrier below
    int loc = 0;
    for (int b = 0; b < per; ++b) loc += hist[w * nb + tid * per + b];
    int incl = loc;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) s_scan[wid] = incl;
    __syncthreads();
    int base = 0;
    for (int i = 0; i < wid; ++i) base += s_scan[i];
    const int excl = base + incl - loc;
    if (excl < need && need <= excl + loc) {
      int c = excl, b = 0;
      for (; b < per - 1; ++b) {
        if (c + hist[w * nb + tid * per + b] >= need) break;
        c += hist[w * nb + tid * per + b];
      }
      st->need[w] = need - c;
      st->pval[w] |= (unsigned)(tid * per + b) << shift;
      st->pmask[w] |= (unsigned)(nb - 1) << shift;
    }
    __syncthreads();
  }
  for (int i = tid; i < 2 * 2048; i += blockDim.x) hist[i] = 0;
}

__global__ void k_rl_thr(RelocState* st) {
  const float lo = __uint_as_float(st->pval[0]), hi = __uint_as_float(st->pval[1]);
  const float w = st->weight;
  // torch lerp: weight < 0.5 ? a + w (b - a) : b - (b - a)(1 - w)
  st->thr = w < 0.5f ? lo + w * (hi - lo) : hi - (hi - lo) * (1.f - w);
}

// Block-level dead count and alive opacity sum (double), in a fixed reduction order.
__global__ void __launch_bounds__(RL_BLOCK) k_rl_count(const float* __restrict__ params, int G,
                                                       const RelocState* __restrict__ st, int* __restrict__ bcnt,
                                                       double* __restrict__ bsum) {
  __shared__ int sc[RL_BLOCK / 32];
  __shared__ double ss[RL_BLOCK / 32];
  const ParamLayout L{G};
  const int g = blockIdx.x * RL_BLOCK + threadIdx.x;
  int dead = 0;
  double alive = 0.0;
  if (g < G) {
    const float o = opacity_of(params, L, g);
    if (o < st->thr) dead = 1;
    else alive = (double)o;
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    dead += __shfl_xor_sync(0xffffffffu, dead, d);
    alive += __shfl_xor_sync(0xffffffffu, alive, d);
  }
  if ((threadIdx.x & 31) == 0) {
    sc[threadIdx.x >> 5] = dead;
    ss[threadIdx.x >> 5] = alive;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0;
    double s = 0.0;
    for (int i = 0; i < RL_BLOCK / 32; ++i) {
      c += sc[i];
      s += ss[i];
    }
    bcnt[blockIdx.x] = c;
    bsum[blockIdx.x] = s;
  }
}

// Exclusive scan of the per-block dead counts and alive sums (one block; blocks of the
// opacity array are split into contiguous runs per thread, so the order of the sums is fixed).
__global__ void __launch_bounds__(1024) k_rl_scan(int nblk, int G, int* bcnt, double* bsum, RelocState* st,
                                                  int* n_dead_out) {
  __shared__ int sc[32];
  __shared__ double ss[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (nblk + 1023) / 1024;
  const int beg = min(nblk, tid * per), end = min(nblk, beg + per);
  int c = 0;
  double s = 0.0;
  for (int b = beg; b < end; ++b) {
    c += bcnt[b];
    s += bsum[b];
  }
  int ci = c;
  double si = s;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int yc = __shfl_up_sync(0xffffffffu, ci, d);
    const double ys = __shfl_up_sync(0xffffffffu, si, d);
    if (lane >= d) {
      ci += yc;
      si += ys;
    }
  }
  if (lane == 31) {
    sc[wid] = ci;
    ss[wid] = si;
  }
  __syncthreads();
  int cb = 0;
  double sb = 0.0;
  for (int w = 0; w < wid; ++w) {
    cb += sc[w];
    sb += ss[w];
  }
  int runc = cb + ci - c;
  double runs = sb + si - s;
  for (int b = beg; b < end; ++b) {
    const int x = bcnt[b];
    const double y = bsum[b];
    bcnt[b] = runc;
    bsum[b] = runs;
    runc += x;
    runs += y;
  }
  if (tid == 1023) {
    const int n_dead = runc;
    const int n_alive = G - n_dead;
    st->n_dead = (n_dead == 0 || n_alive == 0) ? 0 : n_dead;   // the reference moves nothing then
    st->n_alive = n_alive;
    st->total = runs;
    *n_dead_out = st->n_dead;
  }
}

__global__ void __launch_bounds__(RL_BLOCK) k_rl_lists(const float* __restrict__ params, int G,
                                                       const RelocState* __restrict__ st, const int* __restrict__ bcnt,
                                                       const double* __restrict__ bsum, int* __restrict__ dead_list,
                                                       double* __restrict__ cdf) {
  __shared__ int sc[RL_BLOCK / 32];
  __shared__ double ss[RL_BLOCK / 32];
  const ParamLayout L{G};
  const int g = blockIdx.x * RL_BLOCK + threadIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int dead = 0;
  double alive = 0.0;
  if (g < G) {
    const float o = opacity_of(params, L, g);
    if (o < st->thr) dead = 1;
    else alive = (double)o;
  }
  int ci = dead;
  double si = alive;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int yc = __shfl_up_sync(0xffffffffu, ci, d);
    const double ys = __shfl_up_sync(0xffffffffu, si, d);
    if (lane >= d) {
      ci += yc;
      si += ys;
    }
  }
  if (lane == 31) {
    sc[wid] = ci;
    ss[wid] = si;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0;
    double s = 0.0;
    for (int i = 0; i < RL_BLOCK / 32; ++i) {
      const int tc = sc[i];
      const double ts = ss[i];
      sc[i] = c;
      ss[i] = s;
      c += tc;
      s += ts;
    }
  }
  __syncthreads();
  if (g >= G) return;
  const int rank = bcnt[blockIdx.x] + sc[wid] + ci - dead;
  const double incl = bsum[blockIdx.x] + ss[wid] + si;
  if (dead) dead_list[rank] = g;
  cdf[g] = incl;
}

__global__ void k_rl_sample(const RelocState* __restrict__ st, const double* __restrict__ cdf, int G,
                            const int* __restrict__ targets_in, const int* __restrict__ step_ptr,
                            unsigned long long seed, int* __restrict__ targets, int* __restrict__ nat) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= st->n_dead) return;
  int t;
  if (targets_in) {
    t = targets_in[i];
  } else {
    const U4 r = philox4x32_10(U4{(uint32_t)i, 1u, (uint32_t)*step_ptr, 0x524cu}, (uint32_t)seed, (uint32_t)(seed >> 32));
    const double u = ((double)(r.x >> 5) * 67108864.0 + (double)(r.y >> 6)) * (1.0 / 9007199254740992.0);
    const double x = u * st->total;
    int lo = 0, hi = G - 1;   // first g with cdf[g] > x (always an alive gaussian)
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cdf[mid] > x) hi = mid;
      else lo = mid + 1;
    }
    t = lo;
  }
  targets[i] = t;
  atomicAdd(nat + t, 1);
}

__device__ __forceinline__ float split_logit(float o, int n) {
  float p = o / (float)n;
  p = fminf(fmaxf(p, 1e-6f), 1.f - 1e-6f);
  return logf(p / (1.f - p));
}

__device__ __forceinline__ void zero_moments(float* m, float* v, const ParamLayout& L, int g) {
#pragma unroll
  for (int c = 0; c < 3; c++) {
    m[L.means() + 3 * g + c] = 0.f; v[L.means() + 3 * g + c] = 0.f;
    m[L.log_scales() + 3 * g + c] = 0.f; v[L.log_scales() + 3 * g + c] = 0.f;
    m[L.color_dc() + 3 * g + c] = 0.f; v[L.color_dc() + 3 * g + c] = 0.f;
  }
#pragma unroll
  for (int c = 0; c < 4; c++) { m[L.quats() + 4 * g + c] = 0.f; v[L.quats() + 4 * g + c] = 0.f; }
  m[L.opacity() + g] = 0.f;
  v[L.opacity() + g] = 0.f;
  for (int c = 0; c < 45; c++) { m[L.color_rest() + 45 * g + c] = 0.f; v[L.color_rest() + 45 * g + c] = 0.f; }
}

// One warp per dead slot: lanes copy the 59 parameters of the target and zero the moments.
__global__ void __launch_bounds__(256)
    k_rl_apply_dead(float* __restrict__ params, float* __restrict__ m, float* __restrict__ v, int G,
                    const RelocState* __restrict__ st, const int* __restrict__ dead_list,
                    const int* __restrict__ targets, const int* __restrict__ nat, float offset,
                    const float* __restrict__ noise_in, const int* __restrict__ step_ptr, unsigned long long seed) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= st->n_dead) return;
  const ParamLayout L{G};
  const int d = dead_list[i], t = targets[i];
  // field f of the 59 per-gaussian parameters -> flat index for gaussian x
  auto at = [&](int f, int x) -> long long {
    return f < 3 ? L.means() + 3LL * x + f
         : f < 6 ? L.log_scales() + 3LL * x + (f - 3)
         : f < 10 ? L.quats() + 4LL * x + (f - 6)
         : f < 11 ? L.opacity() + (long long)x
         : f < 14 ? L.color_dc() + 3LL * x + (f - 11)
         : L.color_rest() + 45LL * x + (f - 14);
  };
  float e[3] = {0.f, 0.f, 0.f};
  if (lane < 3) {
    if (noise_in) {
      e[0] = noise_in[3 * i + lane];
    } else {
      const U4 r = philox4x32_10(U4{(uint32_t)i, 2u, (uint32_t)*step_ptr, 0x4f46u}, (uint32_t)seed, (uint32_t)(seed >> 32));
      float n3;
      box_muller(r.x, r.y, e[0], e[1]);
      box_muller(r.z, r.w, e[2], n3);
      e[0] = e[lane];
    }
  }
  for (int f = lane; f < 59; f += 32) {
    const long long src = at(f, t), dst = at(f, d);
    float val;
    if (f < 3) val = params[src] + offset * e[0];
    else if (f == 10) val = split_logit(opacity_of(params, L, t), nat[t] + 1);
    else val = params[src];
    params[dst] = val;
    m[dst] = 0.f;
    v[dst] = 0.f;
  }
}

__global__ void k_rl_apply_targets(float* __restrict__ params, float* __restrict__ m, float* __restrict__ v, int G,
                                   const int* __restrict__ nat) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  const int n = nat[g];
  if (n == 0) return;
  const ParamLayout L{G};
  params[L.opacity() + g] = split_logit(opacity_of(params, L, g), n + 1);
  zero_moments(m, v, L, g);
}

static size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

struct RelocWs {
  RelocState* st;
  int* hist;
  int* bcnt;
  double* bsum;
  int* dead_list;
  double* cdf;
  int* nat;
};

static size_t reloc_bytes(int G, RelocWs* w, char* base) {
  const int nblk = (G + RL_BLOCK - 1) / RL_BLOCK;
  size_t off = 0;
  auto take = [&](size_t n) {
    char* p = base ? base + off : nullptr;
    off += a256(n);
    return p;
  };
  char* p0 = take(sizeof(RelocState));
  char* p1 = take(2 * 2048 * 4);
  char* p2 = take((size_t)nblk * 4);
  char* p3 = take((size_t)nblk * 8);
  char* p4 = take((size_t)G * 4);
  char* p5 = take((size_t)G * 8);
  char* p6 = take((size_t)G * 4);
  if (w) {
    w->st = reinterpret_cast<RelocState*>(p0);
    w->hist = reinterpret_cast<int*>(p1);
    w->bcnt = reinterpret_cast<int*>(p2);
    w->bsum = reinterpret_cast<double*>(p3);
    w->dead_list = reinterpret_cast<int*>(p4);
    w->cdf = reinterpret_cast<double*>(p5);
    w->nat = reinterpret_cast<int*>(p6);
  }
  return off;
}

}  // namespace tts

using namespace tts;

extern "C" size_t tts_relocate_workspace_bytes(int G) { return G > 0 ? reloc_bytes(G, nullptr, nullptr) : 0; }

extern "C" int tts_relocate(float* params, float* m, float* v, int G, float dead_thr, float dead_frac, float offset,
                            const int32_t* targets_in, const float* offset_noise_in, const int32_t* step, uint64_t seed,
                            int32_t* n_dead_out, int32_t* targets_out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  TTS_REQUIRE(G >= 2, "relocation needs G >= 2");
  TTS_REQUIRE(params && m && v && step && n_dead_out && targets_out && workspace, "null pointer");
  TTS_REQUIRE(dead_frac < 1.f, "dead_frac must be < 1");
  if (workspace_bytes < tts_relocate_workspace_bytes(G)) return fail(TTS_ERR_CAPACITY, "relocation workspace too small");
  RelocWs w;
  reloc_bytes(G, &w, static_cast<char*>(workspace));
  cudaStream_t st = as_stream(stream);
  const int nblk = (G + RL_BLOCK - 1) / RL_BLOCK;
  if (cudaMemsetAsync(w.hist, 0, 2 * 2048 * 4, st) != cudaSuccess) return check_launch("memset hist");
  if (cudaMemsetAsync(w.nat, 0, (size_t)G * 4, st) != cudaSuccess) return check_launch("memset nat");
  k_rl_init<<<1, 1, 0, st>>>(w.st, G, dead_thr, dead_frac);
  if (dead_frac > 0.f) {
    const int shifts[3] = {21, 10, 0}, bits[3] = {11, 11, 10};
    const int hb = min(148 * 4, (G + 255) / 256);
    for (int d = 0; d < 3; ++d) {
      k_rl_hist<<<hb, 256, 0, st>>>(params, G, shifts[d], bits[d], w.st, w.hist);
      k_rl_pick<<<1, 256, 0, st>>>(w.st, w.hist, shifts[d], bits[d]);
    }
    k_rl_thr<<<1, 1, 0, st>>>(w.st);
  }
  k_rl_count<<<nblk, RL_BLOCK, 0, st>>>(params, G, w.st, w.bcnt, w.bsum);
  k_rl_scan<<<1, 1024, 0, st>>>(nblk, G, w.bcnt, w.bsum, w.st, n_dead_out);
  k_rl_lists<<<nblk, RL_BLOCK, 0, st>>>(params, G, w.st, w.bcnt, w.bsum, w.dead_list, w.cdf);
  k_rl_sample<<<(G + 255) / 256, 256, 0, st>>>(w.st, w.cdf, G, targets_in, step, seed, targets_out, w.nat);
  k_rl_apply_dead<<<(unsigned)(((long long)G * 32 + 255) / 256), 256, 0, st>>>(params, m, v, G, w.st, w.dead_list, targets_out, w.nat, offset,
                                                    offset_noise_in, step, seed);
  k_rl_apply_targets<<<(G + 255) / 256, 256, 0, st>>>(params, m, v, G, w.nat);
  return check_launch("relocate");
}
