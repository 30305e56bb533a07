// 3DGS-MCMC relocation on the device (replaces relocate + reset_adam_state, spike/mcmc.py:41-87).
//
// One cooperative kernel (all blocks co-resident; phases separated by a grid barrier whose
// wait is bounded) over contiguous per-block ranges of the gaussians:
//   1. threshold: dead_thr, or the torch.quantile of the opacities at dead_frac, found by an
//      exact MSB radix select (11/11/10-bit digits of the fp32 bit pattern, order-preserving
//      for the non-negative opacities) of the two bracketing order statistics; every block
//      reads the merged digit histogram and picks the same bucket; the members of the first
//      digit's buckets (up to SEL_CAP) are then listed once, and every block selects the last two
//      digits among them in shared memory;
//   2. per-block dead counts and alive opacity sums; each block sums its predecessors in block
//      order and writes its part of the ascending dead list and of the inclusive opacity CDF
//      over the alive set (float64, one fixed summation order);
//   3. one target per dead slot, drawn with replacement proportional to opacity (binary search
//      of a Philox uniform in the CDF) or injected; per-target occurrence counts n;
//   4. dead slots take the target's parameters (+ offset * N(0,1) on the means) and the split
//      opacity logit(o_t / (n_t + 1)), from the target's logit saved in phase 3; in the same
//      phase the targets get the same split; Adam moments of every touched gaussian are zeroed.
#include <algorithm>

#include "peer.cuh"
#include "sgld.cuh"

namespace tts {

constexpr int RK_THREADS = 512;
// Members of the buckets that the first (11-bit) digit of the quantile select picks, held in
// shared memory so that the last two digits need no grid barrier; more members take the
// grid-wide passes.
constexpr int SEL_CAP = 6144;
constexpr int STATUS_GRID_TIMEOUT = 2;

struct GridBar {
  unsigned count, gen;
};

__device__ __forceinline__ float opacity_of(const float* params, const ParamLayout& L, int g) {
  return sigmoidf(params[L.opacity() + g]);
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned x) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(x) : "memory");
  return old;
}
__device__ __forceinline__ void red_add_release_gpu(unsigned* p, unsigned x) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(x) : "memory");
}

// Grid-wide barrier for a cooperative launch: thread 0 of each block arrives with an acq_rel
// increment (its release covers the block's writes, ordered before it by the block barrier); the
// last to arrive resets the count and bumps the generation with a release, which the others
// acquire while they poll, with an iteration limit (on timeout the status word records it and the
// kernel unwinds: every later barrier also gives up).  The generation is read before arriving, so
// a fast last arriver cannot bump it unseen.
__device__ __forceinline__ bool grid_sync(GridBar* bar, unsigned nblocks, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned gen = ld_acquire_gpu(&bar->gen);
    const unsigned arrived = atom_add_acq_rel_gpu(&bar->count, 1u);
    int ok = 1;
    if (arrived == nblocks - 1) {
      bar->count = 0u;
      red_add_release_gpu(&bar->gen, 1u);
    } else {
      int it = 0;
      while (ld_acquire_gpu(&bar->gen) == gen) {
        if (++it > (1 << 24)) {
          ok = 0;
          atomicOr(&g_status, STATUS_GRID_TIMEOUT);
          break;
        }
        __nanosleep(32);
      }
    }
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

// Block-wide inclusive scan of (int, double) pairs in thread order; returns the block totals.
struct ScanPair {
  int c;
  double s;
};
__device__ __forceinline__ ScanPair block_incl_scan(int c, double x, int& ci, double& si, ScanPair* s_w) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  ci = c;
  si = x;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int yc = __shfl_up_sync(0xffffffffu, ci, d);
    const double ys = __shfl_up_sync(0xffffffffu, si, d);
    if (lane >= d) {
      ci += yc;
      si += ys;
    }
  }
  if (lane == 31) s_w[wid] = ScanPair{ci, si};
  __syncthreads();
  int cb = 0;
  double sb = 0.0;
  for (int w = 0; w < wid; ++w) {
    cb += s_w[w].c;
    sb += s_w[w].s;
  }
  ci += cb;
  si += sb;
  ScanPair tot{0, 0.0};
  for (int w = 0; w < RK_THREADS / 32; ++w) {
    tot.c += s_w[w].c;
    tot.s += s_w[w].s;
  }
  __syncthreads();
  return tot;
}

struct RelocArgs {
  float* params;
  float* m;
  float* v;
  int G;
  float dead_thr, dead_frac, offset;
  const int* targets_in;
  const float* noise_in;
  const int* step_ptr;
  unsigned long long seed;
  int* n_dead_out;
  int* targets;
  GridBar* bar;
  int* hist;        // [3 passes][2 selections][2048]
  int* sel_count;   // members of the first digit's buckets (zeroed with the histograms)
  unsigned* sel_list;   // [SEL_CAP] their opacity bit patterns
  int* bcnt;        // [nblocks]
  double* bsum;     // [nblocks]
  int* dead_list;   // [G]
  double* cdf;      // [G]
  int* nat;         // [G], zeroed by the kernel (phase 0)
  float* old_logit;  // [G] target opacity logit of each dead slot before the split
  const double* sgld_lr;   // non-null: the SGLD step runs as phase 0 (lr of the means at [0])
  float noise_lr;
  const float* sgld_eps;   // injected SGLD noise [G][3], or null for Philox draws
  const int* peer_mine;    // non-null (multi-GPU step): wait for every rank's phase-1 flag first
  int peer_n;
};

__device__ __forceinline__ long long field_index(const ParamLayout& L, int f, int x) {
  return f < 3 ? L.means() + 3LL * x + f
       : f < 6 ? L.log_scales() + 3LL * x + (f - 3)
       : f < 10 ? L.quats() + 4LL * x + (f - 6)
       : f < 11 ? L.opacity() + (long long)x
       : f < 14 ? L.color_dc() + 3LL * x + (f - 11)
       : L.color_rest() + 45LL * x + (f - 14);
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

__global__ void __launch_bounds__(RK_THREADS) k_relocate(RelocArgs a) {
  __shared__ __align__(16) int sh[2][2048];
  __shared__ ScanPair s_w[RK_THREADS / 32];
  __shared__ int s_flag;
  __shared__ unsigned s_pval[2], s_pmask[2];
  __shared__ int s_need[2];
  __shared__ int s_pick[2][2];     // (bucket, rank consumed before it) per selection
  __shared__ unsigned s_list[SEL_CAP];
  const ParamLayout L{a.G};
  const int G = a.G, tid = threadIdx.x;
  const unsigned nb = gridDim.x;
  const int chunk = (G + (int)nb - 1) / (int)nb;
  const int beg = min(G, (int)blockIdx.x * chunk), end = min(G, beg + chunk);
  const int step = *a.step_ptr;
  if (a.peer_mine) {
    // multi-GPU step: every rank's shard of the update must have arrived (phase 1) before this
    // rank's parameters are read; a block whose wait gave up leaves (status recorded), and the
    // others then give up at the next grid barrier
    if (tid == 0) s_flag = peer_wait(a.peer_mine, a.peer_n, 1, step) ? 1 : 0;
    __syncthreads();
    if (!s_flag) return;
  }
  // ---- 0. the per-target counts of this block's range start at zero; with sgld_lr, the SGLD step
  // of this block's gaussians (add_sgld_noise right before relocate, spike/mcmc.py:97-111): it
  // changes only the means, which nothing reads before the copies of phase 4, grid barriers later
  for (int g = beg + tid; g < end; g += RK_THREADS) a.nat[g] = 0;
  if (a.sgld_lr) {
    const double lr_means = a.sgld_lr[0];
    for (int g = beg + tid; g < end; g += RK_THREADS)
      sgld_one(a.params, L, g, lr_means, a.noise_lr, a.sgld_eps, step, a.seed);
  }
  // ---- 1. threshold ----------------------------------------------------------------------------
  float thr = a.dead_thr;
  if (a.dead_frac > 0.f) {
    // torch.quantile: ranks = q * (n - 1) in the input dtype; below = long(ranks); above = ceil
    const float ranks = a.dead_frac * (float)(G - 1);
    const int lo = (int)ranks, hi = (int)ceilf(ranks);
    const float weight = ranks - (float)lo;
    if (tid < 2) {
      s_pval[tid] = 0u;
      s_pmask[tid] = 0u;
      s_need[tid] = (tid == 0 ? lo : hi) + 1;
    }
    const int shifts[3] = {21, 10, 0}, bits[3] = {11, 11, 10};
    int m_list = -1;   // >= 0: the last two digits select among the s_list members
    for (int d = 0; d < 3; ++d) {
      const int nbins = 1 << bits[d];
      for (int i = tid; i < 2 * 2048; i += RK_THREADS) sh[i >> 11][i & 2047] = 0;
      __syncthreads();
      const unsigned pv0 = s_pval[0], pm0 = s_pmask[0], pv1 = s_pval[1], pm1 = s_pmask[1];
      const int* h0 = &sh[0][0];
      const int* h1 = &sh[1][0];
      if (m_list >= 0) {
        // every block histograms the same member list in its own shared memory
        for (int i = tid; i < m_list; i += RK_THREADS) {
          const unsigned b = s_list[i];
          const unsigned dg = (b >> shifts[d]) & (unsigned)(nbins - 1);
          if ((b & pm0) == pv0) atomicAdd(&sh[0][dg], 1);
          if ((b & pm1) == pv1) atomicAdd(&sh[1][dg], 1);
        }
        __syncthreads();
      } else {
        for (int g = beg + tid; g < end; g += RK_THREADS) {
          const unsigned b = __float_as_uint(opacity_of(a.params, L, g));
          const unsigned dg = (b >> shifts[d]) & (unsigned)(nbins - 1);
          if ((b & pm0) == pv0) atomicAdd(&sh[0][dg], 1);
          if ((b & pm1) == pv1) atomicAdd(&sh[1][dg], 1);
        }
        __syncthreads();
        int* gh = a.hist + d * 2 * 2048;
        for (int i = tid; i < 2 * nbins; i += RK_THREADS) {
          const int w = i / nbins, bin = i - w * nbins;
          const int c = sh[w][bin];
          if (c) atomicAdd(gh + w * 2048 + bin, c);
        }
        if (!grid_sync(a.bar, nb, &s_flag)) return;
        h0 = gh;
        h1 = gh + 2048;
      }
      // every block picks the same buckets from the merged histogram: both selections in one
      // block scan (the second one's counts carried exactly in the scan's double)
      {
        const int per = nbins / RK_THREADS;        // 4 or 2 bins per thread
        const bool glob = m_list < 0;
        int c0[4], c1[4], loc0 = 0, loc1 = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          c0[q] = q < per ? (glob ? __ldcg(h0 + tid * per + q) : h0[tid * per + q]) : 0;
          c1[q] = q < per ? (glob ? __ldcg(h1 + tid * per + q) : h1[tid * per + q]) : 0;
          loc0 += c0[q];
          loc1 += c1[q];
        }
        int ci;
        double si;
        block_incl_scan(loc0, (double)loc1, ci, si, s_w);
        const int incl[2] = {ci, (int)si}, loc[2] = {loc0, loc1};
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int need = s_need[w], excl = incl[w] - loc[w];
          if (excl < need && need <= incl[w]) {
            // the first of this thread's bins that reaches need (unrolled: the counts stay in
            // registers)
            int c = excl, q = 0;
            bool found = false;
#pragma unroll
            for (int qq = 0; qq < 3; ++qq) {
              if (!found && qq < per - 1) {
                const int h = w ? c1[qq] : c0[qq];
                if (c + h >= need) {
                  found = true;
                } else {
                  c += h;
                  q = qq + 1;
                }
              }
            }
            s_pick[w][0] = tid * per + q;
            s_pick[w][1] = c;
          }
        }
        __syncthreads();
        if (tid < 2) {
          s_need[tid] -= s_pick[tid][1];
          s_pval[tid] |= (unsigned)s_pick[tid][0] << shifts[d];
          s_pmask[tid] |= (unsigned)(nbins - 1) << shifts[d];
        }
        __syncthreads();
      }
      if (d == 0) {
        // the members of the two chosen buckets go to one list (opacity bits; the order of the
        // appends does not matter, the selection depends only on the values)
        const unsigned qv0 = s_pval[0], qm0 = s_pmask[0], qv1 = s_pval[1], qm1 = s_pmask[1];
        const int lane = tid & 31;
        for (int base = beg; base < end; base += RK_THREADS) {
          const int g = base + tid;
          unsigned b = 0u;
          bool mem = false;
          if (g < end) {
            b = __float_as_uint(opacity_of(a.params, L, g));
            mem = (b & qm0) == qv0 || (b & qm1) == qv1;
          }
          const unsigned bal = __ballot_sync(0xffffffffu, mem);
          int pos = 0;
          if (lane == 0 && bal) pos = atomicAdd(a.sel_count, __popc(bal));
          pos = __shfl_sync(0xffffffffu, pos, 0) + __popc(bal & ((1u << lane) - 1u));
          if (mem && pos < SEL_CAP) a.sel_list[pos] = b;
        }
        if (!grid_sync(a.bar, nb, &s_flag)) return;
        const int mc = __ldcg(a.sel_count);   // the same in every block
        if (mc <= SEL_CAP) {
          for (int i = tid; i < mc; i += RK_THREADS) s_list[i] = __ldcg(a.sel_list + i);
          m_list = mc;
          __syncthreads();
        }
      }
    }
    const float olo = __uint_as_float(s_pval[0]), ohi = __uint_as_float(s_pval[1]);
    // torch lerp: weight < 0.5 ? a + w (b - a) : b - (b - a)(1 - w)
    thr = weight < 0.5f ? olo + weight * (ohi - olo) : ohi - (ohi - olo) * (1.f - weight);
  }
  // ---- 2. counts, dead list, CDF ----------------------------------------------------------------
  // block totals: tiles of RK_THREADS in ascending order, each by the same block scan that the
  // list pass repeats (so a block's last CDF entry equals its total bit for bit)
  int bc = 0;
  double bs = 0.0;
  for (int base = beg; base < end; base += RK_THREADS) {
    const int g = base + tid;
    int dead = 0;
    double alive = 0.0;
    if (g < end) {
      const float o = opacity_of(a.params, L, g);
      if (o < thr) dead = 1;
      else alive = (double)o;
    }
    int ci;
    double si;
    const ScanPair t = block_incl_scan(dead, alive, ci, si, s_w);
    bc += t.c;
    bs += t.s;
  }
  if (tid == 0) {
    a.bcnt[blockIdx.x] = bc;
    a.bsum[blockIdx.x] = bs;
  }
  if (!grid_sync(a.bar, nb, &s_flag)) return;
  // predecessors (in block order) and the totals, summed identically by every block: the
  // per-block values are fetched in parallel, then added in block order by one thread
  int* s_bc = &sh[0][0];
  double* s_bs = reinterpret_cast<double*>(&sh[1][0]);       // nb <= 1024 doubles fit in sh[1]
  for (unsigned b = tid; b < nb; b += RK_THREADS) {
    s_bc[b] = __ldcg(a.bcnt + b);
    s_bs[b] = __ldcg(a.bsum + b);
  }
  __syncthreads();
  if (tid == 0) {
    int c = 0, cpre = 0;
    double s = 0.0, spre = 0.0;
    for (unsigned b = 0; b < nb; ++b) {
      if (b == blockIdx.x) {
        cpre = c;
        spre = s;
      }
      c += s_bc[b];
      s += s_bs[b];
    }
    s_w[0] = ScanPair{cpre, spre};
    s_w[1] = ScanPair{c, s};
  }
  __syncthreads();
  int runc = s_w[0].c;
  const double spre = s_w[0].s;
  double runs = 0.0;     // in-block running sum, associated like the block total above
  const int n_dead_all = s_w[1].c;
  const double total = s_w[1].s;
  __syncthreads();
  const int n_alive = G - n_dead_all;
  const int n_dead = (n_dead_all == 0 || n_alive == 0) ? 0 : n_dead_all;   // the reference moves nothing then
  if (blockIdx.x == 0 && tid == 0) *a.n_dead_out = n_dead;
  if (n_dead == 0) return;            // uniform across the grid
  for (int base = beg; base < end; base += RK_THREADS) {
    const int g = base + tid;
    int dead = 0;
    double alive = 0.0;
    if (g < end) {
      const float o = opacity_of(a.params, L, g);
      if (o < thr) dead = 1;
      else alive = (double)o;
    }
    int ci;
    double si;
    const ScanPair t = block_incl_scan(dead, alive, ci, si, s_w);
    if (g < end) {
      if (dead) a.dead_list[runc + ci - 1] = g;
      // spre + (in-block inclusive sum): the block's last entry is spre + its total, the next
      // block's prefix exactly, and the grid's last entry equals the total
      a.cdf[g] = spre + (runs + si);
    }
    runc += t.c;
    runs += t.s;
  }
  if (!grid_sync(a.bar, nb, &s_flag)) return;
  // ---- 3. targets: one warp per dead slot; the CDF search splits the range 33 ways per round
  // (32 pivots loaded at once), so a search takes ~log33(G) dependent loads instead of log2(G)
  const int lane = tid & 31;
  const int nwarps = (int)nb * (RK_THREADS / 32);
  for (int i = blockIdx.x * (RK_THREADS / 32) + (tid >> 5); i < n_dead; i += nwarps) {
    int t;
    if (a.targets_in) {
      t = a.targets_in[i];
    } else {
      const U4 r = philox4x32_10(U4{(uint32_t)i, 1u, (uint32_t)step, 0x524cu}, (uint32_t)a.seed,
                                 (uint32_t)(a.seed >> 32));
      const double u = ((double)(r.x >> 5) * 67108864.0 + (double)(r.y >> 6)) * (1.0 / 9007199254740992.0);
      double x = u * total;
      if (x >= total) x = nextafter(total, 0.0);   // u < 1, but the product can round up
      // first g with cdf[g] > x (always an alive gaussian): the answer lies in [lo, hi)
      int lo = 0, hi = G;
      while (hi - lo > 32) {
        const long long span = hi - lo;
        const int piv = lo + (int)(span * (lane + 1) / 33);
        const unsigned bal = __ballot_sync(0xffffffffu, __ldcg(a.cdf + piv) > x);
        const int f = bal ? __ffs(bal) - 1 : 32;
        const int nlo = f > 0 ? lo + (int)(span * f / 33) + 1 : lo;
        const int nhi = f < 32 ? lo + (int)(span * (f + 1) / 33) + 1 : hi;
        lo = nlo;
        hi = nhi;
      }
      const int gq = lo + lane;
      const unsigned bal = __ballot_sync(0xffffffffu, gq < hi && __ldcg(a.cdf + gq) > x);
      t = bal ? lo + __ffs(bal) - 1 : hi - 1;
    }
    if (lane == 0) {
      a.targets[i] = t;
      a.old_logit[i] = a.params[L.opacity() + t];   // before any split of this launch
      atomicAdd(a.nat + t, 1);
    }
  }
  if (!grid_sync(a.bar, nb, &s_flag)) return;
  // ---- 4. dead slots and targets in one phase (disjoint gaussians: targets are alive) ----------
  // 4a. dead slots: one warp per slot copies the target's 59 parameters, the opacity split from
  // the target's logit saved in phase 3 (4b may already have split the target's own)
  for (int i = blockIdx.x * (RK_THREADS / 32) + (tid >> 5); i < n_dead; i += nwarps) {
    const int d = __ldcg(a.dead_list + i), t = __ldcg(a.targets + i);
    float e = 0.f;
    if (lane < 3) {
      if (a.noise_in) {
        e = a.noise_in[3 * i + lane];
      } else {
        const U4 r = philox4x32_10(U4{(uint32_t)i, 2u, (uint32_t)step, 0x4f46u}, (uint32_t)a.seed,
                                   (uint32_t)(a.seed >> 32));
        float n0, n1, n2, n3;
        box_muller(r.x, r.y, n0, n1);
        box_muller(r.z, r.w, n2, n3);
        e = lane == 0 ? n0 : lane == 1 ? n1 : n2;
      }
    }
    const int nt = __ldcg(a.nat + t);
    for (int f = lane; f < 59; f += 32) {
      const long long src = field_index(L, f, t), dst = field_index(L, f, d);
      float val;
      if (f < 3) val = a.params[src] + a.offset * e;
      else if (f == 10) val = split_logit(sigmoidf(__ldcg(a.old_logit + i)), nt + 1);
      else val = a.params[src];
      a.params[dst] = val;
      a.m[dst] = 0.f;
      a.v[dst] = 0.f;
    }
  }
  // 4b. targets: split opacity, zero moments
  for (int g = beg + tid; g < end; g += RK_THREADS) {
    const int n = __ldcg(a.nat + g);
    if (n == 0) continue;
    a.params[L.opacity() + g] = split_logit(opacity_of(a.params, L, g), n + 1);
    zero_moments(a.m, a.v, L, g);
  }
}

static size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

static int reloc_grid() {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k_relocate, RK_THREADS, 0);
  int n = sms * (per > 2 ? 2 : per);      // co-resident by construction; two blocks per SM at most
  if (n < 1) n = 1;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

static size_t reloc_bytes(int G, int nblk, RelocArgs* w, char* base) {
  size_t off = 0;
  auto take = [&](size_t n) {
    char* p = base ? base + off : nullptr;
    off += a256(n);
    return p;
  };
  char* p0 = take(sizeof(GridBar));
  char* p1 = take(3 * 2 * 2048 * 4 + 4);    // + the bucket-member count
  char* p7 = take((size_t)SEL_CAP * 4);
  char* p2 = take((size_t)nblk * 4);
  char* p3 = take((size_t)nblk * 8);
  char* p4 = take((size_t)G * 4);
  char* p5 = take((size_t)G * 8);
  char* p6 = take((size_t)G * 4);
  char* p8 = take((size_t)G * 4);
  if (w) {
    w->bar = reinterpret_cast<GridBar*>(p0);
    w->hist = reinterpret_cast<int*>(p1);
    w->sel_count = reinterpret_cast<int*>(p1) + 3 * 2 * 2048;
    w->sel_list = reinterpret_cast<unsigned*>(p7);
    w->old_logit = reinterpret_cast<float*>(p8);
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

// Sized for up to 1024 blocks, more than any grid reloc_grid() returns.
extern "C" size_t tts_relocate_workspace_bytes(int G) { return G > 0 ? reloc_bytes(G, 1024, nullptr, nullptr) : 0; }

static int relocate_core(float* params, float* m, float* v, int G, float dead_thr, float dead_frac, float offset,
                         const int32_t* targets_in, const float* offset_noise_in, const int32_t* step, uint64_t seed,
                         int32_t* n_dead_out, int32_t* targets_out, const double* sgld_lr, float noise_lr,
                         const float* sgld_eps, const int32_t* peer_mine, int peer_n, void* workspace,
                         size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(G >= 2, "relocation needs G >= 2");
  TTS_REQUIRE(params && m && v && step && n_dead_out && targets_out && workspace, "null pointer");
  TTS_REQUIRE(dead_frac < 1.f, "dead_frac must be < 1");
  if (workspace_bytes < tts_relocate_workspace_bytes(G)) return fail(TTS_ERR_CAPACITY, "relocation workspace too small");
  RelocArgs a;
  const int nblk = std::min(reloc_grid(), 1024);
  reloc_bytes(G, 1024, &a, static_cast<char*>(workspace));
  a.params = params;
  a.m = m;
  a.v = v;
  a.G = G;
  a.dead_thr = dead_thr;
  a.dead_frac = dead_frac;
  a.offset = offset;
  a.targets_in = targets_in;
  a.noise_in = offset_noise_in;
  a.step_ptr = step;
  a.seed = seed;
  a.n_dead_out = n_dead_out;
  a.targets = targets_out;
  a.sgld_lr = sgld_lr;
  a.noise_lr = noise_lr;
  a.sgld_eps = sgld_eps;
  a.peer_mine = peer_mine;
  a.peer_n = peer_n;
  cudaStream_t st = as_stream(stream);
  // the barrier word, the digit histograms and the bucket-member count start at zero (the
  // per-target counts are zeroed by the kernel)
  const size_t head = reinterpret_cast<char*>(a.sel_list) - static_cast<char*>(workspace);
  if (cudaMemsetAsync(workspace, 0, head, st) != cudaSuccess) return check_launch("memset relocation state");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nblk);
  cfg.blockDim = dim3(RK_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_relocate, a) != cudaSuccess) return check_launch("relocate (cooperative launch)");
  return check_launch("relocate");
}

extern "C" int tts_relocate(float* params, float* m, float* v, int G, float dead_thr, float dead_frac, float offset,
                            const int32_t* targets_in, const float* offset_noise_in, const int32_t* step, uint64_t seed,
                            int32_t* n_dead_out, int32_t* targets_out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  return relocate_core(params, m, v, G, dead_thr, dead_frac, offset, targets_in, offset_noise_in, step, seed,
                       n_dead_out, targets_out, nullptr, 0.f, nullptr, nullptr, 0, workspace, workspace_bytes,
                       stream);
}

extern "C" int tts_sgld_relocate(float* params, float* m, float* v, int G, const double* lr7, float noise_lr,
                                 const float* eps_noise, float dead_thr, float dead_frac, float offset,
                                 const int32_t* targets_in, const float* offset_noise_in, const int32_t* step,
                                 uint64_t seed, int32_t* n_dead_out, int32_t* targets_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(lr7, "null learning-rate table");
  return relocate_core(params, m, v, G, dead_thr, dead_frac, offset, targets_in, offset_noise_in, step, seed,
                       n_dead_out, targets_out, lr7, noise_lr, eps_noise, nullptr, 0, workspace, workspace_bytes,
                       stream);
}

extern "C" int tts_peer_sgld_relocate(float* params, float* m, float* v, int G, const double* lr7, float noise_lr,
                                      const float* eps_noise, float dead_thr, float dead_frac, float offset,
                                      const int32_t* step, uint64_t seed, int32_t* n_dead_out, int32_t* targets_out,
                                      int32_t* const* flags, int rank, int N, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  TTS_REQUIRE(lr7 && flags && N >= 1 && N <= PEER_MAX && rank >= 0 && rank < N && flags[rank],
              "bad peer SGLD + relocation arguments");
  return relocate_core(params, m, v, G, dead_thr, dead_frac, offset, nullptr, nullptr, step, seed, n_dead_out,
                       targets_out, lr7, noise_lr, eps_noise, flags[rank], N, workspace, workspace_bytes, stream);
}
