// Spatial-hash binning (replaces assign_bins, tools/m4_train_binned.py:75-127).
//
// Each kept gaussian scatters to one home cell (cell size = tile size = 16 px); each 16x16
// tile gathers the candidates of its (2R+1)^2 neighbour cells, keys them exactly as the
// reference (tile-local key q = clamp(long(dist2), 0, 2047) with dist2 in fp32, no FMA
// contraction), and keeps the K smallest of (q, stencil offset j, gaussian id) in ascending
// order — the stable order of the reference's packed sort key.  A warp per tile selects and
// sorts up to WCAP candidates in shared memory (32-bit keys when ids and stencil offsets fit
// them, else 64-bit); a block per tile takes larger candidate sets, with an MSB radix select
// over the 51-bit key (digits q | j | g) until at most SORT_CAP keys remain to sort.
// The epilogue writes idx/count/cand, the stencil-indexed inverse table used by the
// deterministic slot->gaussian reduction, and (optionally) the packed slot rows
// theta_u[6] | color_o[3] | o_col of _operands (:207-211, theta_u_gathered :130-143).
#include <mutex>
#include <string>

#include "common.cuh"

namespace tts {

constexpr int BS_THREADS = 512;
constexpr int BS_CAP = 8192;           // keys held in (dynamic) shared memory: 64 KB
constexpr int SORT_CAP = 1024;         // keys the block sorts after its radix select
constexpr int BS_MAXS = 49;  // (2R+1)^2 for R <= 3
typedef unsigned long long u64;

// Home cell coordinate: clamp(long(floor(m/16)), 0, n-1) with torch's conversion of
// non-finite / out-of-range values to INT64_MIN (which then clamps to 0).
__device__ __forceinline__ int cell_coord(float m, int n) {
  const float v = floorf(__fdiv_rn(m, 16.0f));
  if (!(v >= 0.0f && v < 9.223372036854775808e18f)) return 0;
  return v >= (float)(n - 1) ? n - 1 : (int)v;
}

// Warp-aggregated atomic increment of per-cell counters; returns this lane's rank in its cell.
__device__ __forceinline__ void count_cell(int cell, int* counters, int2* out) {
  const unsigned mask = __ballot_sync(0xffffffffu, cell >= 0);
  if (cell < 0) return;
  const unsigned peers = __match_any_sync(mask, cell);
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(peers) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(counters + cell, __popc(peers));
  base = __shfl_sync(peers, base, leader);
  *out = make_int2(cell, base + __popc(peers & ((1u << lane) - 1u)));
}

__global__ void k_cell_count(const float2* __restrict__ mu2d, const uint8_t* __restrict__ keep, int G,
                             int ntx, int nty, int* __restrict__ cell_count, int2* __restrict__ cell_rank) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int v = blockIdx.y;
  const int T = ntx * nty;
  int cell = -1;
  if (g < G) {
    const long long o = (long long)v * G + g;
    if (keep[o]) {
      const float2 m = mu2d[o];
      cell = cell_coord(m.y, nty) * ntx + cell_coord(m.x, ntx);
    } else {
      cell_rank[o] = make_int2(-1, 0);
    }
  }
  int2 cr;
  count_cell(cell, cell_count + (long long)v * T, &cr);
  if (cell >= 0) cell_rank[(long long)v * G + g] = cr;
}

// Exclusive scan of the per-cell counts of one view: start[0..T], start[T] = total.
__global__ void __launch_bounds__(1024) k_cell_scan(const int* __restrict__ cnt, int* __restrict__ start, int T) {
  __shared__ int warp_sums[32];
  const int v = blockIdx.x;
  const int* c = cnt + (long long)v * T;
  int* s = start + (long long)v * (T + 1);
  const int per = (T + blockDim.x - 1) / blockDim.x;
  const int beg = min(T, (int)threadIdx.x * per), end = min(T, beg + per);
  int local = 0;
  for (int i = beg; i < end; ++i) local += c[i];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) warp_sums[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    int ws = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, ws, d);
      if (lane >= d) ws += y;
    }
    if (lane < nw) warp_sums[lane] = ws;
  }
  __syncthreads();
  int run = incl - local + (wid > 0 ? warp_sums[wid - 1] : 0);
  for (int i = beg; i < end; ++i) {
    s[i] = run;
    run += c[i];
  }
  if (threadIdx.x == blockDim.x - 1) s[T] = run;
}

__global__ void k_cell_scatter(const float2* __restrict__ mu2d, const int2* __restrict__ cell_rank,
                               const int* __restrict__ start, int G, int T, float4* __restrict__ rec) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int v = blockIdx.y;
  if (g >= G) return;
  const long long o = (long long)v * G + g;
  const int2 cr = cell_rank[o];
  if (cr.x < 0) return;
  const float2 m = mu2d[o];
  rec[(long long)v * G + start[(long long)v * (T + 1) + cr.x] + cr.y] = make_float4(__int_as_float(g), m.x, m.y, 0.f);
}

// Exclusive prefix sum over the block (BS_THREADS threads); ends with a barrier.
__device__ __forceinline__ int block_excl_scan(int x, int* s_scan) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = x;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_scan[wid] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < wid; ++w) base += s_scan[w];
  __syncthreads();
  return base + incl - x;
}

__device__ __forceinline__ void bitonic_sort(u64* s, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < (P >> 1); i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool asc = (lo & size) == 0;
        const u64 a = s[lo], b = s[hi];
        if ((a > b) == asc) {
          s[lo] = b;
          s[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Packed sort keys (q, stencil offset j, gaussian id g), compared as unsigned integers: the
// 64-bit form q<<40 | j<<32 | g holds any problem; the 32-bit form q<<21 | j<<17 | g holds
// G <= 2^17 and S <= 16 stencil offsets (R <= 1) in the same order, and halves the warp's key
// buffer and its compare and shuffle work.  dsh/dwd: shift and width of the digits of the bits
// below q (j, then g) that the tie narrowing walks, most significant first.
template <class KT>
struct KeyBits;
template <>
struct KeyBits<u64> {
  static constexpr int QS = 40, JS = 32, ND = 7;
  static constexpr u64 GM = 0xffffffffull, JM = 0xffull;
  // digits 32, 26, 20, 14, 8, 2 (6 bits) and 0 (2 bits)
  __device__ static int dsh(int d) { return d < 6 ? 32 - 6 * d : 0; }
  __device__ static int dwd(int d) { return d < 6 ? 6 : 2; }
};
template <>
struct KeyBits<unsigned> {
  static constexpr int QS = 21, JS = 17, ND = 4;
  static constexpr unsigned GM = 0x1ffffu, JM = 0xfu;
  // digits 15, 9, 3 (6 bits) and 0 (3 bits)
  __device__ static int dsh(int d) { return d < 3 ? 15 - 6 * d : 0; }
  __device__ static int dwd(int d) { return d < 3 ? 6 : 3; }
};
constexpr int KEY32_MAX_G = 1 << 17, KEY32_MAX_S = 16;

// Quantised distance of the reference: clamp(long(dist2), 0, 2047), torch's INT64_MIN for
// non-finite or >= 2^63 values clamping to 0.
template <class KT = u64>
__device__ __forceinline__ KT make_key(int j, float4 r, float ctx, float cty) {
  const float dx = __fsub_rn(r.y, ctx);
  const float dy = __fsub_rn(r.z, cty);
  const float d2 = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
  unsigned q = 0;
  if (d2 >= 0.0f && d2 < 9.223372036854775808e18f) q = d2 >= 2047.0f ? 2047u : (unsigned)d2;
  using KB = KeyBits<KT>;
  return ((KT)q << KB::QS) | ((KT)(unsigned)j << KB::JS) | (KT)(unsigned)__float_as_int(r.x);
}

// Writes the outputs of one tile from its sorted keys (threads first, first+step, ... of the
// caller's group): idx/count/cand, the stencil-indexed inverse table and, with PACK, the slot
// rows theta_u (tools/m4_train_binned.py:130-143, the reference's fp32 op order) | color_o | keo.
template <int PACK, class KT = u64>
__device__ __forceinline__ void emit_tile(const KT* keys, int n, int v, int t, int ntx, int T, int G, int S, int K,
                                          const float* __restrict__ proj, float inv_k, int* __restrict__ idx,
                                          int* __restrict__ inv, void* __restrict__ slots, int first, int step) {
  using KB = KeyBits<KT>;
  const int cnt = min(n, K);
  const int tx = t % ntx, ty = t / ntx;
  const float ox = (float)(tx * 16), oy = (float)(ty * 16);
  for (int k = first; k < K; k += step) {
    const long long o = ((long long)v * T + t) * K + k;
    if (k < cnt) {
      const KT key = keys[k];
      const int g = (int)(unsigned)(key & KB::GM);
      const int j = (int)((key >> KB::JS) & KB::JM);
      idx[o] = g;
      // a slot the fp32 packing marks dead gets no inverse entry: its gradient row is zero, so
      // the slot->gaussian gather may skip it (and a view where all of a gaussian's slots are
      // dead drops out of its parameter backward) without changing a bit
      if (inv && PACK != 1) inv[((long long)v * G + g) * S + j] = t * K + k;
      if (PACK) {
        const float4* p = reinterpret_cast<const float4*>(proj + ((long long)v * G + g) * TTS_PROJ_FLOATS);
        const float4 p0 = p[0], p1 = p[1], p2 = p[2];
        const float mux = __fsub_rn(p0.x, ox), muy = __fsub_rn(p0.y, oy);
        const float a = p0.z, b = p0.w, c = p1.x;
        const float Q = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(a, mux), mux),
                                            __fmul_rn(__fmul_rn(__fmul_rn(2.0f, b), mux), muy)),
                                  __fmul_rn(__fmul_rn(c, muy), muy));
        const float th[6] = {__fmul_rn(-a, inv_k), __fmul_rn(-c, inv_k), __fmul_rn(__fmul_rn(-2.0f, b), inv_k),
                             __fmul_rn(__fmul_rn(2.0f, __fadd_rn(__fmul_rn(a, mux), __fmul_rn(b, muy))), inv_k),
                             __fmul_rn(__fmul_rn(2.0f, __fadd_rn(__fmul_rn(b, mux), __fmul_rn(c, muy))), inv_k),
                             __fsub_rn(1.0f, __fmul_rn(Q, inv_k))};
        if (PACK == 1) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(slots) + o * TTS_SLOT_FLOATS);
          dst[0] = make_float4(th[0], th[1], th[2], th[3]);
          dst[1] = make_float4(th[4], th[5], p1.y, p1.z);
          // field 10 marks a slot whose weight is zero at every pixel of the tile (the tile
          // kernels skip it; the tables keep it, as the reference's do)
          const bool dead = slot_dead(th[0], th[1], th[2], th[3], th[4], th[5]);
          dst[2] = make_float4(p1.w, p2.x, dead ? 1.f : 0.f, 0.f);
          if (inv && !dead) inv[((long long)v * G + g) * S + j] = t * K + k;
        } else {
          // compact bf16 row: theta_u as a bf16 (hi, lo) pair (hi + lo carries ~16 significant
          // bits, which u = Phi.theta needs), colour_o and o_col as bf16
          __nv_bfloat16 r[16];
#pragma unroll
          for (int q = 0; q < 6; ++q) {
            r[q] = __float2bfloat16_rn(th[q]);
            r[6 + q] = __float2bfloat16_rn(__fsub_rn(th[q], __bfloat162float(r[q])));
          }
          r[12] = __float2bfloat16_rn(p1.y);
          r[13] = __float2bfloat16_rn(p1.z);
          r[14] = __float2bfloat16_rn(p1.w);
          r[15] = __float2bfloat16_rn(p2.x);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(slots) + o * TTS_SLOT_BF16);
          dst[0] = *reinterpret_cast<const uint4*>(&r[0]);
          dst[1] = *reinterpret_cast<const uint4*>(&r[8]);
        }
      }
    } else {
      idx[o] = -1;
    }
  }
}

// Cell ranges of the tile's stencil: entry j = (dy+R)*D + (dx+R) holds the home cell of the
// gaussians that see this tile at offset (dy, dx), i.e. cell = tile - (dy, dx).
__device__ __forceinline__ void stencil_range(int j, int R, int tx, int ty, int ntx, int nty, const int* cs, int& beg,
                                              int& len) {
  const int D = 2 * R + 1;
  const int dy = j / D - R, dx = j % D - R;
  const int cy = ty - dy, cx = tx - dx;
  beg = 0;
  len = 0;
  if (cy >= 0 && cy < nty && cx >= 0 && cx < ntx) {
    const int c = cy * ntx + cx;
    beg = cs[c];
    len = cs[c + 1] - beg;
  }
}

constexpr int WB_WARPS = 4;
// Keys per warp: 896 (7 KB) keeps six 4-warp blocks per SM within shared memory and covers every
// tile of the config-2 workload (none has more candidates); larger tiles go to the block kernel,
// whose per-tile latency (~16 µs) would otherwise bound the stage even for a few tiles.
constexpr int WCAP = 896;
constexpr int WTIE_NARROW = 256; // above this many keys at or below q*, narrow among the ties
constexpr int WTIES = 64;   // ties at the selection boundary resolved by rank (more: narrowed or sorted)

// Warp bucket sort of keys[0, m) (m <= WCAP/2; the upper half of the warp's buffer is the
// scratch): keys are distributed into 64 buckets by the top 6 bits of their 11-bit distance
// (exclusive offsets from a histogram), then each key's position inside its bucket is its rank
// among the bucket's keys (keys are unique: one stencil offset per gaussian and tile).  Buckets
// beyond 64 keys would make the ranking quadratic: the caller then falls back to the bitonic
// sort.  Returns false (keys untouched) in that case.
template <class KT>
__device__ __forceinline__ bool bucket_sort(KT* keys, int m, int lane, int* hist, int* start) {
  constexpr int BS = KeyBits<KT>::QS + 5;
  KT* tmp = keys + WCAP / 2;
  hist[lane] = 0;
  hist[lane + 32] = 0;
  __syncwarp();
  for (int i = lane; i < m; i += 32) atomicAdd(&hist[(int)((keys[i] >> BS) & 63u)], 1);
  __syncwarp();
  const int h0 = hist[2 * lane], h1 = hist[2 * lane + 1];
  if (__any_sync(0xffffffffu, h0 > 64 || h1 > 64)) return false;
  int incl = h0 + h1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  const int excl = incl - h0 - h1;
  start[2 * lane] = excl;
  start[2 * lane + 1] = excl + h0;
  hist[2 * lane] = excl;            // hist becomes the scatter cursor
  hist[2 * lane + 1] = excl + h0;
  if (lane == 31) start[64] = incl;
  __syncwarp();
  for (int i = lane; i < m; i += 32) {
    const KT k = keys[i];
    tmp[atomicAdd(&hist[(int)((k >> BS) & 63u)], 1)] = k;
  }
  __syncwarp();
  for (int i = lane; i < m; i += 32) {
    const KT k = tmp[i];
    const int b = (int)((k >> BS) & 63u);
    const int s = start[b], e = start[b + 1];
    int r = 0;
    for (int t = s; t < e; ++t) r += tmp[t] < k;
    keys[s + r] = k;
  }
  __syncwarp();
  return true;
}

// Warp-synchronous bitonic sort of keys[0, m) in place (padded with ~0 up to the next power of
// two, which must fit the buffer).
template <class KT>
__device__ __forceinline__ void sort_front(KT* keys, int m, int lane) {
  int P = 1;
  while (P < m) P <<= 1;
  for (int i = m + lane; i < P; i += 32) keys[i] = ~(KT)0;
  __syncwarp();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = lane; i < (P >> 1); i += 32) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool asc = (lo & size) == 0;
        const KT a = keys[lo], b = keys[hi];
        if ((a > b) == asc) {
          keys[lo] = b;
          keys[hi] = a;
        }
      }
      __syncwarp();
    }
  }
}

constexpr int KG_UNROLL = 4;   // candidate records in flight per lane during key generation

// One warp per tile for tiles with at most WCAP candidates (tiles with more are appended to the
// overflow list for the block kernel).  Keys in per-warp shared memory; when n > K a two-level
// histogram of q (64 then 32 bins) finds q*, the keys with q <= q* are compacted in place and
// only those are sorted (warp-synchronous bitonic sort, no block barriers).
template <int PACK, class KT>
__global__ void __launch_bounds__(WB_WARPS * 32)
    k_bin_warp(const int* __restrict__ cell_start, const float4* __restrict__ rec, int G, int ntx, int nty, int R,
               int K, int V, const float* __restrict__ proj, float inv_k, int* __restrict__ idx,
               int* __restrict__ count, int* __restrict__ cand, int* __restrict__ inv, void* __restrict__ slots,
               int* __restrict__ ovf_list, int* __restrict__ ovf_count) {
  using KB = KeyBits<KT>;
  extern __shared__ __align__(8) unsigned char wsm_raw[];
  __shared__ int whist[WB_WARPS][64];
  __shared__ int wstart[WB_WARPS][65];
  __shared__ KT wties[WB_WARPS][WTIES];
  __shared__ int wbeg[WB_WARPS][BS_MAXS], wlen[WB_WARPS][BS_MAXS], woff[WB_WARPS][BS_MAXS + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = ntx * nty;
  const long long gt = (long long)blockIdx.x * WB_WARPS + warp;
  if (gt >= (long long)V * T) return;
  const int v = (int)(gt / T), t = (int)(gt % T);
  const int tx = t % ntx, ty = t / ntx;
  const int D = 2 * R + 1, S = D * D;
  KT* buf = reinterpret_cast<KT*>(wsm_raw) + (size_t)warp * WCAP;
  int* hist = whist[warp];
  const int* cs = cell_start + (long long)v * (T + 1);
  const float4* rv = rec + (long long)v * G;
  for (int j = lane; j < S; j += 32) {
    int b, l;
    stencil_range(j, R, tx, ty, ntx, nty, cs, b, l);
    wbeg[warp][j] = b;
    wlen[warp][j] = l;
  }
  __syncwarp();
  if (lane == 0) {
    int o = 0;
    for (int j = 0; j < S; ++j) {
      woff[warp][j] = o;
      o += wlen[warp][j];
    }
    woff[warp][S] = o;
  }
  __syncwarp();
  const int n = woff[warp][S];
  if (n > WCAP) {
    if (lane == 0) ovf_list[atomicAdd(ovf_count, 1)] = (int)gt;
    return;
  }
  const float ctx = __fmul_rn(__fadd_rn((float)tx, 0.5f), 16.0f);
  const float cty = __fmul_rn(__fadd_rn((float)ty, 0.5f), 16.0f);
  // candidate c of the tile's concatenated cell lists -> (stencil offset j, record): each lane
  // issues the loads of KG_UNROLL candidates before keying them, so a tile costs ~n / (32 KG_UNROLL)
  // round trips to L2 instead of one per cell
  {
    int jc = 0;
    for (int c0 = 0; c0 < n; c0 += 32 * KG_UNROLL) {
      float4 r[KG_UNROLL];
      int jj[KG_UNROLL];
#pragma unroll
      for (int u = 0; u < KG_UNROLL; ++u) {
        const int c = c0 + 32 * u + lane;
        jj[u] = -1;
        if (c < n) {
          while (c >= woff[warp][jc + 1]) ++jc;   // c only grows along a lane: empty cells are skipped
          jj[u] = jc;
          r[u] = rv[wbeg[warp][jc] + c - woff[warp][jc]];
        }
      }
#pragma unroll
      for (int u = 0; u < KG_UNROLL; ++u)
        if (jj[u] >= 0) buf[c0 + 32 * u + lane] = make_key<KT>(jj[u], r[u], ctx, cty);
    }
  }
  __syncwarp();
  int m = n;
  if (n > K) {
    // level 1: the top 6 of the 11 bits of q
    hist[lane] = 0;
    hist[lane + 32] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) atomicAdd(&hist[(int)((buf[i] >> (KB::QS + 5)) & 63u)], 1);
    __syncwarp();
    const int h0 = hist[2 * lane], h1 = hist[2 * lane + 1];
    int incl = h0 + h1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    const int excl = incl - h0 - h1;
    const bool hit1 = excl < K && K <= incl;
    const int src1 = __ffs(__ballot_sync(0xffffffffu, hit1)) - 1;
    const int b1_l = (excl + h0 >= K) ? 2 * lane : 2 * lane + 1;
    const int below_l = (excl + h0 >= K) ? excl : excl + h0;
    const int b1 = __shfl_sync(0xffffffffu, b1_l, src1);
    const int below1 = __shfl_sync(0xffffffffu, below_l, src1);
    __syncwarp();
    // level 2: the low 5 bits of q among keys in bucket b1
    hist[lane] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const unsigned q = (unsigned)(buf[i] >> KB::QS);
      if ((int)(q >> 5) == b1) atomicAdd(&hist[q & 31u], 1);
    }
    __syncwarp();
    const int hv = hist[lane];
    int incl2 = hv;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl2, d);
      if (lane >= d) incl2 += y;
    }
    const int need = K - below1;
    const bool hit2 = (incl2 - hv) < need && need <= incl2;
    const int src2 = __ffs(__ballot_sync(0xffffffffu, hit2)) - 1;
    const unsigned qstar = (unsigned)(b1 * 32 + src2);
    m = below1 + __shfl_sync(0xffffffffu, incl2, src2);
    const int hq = __shfl_sync(0xffffffffu, hv, src2);    // keys with q == q*
    const int c_lt = m - hq;                                 // keys with q < q* (all kept)
    const unsigned lt = (1u << lane) - 1u;
    if (m > K && hq <= WTIES) {
      // Ties at q* straddle the K boundary: the keys with q < q* go to the front, the ties to a
      // side list; each tie's rank among the ties (by stencil offset, then id: unique per tile)
      // places the K - c_lt smallest directly behind the sorted front, so only c_lt < K keys
      // need sorting.
      KT* ties = wties[warp];
      int w = 0, tw = 0;
      for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const KT key = i < n ? buf[i] : ~(KT)0;
        const unsigned q = (unsigned)(key >> KB::QS);
        const bool lo = i < n && q < qstar, eq = i < n && q == qstar;
        const unsigned bl = __ballot_sync(0xffffffffu, lo), be = __ballot_sync(0xffffffffu, eq);
        __syncwarp();
        if (lo) buf[w + __popc(bl & lt)] = key;
        if (eq) ties[tw + __popc(be & lt)] = key;
        w += __popc(bl);
        tw += __popc(be);
        __syncwarp();
      }
      if (c_lt > WCAP / 2 || !bucket_sort(buf, c_lt, lane, hist, wstart[warp])) sort_front(buf, c_lt, lane);
      const int need = K - c_lt;
      for (int i = lane; i < hq; i += 32) {
        const KT key = ties[i];
        int rank = 0;
        for (int t2 = 0; t2 < hq; ++t2) rank += ties[t2] < key;
        if (rank < need) buf[c_lt + rank] = key;
      }
      __syncwarp();
      m = -1;    // sorted
    } else if (m > WTIE_NARROW) {
      // Many ties at q* (border tiles collect off-screen gaussians, all at the clamped q = 2047):
      // narrow among the ties on the key's low 40 bits (stencil offset j, then id g) in 6-bit
      // digits, with warp-aggregated histogram increments, down to the exact threshold key t*
      // (the (K - c_lt)-th smallest tie).  The kept keys are those at or below t*: exactly K.
      int need = K - c_lt;
      KT pmask = (KT)0x7FF << KB::QS, pval = (KT)qstar << KB::QS;
      for (int d = 0; d < KB::ND; ++d) {
        const int sh = KB::dsh(d);
        const KT dm = (KT)((1 << KB::dwd(d)) - 1);
        hist[lane] = 0;
        hist[lane + 32] = 0;
        __syncwarp();
        for (int base = 0; base < n; base += 32) {
          const int i = base + lane;
          const KT key = i < n ? buf[i] : (KT)0;
          const bool act = i < n && (key & pmask) == pval;
          const int bin = (int)((key >> sh) & dm);
          const unsigned am = __ballot_sync(0xffffffffu, act);
          if (act) {
            const unsigned peers = __match_any_sync(am, bin);
            if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
          }
        }
        __syncwarp();
        const int g0 = hist[2 * lane], g1 = hist[2 * lane + 1];
        int gin = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, gin, o);
          if (lane >= o) gin += y;
        }
        const int gex = gin - g0 - g1;
        const bool first = gex + g0 >= need;
        const int src = __ffs(__ballot_sync(0xffffffffu, gex < need && need <= gin)) - 1;
        const int bkt = __shfl_sync(0xffffffffu, first ? 2 * lane : 2 * lane + 1, src);
        const int below = __shfl_sync(0xffffffffu, first ? gex : gex + g0, src);
        const int inb = __shfl_sync(0xffffffffu, first ? g0 : g1, src);
        need -= below;
        pval |= (KT)bkt << sh;
        pmask |= dm << sh;
        __syncwarp();
        if (inb == 1) break;    // the bucket holds t* alone
      }
      // keys at or below t*: a smaller prefix under pmask (q < q* included), or t* itself
      int w = 0;
      for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const KT key = i < n ? buf[i] : ~(KT)0;
        const bool sel = i < n && (key & pmask) <= pval;
        const unsigned bal = __ballot_sync(0xffffffffu, sel);
        __syncwarp();
        if (sel) buf[w + __popc(bal & lt)] = key;
        w += __popc(bal);
        __syncwarp();
      }
      m = w;    // = K
    } else {
      // compact the keys with q <= q* to the front (writes never pass the chunk being read)
      int w = 0;
      for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const KT key = i < n ? buf[i] : ~(KT)0;
        const bool sel = i < n && (unsigned)(key >> KB::QS) <= qstar;
        const unsigned bal = __ballot_sync(0xffffffffu, sel);
        __syncwarp();
        if (sel) buf[w + __popc(bal & lt)] = key;
        w += __popc(bal);
        __syncwarp();
      }
    }
  }
  if (m >= 0 && (m > WCAP / 2 || !bucket_sort(buf, m, lane, hist, wstart[warp]))) sort_front(buf, m, lane);
  emit_tile<PACK, KT>(buf, n, v, t, ntx, T, G, S, K, proj, inv_k, idx, inv, slots, lane, 32);
  if (lane == 0) {
    count[(long long)v * T + t] = min(n, K);
    cand[(long long)v * T + t] = n;
  }
}

// Two blocks per SM (64 registers, no spills; 2 x ~73 KB of shared memory): the 296-block grid
// is one resident wave, so both blocks of an SM walk the tile list at once and one block's
// barrier waits hide behind the other's work.  Unbounded, the kernel took ~118 registers, one
// block fitted per SM and the second half of the grid started only after the first had walked
// its whole share of the list.
template <int PACK>
__global__ void __launch_bounds__(BS_THREADS, 2)
    k_bin_select(const int* __restrict__ cell_start, const float4* __restrict__ rec, int G, int ntx, int nty,
                 int R, int K, const float* __restrict__ proj, float inv_k, int* __restrict__ idx,
                 int* __restrict__ count, int* __restrict__ cand, int* __restrict__ inv,
                 void* __restrict__ slots, const int* __restrict__ list, const int* __restrict__ list_count) {
  extern __shared__ u64 skeys[];       // [BS_CAP]
  __shared__ int shist[2048];
  __shared__ int s_beg[BS_MAXS], s_len[BS_MAXS], s_off[BS_MAXS + 1];
  __shared__ u64 s_pval, s_pmask;
  __shared__ int s_below, s_le, s_cnt;
  __shared__ int s_scan[BS_THREADS / 32];

  const int T = ntx * nty;
  const int D = 2 * R + 1, S = D * D;
  const int tid = threadIdx.x;
  const int n_list = *list_count;
  for (int li = blockIdx.x; li < n_list; li += gridDim.x) {
  const int gt = list[li];
  const int v = gt / T, t = gt % T;
  const int tx = t % ntx, ty = t / ntx;
  const int* cs = cell_start + (long long)v * (T + 1);
  const float4* rv = rec + (long long)v * G;
  __syncthreads();   // the previous tile's shared state is no longer read

  if (tid < S) {
    int beg, len;
    stencil_range(tid, R, tx, ty, ntx, nty, cs, beg, len);
    s_beg[tid] = beg;
    s_len[tid] = len;
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0;
    for (int j = 0; j < S; ++j) {
      s_off[j] = o;
      o += s_len[j];
    }
    s_off[S] = o;
  }
  __syncthreads();
  const int n = s_off[S];
  const float ctx = __fmul_rn(__fadd_rn((float)tx, 0.5f), 16.0f);
  const float cty = __fmul_rn(__fadd_rn((float)ty, 0.5f), 16.0f);

  int nsel;
  if (n <= BS_CAP) {
    for (int j = 0; j < S; ++j) {
      const int len = s_len[j], beg = s_beg[j], off = s_off[j];
#pragma unroll 4
      for (int i = tid; i < len; i += BS_THREADS) skeys[off + i] = make_key(j, rv[beg + i], ctx, cty);
    }
    nsel = n;
    if (n > K) {
      // MSB radix select over the keys in shared memory (digits q | j | g of 11/8/11/11/10 bits):
      // after each digit the bucket holding the K-th smallest key is known; stop once the keys at
      // or below it fit a small sort (SORT_CAP).  Tiles whose candidates share one quantised
      // distance (border tiles collect off-screen gaussians, all at q = 2047) are settled by the
      // stencil and id digits instead of sorting thousands of ties.  Histogram increments are
      // aggregated per warp over lanes with the same bin (match_any).
      const int shifts[5] = {40, 32, 21, 10, 0};
      const int bits[5] = {11, 8, 11, 11, 10};
      if (tid == 0) {
        s_pval = 0ull;
        s_pmask = 0ull;
        s_below = 0;
      }
      __syncthreads();
      const int lane = tid & 31;
      int shift = 0;
      for (int d = 0; d < 5; ++d) {
        shift = shifts[d];
        const int nb = 1 << bits[d];
        for (int i = tid; i < nb; i += BS_THREADS) shist[i] = 0;
        if (tid == 0) s_le = n;
        __syncthreads();
        const u64 pval = s_pval, pmask = s_pmask;
        for (int i0 = 0; i0 < n; i0 += BS_THREADS) {
          const int i = i0 + tid;
          u64 key = 0;
          bool act = false;
          if (i < n) {
            key = skeys[i];
            act = (key & pmask) == pval;
          }
          const int bin = (int)((key >> shift) & (u64)(nb - 1));
          const unsigned am = __ballot_sync(0xffffffffu, act);
          if (act) {
            const unsigned peers = __match_any_sync(am, bin);
            if (lane == __ffs(peers) - 1) atomicAdd(&shist[bin], __popc(peers));
          }
        }
        __syncthreads();
        const int need = K - s_below;
        const int per = nb >= BS_THREADS ? nb / BS_THREADS : 1;
        int loc = 0;
        if (tid * per < nb)
          for (int q = 0; q < per; ++q) loc += shist[tid * per + q];
        const int excl = block_excl_scan(loc, s_scan);
        if (excl < need && need <= excl + loc) {
          int c = excl, b = 0;
          for (; b < per - 1; ++b) {
            if (c + shist[tid * per + b] >= need) break;
            c += shist[tid * per + b];
          }
          const int bucket = tid * per + b;
          s_below += c;
          s_pval = pval | ((u64)bucket << shift);
          s_pmask = pmask | ((u64)(nb - 1) << shift);
          s_le = s_below + shist[bucket];
        }
        __syncthreads();
        if (s_le <= SORT_CAP) break;   // at the last digit the bucket is the K-th key alone
      }
      const u64 upper = s_pval | ((1ull << shift) - 1ull);
      // compact the keys at or below the bucket to the front: each thread stages its contiguous
      // chunk in registers first, so no write passes a key not yet read
      const int per = (n + BS_THREADS - 1) / BS_THREADS;   // <= BS_CAP / BS_THREADS = 16
      u64 mine[BS_CAP / BS_THREADS];
      int cnt = 0;
#pragma unroll
      for (int j = 0; j < BS_CAP / BS_THREADS; ++j) {
        const int i = tid * per + j;
        mine[j] = (j < per && i < n) ? skeys[i] : ~0ull;
        cnt += (j < per && i < n && mine[j] <= upper) ? 1 : 0;
      }
      const int off = block_excl_scan(cnt, s_scan);
#pragma unroll
      for (int j = 0, w = off; j < BS_CAP / BS_THREADS; ++j) {
        if (j < per && tid * per + j < n && mine[j] <= upper) skeys[w++] = mine[j];
      }
      __syncthreads();
      nsel = s_le;
    }
  } else {
    // MSB radix select of the K-th smallest key; stop as soon as the keys at or below the
    // current bucket fit in shared memory, then collect them.
    const int shifts[5] = {40, 32, 21, 10, 0};
    const int bits[5] = {11, 8, 11, 11, 10};
    if (tid == 0) {
      s_pval = 0ull;
      s_pmask = 0ull;
      s_below = 0;
    }
    __syncthreads();
    nsel = 0;
    for (int d = 0; d < 5; ++d) {
      const int shift = shifts[d], nb = 1 << bits[d];
      for (int i = tid; i < nb; i += BS_THREADS) shist[i] = 0;
      if (tid == 0) s_le = n;   // replaced by the bucket's count below (n > BS_CAP: not yet collected)
      __syncthreads();
      const u64 pval = s_pval, pmask = s_pmask;
      for (int j = 0; j < S; ++j) {
        const int len = s_len[j], beg = s_beg[j];
#pragma unroll 4
        for (int i = tid; i < len; i += BS_THREADS) {
          const u64 key = make_key(j, rv[beg + i], ctx, cty);
          if ((key & pmask) == pval) atomicAdd(&shist[(int)((key >> shift) & (u64)(nb - 1))], 1);
        }
      }
      __syncthreads();
      // the bucket holding the need-th key (the first whose cumulative count reaches it): each
      // thread sums its nb / BS_THREADS consecutive bins (one bin, or none, when nb is smaller),
      // a block scan gives the thread offsets, and the one thread whose range holds it walks its
      // own bins
      const int need = K - s_below;
      const int per = nb >= BS_THREADS ? nb / BS_THREADS : 1;
      int loc = 0;
      if (tid * per < nb)
        for (int q = 0; q < per; ++q) loc += shist[tid * per + q];
      const int excl = block_excl_scan(loc, s_scan);
      if (excl < need && need <= excl + loc) {
        int c = excl, b = 0;
        for (; b < per - 1; ++b) {
          if (c + shist[tid * per + b] >= need) break;
          c += shist[tid * per + b];
        }
        const int bucket = tid * per + b;
        s_below += c;
        s_pval = pval | ((u64)bucket << shift);
        s_pmask = pmask | ((u64)(nb - 1) << shift);
        s_le = s_below + shist[bucket];
        s_cnt = 0;
      }
      __syncthreads();
      if (s_le <= BS_CAP) {
        // collect the keys at or below the bucket: one shared-memory atomic per warp (ballot)
        const u64 upper = s_pval | ((1ull << shift) - 1ull);
        const int lane = tid & 31;
        for (int j = 0; j < S; ++j) {
          const int len = s_len[j], beg = s_beg[j];
          for (int i0 = 0; i0 < len; i0 += BS_THREADS) {
            const int i = i0 + tid;
            u64 key = 0;
            bool sel = false;
            if (i < len) {
              key = make_key(j, rv[beg + i], ctx, cty);
              sel = key <= upper;
            }
            const unsigned bal = __ballot_sync(0xffffffffu, sel);
            int base = 0;
            if (lane == 0 && bal) base = atomicAdd(&s_cnt, __popc(bal));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (sel) skeys[base + __popc(bal & ((1u << lane) - 1u))] = key;
          }
        }
        __syncthreads();
        nsel = s_cnt;
        break;
      }
    }
  }
  int P = 1;
  while (P < nsel) P <<= 1;
  for (int i = nsel + tid; i < P; i += BS_THREADS) skeys[i] = ~0ull;
  __syncthreads();
  bitonic_sort(skeys, P);

  emit_tile<PACK>(skeys, n, v, t, ntx, T, G, S, K, proj, inv_k, idx, inv, slots, tid, BS_THREADS);
  if (tid == 0) {
    count[(long long)v * T + t] = min(n, K);
    cand[(long long)v * T + t] = n;
  }
  }
}

// ---- host launchers --------------------------------------------------------------------------
struct BinWorkspace {
  int* cell_count;   // [V][T]
  int* cell_start;   // [V][T+1]
  int2* cell_rank;   // [V][G]
  float4* rec;       // [V][G]
  int* ovf;          // [1 + V*T]: count, then the tiles left to the block kernel
};

static size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

size_t bin_workspace_bytes(int G, int V, int T) {
  return align_up((size_t)V * T * 4) + align_up((size_t)V * (T + 1) * 4) + align_up((size_t)V * G * 8) +
         align_up((size_t)V * G * 16) + align_up((size_t)(V * T + 1) * 4);
}

static BinWorkspace carve(void* ws, int G, int V, int T) {
  char* p = static_cast<char*>(ws);
  BinWorkspace w;
  w.cell_count = reinterpret_cast<int*>(p);
  p += align_up((size_t)V * T * 4);
  w.cell_start = reinterpret_cast<int*>(p);
  p += align_up((size_t)V * (T + 1) * 4);
  w.cell_rank = reinterpret_cast<int2*>(p);
  p += align_up((size_t)V * G * 8);
  w.rec = reinterpret_cast<float4*>(p);
  p += align_up((size_t)V * G * 16);
  w.ovf = reinterpret_cast<int*>(p);
  return w;
}

static int bin_core(const float* mu2d, const int* cell_count, const int2* cell_rank, int G, int V, int ntx,
                    int nty, int R, int K, const float* proj, float inv_k, int* idx, int* count, int* cand,
                    int* inv, void* slots, int slot_format, BinWorkspace w, cudaStream_t st) {
  const int T = ntx * nty;
  const int S = (2 * R + 1) * (2 * R + 1);
  if (inv) {
    if (cudaMemsetAsync(inv, 0xff, (size_t)V * G * S * 4, st) != cudaSuccess) return check_launch("memset inv");
  }
  k_cell_scan<<<V, 1024, 0, st>>>(cell_count, w.cell_start, T);
  dim3 gg((G + 255) / 256, V);
  if (G > 0) k_cell_scatter<<<gg, 256, 0, st>>>(reinterpret_cast<const float2*>(mu2d), cell_rank, w.cell_start, G, T, w.rec);
  if (cudaMemsetAsync(w.ovf, 0, 4, st) != cudaSuccess) return check_launch("memset overflow count");
  const long long tiles = (long long)V * T;
  const unsigned wblocks = (unsigned)((tiles + WB_WARPS - 1) / WB_WARPS);
  // 32-bit keys when the id and the stencil offset fit them (same order, half the shared memory)
  const bool key32 = G <= KEY32_MAX_G && S <= KEY32_MAX_S;
  const size_t wsmem64 = (size_t)WB_WARPS * WCAP * sizeof(u64), wsmem32 = (size_t)WB_WARPS * WCAP * sizeof(unsigned);
  static std::atomic<unsigned long long> attr_done{0};
  once_per_device(attr_done, [&] {
    cudaFuncSetAttribute(k_bin_warp<0, u64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem64);
    cudaFuncSetAttribute(k_bin_warp<1, u64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem64);
    cudaFuncSetAttribute(k_bin_warp<2, u64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem64);
    cudaFuncSetAttribute(k_bin_warp<0, unsigned>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem32);
    cudaFuncSetAttribute(k_bin_warp<1, unsigned>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem32);
    cudaFuncSetAttribute(k_bin_warp<2, unsigned>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem32);
    cudaFuncSetAttribute(k_bin_select<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(BS_CAP * sizeof(u64)));
    cudaFuncSetAttribute(k_bin_select<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(BS_CAP * sizeof(u64)));
    cudaFuncSetAttribute(k_bin_select<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(BS_CAP * sizeof(u64)));
  });
  const unsigned bblocks = (unsigned)(tiles < 296 ? tiles : 296);   // two blocks per SM loop over the list
  const size_t bsmem = (size_t)BS_CAP * sizeof(u64);
#define TTS_BIN_LAUNCH(P, PR, SL)                                                                              \
  if (key32)                                                                                                   \
    k_bin_warp<P, unsigned><<<wblocks, WB_WARPS * 32, wsmem32, st>>>(w.cell_start, w.rec, G, ntx, nty, R, K, V, PR, \
                                                                     inv_k, idx, count, cand, inv, SL, w.ovf + 1,   \
                                                                     w.ovf);                                        \
  else                                                                                                         \
    k_bin_warp<P, u64><<<wblocks, WB_WARPS * 32, wsmem64, st>>>(w.cell_start, w.rec, G, ntx, nty, R, K, V, PR,      \
                                                                inv_k, idx, count, cand, inv, SL, w.ovf + 1, w.ovf); \
  k_bin_select<P><<<bblocks, BS_THREADS, bsmem, st>>>(w.cell_start, w.rec, G, ntx, nty, R, K, PR, inv_k, idx, count,   \
                                                  cand, inv, SL, w.ovf + 1, w.ovf);
  if (proj && slots && slot_format == 1) {
    TTS_BIN_LAUNCH(2, proj, slots)
  } else if (proj && slots) {
    TTS_BIN_LAUNCH(1, proj, slots)
  } else {
    TTS_BIN_LAUNCH(0, nullptr, nullptr)
  }
#undef TTS_BIN_LAUNCH
  return check_launch("binning");
}

static int validate(int G, int V, int H, int W, int R, int K) {
  TTS_REQUIRE(G >= 0 && V >= 1, "G must be >= 0 and V >= 1");
  TTS_REQUIRE(H > 0 && W > 0 && H % 16 == 0 && W % 16 == 0, "H and W must be positive multiples of 16");
  TTS_REQUIRE(R >= 0 && R <= 3, "R must be in [0, 3]");
  TTS_REQUIRE(K >= 1 && K <= 256, "K must be in [1, 256]");
  return TTS_OK;
}

// ---- operands from cached tables (a (idx, valid) pair returned by an earlier binning) ----------
// The slot rows are rebuilt from the current projection; the inverse table needs, per gaussian, a
// slot index j in [0, S) that is distinct for each of its tiles.  An earlier binning put a
// gaussian only in the D x D tiles around its home cell then, so j is its tile's position in the
// D x D box starting at the smallest tile column and row it occupies (two atomicMin, independent
// of their order); tables that spread a gaussian wider are flagged in the status word.
constexpr int STATUS_TABLE_SPREAD = 8;

__global__ void k_cached_box(const int* __restrict__ idx, long long n, int T, int K, int ntx, int G,
                             int2* __restrict__ box) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int g = idx[i];
  if (g < 0 || g >= G) return;
  const long long vt = i / K;
  const int v = (int)(vt / T), t = (int)(vt % T);
  int2* b = box + (long long)v * G + g;
  atomicMin(&b->x, t % ntx);
  atomicMin(&b->y, t / ntx);
}

__global__ void __launch_bounds__(WB_WARPS * 32)
    k_cached_emit(const int* __restrict__ idx_in, const int2* __restrict__ box, int G, int V, int ntx, int nty, int R,
                  int K, const float* __restrict__ proj, float inv_k, int* __restrict__ idx, int* __restrict__ count,
                  int* __restrict__ inv, float* __restrict__ slots) {
  __shared__ u64 keys[WB_WARPS][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = ntx * nty;
  const long long gt = (long long)blockIdx.x * WB_WARPS + warp;
  if (gt >= (long long)V * T) return;
  const int v = (int)(gt / T), t = (int)(gt % T);
  const int tx = t % ntx, ty = t / ntx;
  const int D = 2 * R + 1, S = D * D;
  const int* in = idx_in + gt * K;
  // valid slots lead the tile: the count is the first invalid slot
  int first = K;
  for (int k = lane; k < K; k += 32)
    if (in[k] < 0) {
      first = k;
      break;
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
  const int n = first;
  for (int k = lane; k < n; k += 32) {
    int g = in[k];
    if (g >= G) {   // not a gaussian of this model (the host validates tables before the launch)
      atomicOr(&g_status, STATUS_TABLE_SPREAD);
      g = 0;
    }
    const int2 b = box[(long long)v * G + g];
    const int dx = tx - b.x, dy = ty - b.y;
    int j = dy * D + dx;
    if (dx < 0 || dx >= D || dy < 0 || dy >= D) {
      atomicOr(&g_status, STATUS_TABLE_SPREAD);
      j = 0;
    }
    keys[warp][k] = ((u64)(unsigned)j << 32) | (u64)(unsigned)g;
  }
  __syncwarp();
  if (lane == 0) count[gt] = n;
  emit_tile<1>(keys[warp], n, v, t, ntx, T, G, S, K, proj, inv_k, idx, inv, slots, lane, 32);
}

}  // namespace tts

using namespace tts;

extern "C" size_t tts_bin_workspace_bytes(int G, int V, int H, int W) {
  return bin_workspace_bytes(G, V, (H / 16) * (W / 16));
}

extern "C" int tts_bin_from_mu2d(const float* mu2d, const uint8_t* keep, int G, int V, int H, int W, int R, int K,
                                 int32_t* idx, int32_t* count, int32_t* cand, int32_t* inv, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (int rc = validate(G, V, H, W, R, K)) return rc;
  const int ntx = W / 16, nty = H / 16, T = ntx * nty;
  if (workspace_bytes < bin_workspace_bytes(G, V, T)) return fail(TTS_ERR_CAPACITY, "binning workspace too small");
  TTS_REQUIRE(idx && count && cand && workspace, "null output or workspace pointer");
  TTS_REQUIRE(G == 0 || (mu2d && keep), "null mu2d/keep");
  cudaStream_t st = as_stream(stream);
  BinWorkspace w = carve(workspace, G, V, T);
  if (cudaMemsetAsync(w.cell_count, 0, (size_t)V * T * 4, st) != cudaSuccess) return check_launch("memset counts");
  if (G > 0)
    k_cell_count<<<dim3((G + 255) / 256, V), 256, 0, st>>>(reinterpret_cast<const float2*>(mu2d), keep, G, ntx, nty,
                                                            w.cell_count, w.cell_rank);
  return bin_core(mu2d, w.cell_count, w.cell_rank, G, V, ntx, nty, R, K, nullptr, 0.f, idx, count, cand, inv, nullptr,
                  0, w, st);
}

extern "C" int tts_bin_pack(const float* mu2d, const uint8_t* keep, const float* proj, const int32_t* cell_count,
                            const int32_t* cell_rank, int G, int V, int H, int W, int R, int K, float k_poly,
                            int32_t* idx, int32_t* count, int32_t* cand, int32_t* inv, void* slots,
                            int slot_format, void* workspace, size_t workspace_bytes, void* stream) {
  (void)keep;
  TTS_REQUIRE(slot_format == 0 || slot_format == 1, "slot_format must be 0 (fp32 rows) or 1 (compact bf16 rows)");
  if (int rc = validate(G, V, H, W, R, K)) return rc;
  const int ntx = W / 16, nty = H / 16, T = ntx * nty;
  if (workspace_bytes < bin_workspace_bytes(G, V, T)) return fail(TTS_ERR_CAPACITY, "binning workspace too small");
  TTS_REQUIRE(idx && count && cand && slots && proj && cell_count && cell_rank, "null pointer");
  TTS_REQUIRE(aligned16(proj) && aligned16(slots), "proj and slots must be 16-byte aligned");
  TTS_REQUIRE(k_poly > 0.f, "k must be positive");
  BinWorkspace w = carve(workspace, G, V, T);
  return bin_core(mu2d, cell_count, reinterpret_cast<const int2*>(cell_rank), G, V, ntx, nty, R, K, proj,
                  (float)(1.0 / (double)k_poly), idx, count, cand, inv, slots, slot_format, w, as_stream(stream));
}

extern "C" size_t tts_pack_cached_workspace_bytes(int G, int V) {
  return (G > 0 && V > 0) ? (size_t)V * G * sizeof(int2) : 0;
}

extern "C" int tts_pack_cached(const float* proj, int G, int V, int H, int W, int R, int K, float k_poly,
                               const int32_t* idx_in, int32_t* idx, int32_t* count, int32_t* inv, float* slots,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate(G, V, H, W, R, K)) return rc;
  TTS_REQUIRE(proj && idx_in && idx && count && slots, "null pointer");
  TTS_REQUIRE(aligned16(proj) && aligned16(slots), "proj and slots must be 16-byte aligned");
  TTS_REQUIRE(k_poly > 0.f, "k must be positive");
  if (workspace_bytes < tts_pack_cached_workspace_bytes(G, V))
    return fail(TTS_ERR_CAPACITY, "cached-table workspace too small");
  const int ntx = W / 16, nty = H / 16, T = ntx * nty, S = (2 * R + 1) * (2 * R + 1);
  cudaStream_t st = as_stream(stream);
  int2* box = static_cast<int2*>(workspace);
  if (G > 0 && cudaMemsetAsync(box, 0x7f, (size_t)V * G * sizeof(int2), st) != cudaSuccess)
    return check_launch("memset box");
  if (inv && cudaMemsetAsync(inv, 0xff, (size_t)V * G * S * 4, st) != cudaSuccess) return check_launch("memset inv");
  const long long n = (long long)V * T * K;
  if (G > 0) k_cached_box<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(idx_in, n, T, K, ntx, G, box);
  if (int rc = check_launch("cached_box")) return rc;
  const unsigned blocks = (unsigned)(((long long)V * T + WB_WARPS - 1) / WB_WARPS);
  k_cached_emit<<<blocks, WB_WARPS * 32, 0, st>>>(idx_in, box, G, V, ntx, nty, R, K, proj,
                                                   (float)(1.0 / (double)k_poly), idx, count, inv, slots);
  return check_launch("cached_emit");
}

// ---- allocation-free binning -------------------------------------------------------------------
// Some callers cannot allocate device memory at the point where they bin: code that records the
// binning into a CUDA graph while stream capture is active (cudaMalloc is not allowed there),
// renderers embedded in another runtime that owns the device allocator and hands this library only
// its input and output buffers, and real-time loops that forbid allocation (and the device-wide
// synchronisation cudaMalloc/cudaFree can cause) after start-up.  For them, tts_bin_from_mu2d_noalloc
// runs the same binning with its scratch in a fixed static device array instead of a caller
// workspace.  The array is NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the library
// until the process exits; problems whose workspace (tts_bin_workspace_bytes) exceeds it are
// rejected.  All calls share the array, so calls that overlap on the GPU (different streams, or
// different host threads on one device without ordering) race on it and must be serialised.
namespace {
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(16) << 20;   // 16 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// The host-side name g_noalloc_scratch is only a stand-in for the symbol: its device address is
// looked up once per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(TTS_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(TTS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return TTS_OK;
}
}  // namespace

extern "C" int tts_bin_from_mu2d_noalloc(const float* mu2d, const uint8_t* keep, int G, int V, int H, int W, int R,
                                         int K, int32_t* idx, int32_t* count, int32_t* cand, int32_t* inv,
                                         void* stream) {
  if (int rc = validate(G, V, H, W, R, K)) return rc;
  const size_t need = bin_workspace_bytes(G, V, (H / 16) * (W / 16));
  if (need > NOALLOC_SCRATCH_BYTES)
    return fail(TTS_ERR_CAPACITY, "binning needs " + std::to_string(need) + " bytes of scratch, more than the " +
                                      std::to_string(NOALLOC_SCRATCH_BYTES) +
                                      "-byte static buffer of the allocation-free entry point");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // same launches as tts_bin_from_mu2d; the counters it needs at zero are cleared there
  return tts_bin_from_mu2d(mu2d, keep, G, V, H, W, R, K, idx, count, cand, inv, scratch, NOALLOC_SCRATCH_BYTES,
                           stream);
}
