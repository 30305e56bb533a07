// Multi-GPU optimizer step over NVLink peer memory (one process per GPU, buffers shared with
// CUDA IPC; no library collective on the data path).
//
// The reference trains one process on one device (spike/train.py:15-33): the batch gradient is
// the mean over the views (:27) followed by torch.optim.Adam.  With the views split over N
// GPUs, each rank owns 1/N of the flat parameter vector:
//   barrier 0   every rank has written its gradient (and loss) for this step;
//   reduce+Adam for its shard: the N ranks' gradients are read over NVLink and summed in rank
//               order, Adam updates the shard with the rank's (shard-owned) moments, and the
//               new values are stored into every rank's parameter buffer (peer stores);
//   barrier 1   every shard has arrived everywhere, so the replicas are bitwise equal.
// This replaces an all-reduce of the gradient followed by N replicated Adam passes: the bytes
// on NVLink are the same as a reduce-scatter + all-gather, the Adam work is divided by N, and
// the whole step stays inside one CUDA graph.  The barriers are single-block kernels that spin
// on flags written by the peers with an iteration limit (status word on timeout).
#include <algorithm>
#include <cstring>

#include "peer.cuh"
#include "sgld.cuh"

namespace tts {

// Signal and/or wait as a kernel of its own (one thread does it).
__global__ void k_peer_sync(PeerI flags, int* mine, int rank, int N, int phase, const int* __restrict__ epoch_ptr,
                            int do_signal, int do_wait) {
  if (threadIdx.x != 0) return;
  const int epoch = *epoch_ptr;
  if (do_signal) peer_signal(flags, rank, N, phase, epoch);   // earlier kernels' writes precede it
  if (do_wait) peer_wait(mine, N, phase, epoch);
}

// SGLD for every gaussian once all ranks' shards of the update have arrived (phase 1).
__global__ void __launch_bounds__(256) k_sgld_peer(float* __restrict__ params, int G, double lr_means, float noise_lr,
                                                    const float* __restrict__ eps_noise, const int* __restrict__ step_ptr,
                                                    unsigned long long seed, const int* mine, int N) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = peer_wait(mine, N, 1, *step_ptr);
  __syncthreads();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  // a block whose wait gave up adds no noise to parameters whose update may still be arriving
  if (!s_ok || g >= G) return;
  sgld_one(params, ParamLayout{G}, g, lr_means, noise_lr, eps_noise, *step_ptr, seed);
}

struct PeerAdamScalars {
  float w1, b2, w2, bc2_sqrt, eps, nss[7];
};

__device__ __forceinline__ float adam_one(float p, float g, float& m, float& v, const PeerAdamScalars& a, float nss) {
  m = __fadd_rn(m, __fmul_rn(a.w1, __fsub_rn(g, m)));
  v = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(__fmul_rn(a.w2, g), g));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bc2_sqrt), a.eps);
  return __fadd_rn(p, __fdiv_rn(__fmul_rn(nss, m), denom));
}

__device__ __forceinline__ float lr_seg(long long i, long long G, const float nss[7]) {
  return i < 3 * G ? nss[0] : i < 6 * G ? nss[1] : i < 10 * G ? nss[2] : i < 11 * G ? nss[3] : i < 14 * G ? nss[4] : nss[5];
}

// Shard [lo, hi) of the flat vector (lo, hi multiples of 4) plus, on the owner of w_b_raw,
// element 59G.  Every rank also sums the N per-rank losses (rank order) into loss_total.
__global__ void __launch_bounds__(256)
    k_adam_peer(PeerF params, PeerCF grads, float* __restrict__ m, float* __restrict__ v, int G, long long lo,
                long long hi, int N, int rank, int wb_owner, const int* __restrict__ step_ptr,
                const double* __restrict__ lr7, double beta1, double beta2, double eps, PeerCF loss,
                float* __restrict__ loss_total, PeerI flags, const float* own, int* mine) {
  __shared__ PeerAdamScalars s_a;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const int step = *step_ptr;
    // phase 0: every rank's gradient and loss are written; a block whose wait gave up skips its
    // part of the update (the status word reports it) rather than sum partial gradients
    s_ok = peer_wait(mine, N, 0, step);
    const double bc1 = 1.0 - pow(beta1, (double)step);
    const double bc2 = 1.0 - pow(beta2, (double)step);
    s_a.w1 = (float)(1.0 - beta1);
    s_a.b2 = (float)beta2;
    s_a.w2 = (float)(1.0 - beta2);
    s_a.bc2_sqrt = (float)sqrt(bc2);
    s_a.eps = (float)eps;
    for (int k = 0; k < 7; k++) s_a.nss[k] = (float)(-lr7[k] / bc1);
  }
  __syncthreads();
  const PeerAdamScalars a = s_a;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  // peer loops are unrolled to PEER_MAX with a guard (constant indices: the tables stay in the
  // parameter space); this rank's own buffers come as separate arguments
  auto scalar_update = [&](long long e, float nss) {
    float g = 0.f;
#pragma unroll
    for (int q = 0; q < PEER_MAX; ++q)
      if (q < N) g += grads.p[q][e];
    float mm = m[e], vv = v[e];
    const float pn = adam_one(own[e], g, mm, vv, a, nss);
    m[e] = mm;
    v[e] = vv;
#pragma unroll
    for (int q = 0; q < PEER_MAX; ++q)
      if (q < N) params.p[q][e] = pn;
  };
  if (tid == 0 && s_ok) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < PEER_MAX; ++q)
      if (q < N) s += loss.p[q][0];
    *loss_total = s;
    if (rank == wb_owner) scalar_update(59LL * G, a.nss[6]);
    // the last 1-3 elements of the vector when its length is not a multiple of 4
    for (long long e = hi / 4 * 4; e < hi; ++e) scalar_update(e, lr_seg(e, G, a.nss));
  }
  for (long long i = lo / 4 + tid; s_ok && i < hi / 4; i += stride) {
    float4 g4 = reinterpret_cast<const float4*>(grads.p[0])[i];
#pragma unroll
    for (int q = 1; q < PEER_MAX; ++q) {
      if (q < N) {
        const float4 h = reinterpret_cast<const float4*>(grads.p[q])[i];
        g4.x += h.x;
        g4.y += h.y;
        g4.z += h.z;
        g4.w += h.w;
      }
    }
    float4 p4 = reinterpret_cast<const float4*>(own)[i];
    float4 m4 = reinterpret_cast<const float4*>(m)[i];
    float4 v4 = reinterpret_cast<const float4*>(v)[i];
    const long long e = 4 * i;
    p4.x = adam_one(p4.x, g4.x, m4.x, v4.x, a, lr_seg(e, G, a.nss));
    p4.y = adam_one(p4.y, g4.y, m4.y, v4.y, a, lr_seg(e + 1, G, a.nss));
    p4.z = adam_one(p4.z, g4.z, m4.z, v4.z, a, lr_seg(e + 2, G, a.nss));
    p4.w = adam_one(p4.w, g4.w, m4.w, v4.w, a, lr_seg(e + 3, G, a.nss));
    reinterpret_cast<float4*>(m)[i] = m4;
    reinterpret_cast<float4*>(v)[i] = v4;
#pragma unroll
    for (int q = 0; q < PEER_MAX; ++q)
      if (q < N) reinterpret_cast<float4*>(params.p[q])[i] = p4;
  }
  // The block's stores (local and peer) are made visible system-wide before its count (barrier,
  // then thread 0's system-scope fence, cumulative over the block's stores); the last block to
  // count publishes phase 1 with release stores.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    int* ctr = mine + FLAG_COUNTER;
    if (atomicAdd(ctr, 1) == (int)gridDim.x - 1) {
      *ctr = 0;
      __threadfence_system();
      peer_signal(flags, rank, N, 1, *step_ptr);
    }
  }
}

}  // namespace tts

using namespace tts;

extern "C" size_t tts_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int tts_peer_alloc(size_t bytes, void** ptr) {
  TTS_REQUIRE(ptr && bytes > 0, "null output or zero size");
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return check_launch("peer buffer allocation");
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return check_launch("peer buffer clear");
  return TTS_OK;
}

extern "C" int tts_peer_free(void* ptr) {
  if (ptr && cudaFree(ptr) != cudaSuccess) return check_launch("peer buffer free");
  return TTS_OK;
}

extern "C" int tts_ipc_export(void* ptr, void* handle_out) {
  TTS_REQUIRE(ptr && handle_out, "null pointer");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return check_launch("cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return TTS_OK;
}

extern "C" int tts_ipc_open(const void* handle, void** ptr_out) {
  TTS_REQUIRE(handle && ptr_out, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return check_launch("cudaIpcOpenMemHandle");
  return TTS_OK;
}

extern "C" int tts_ipc_close(void* ptr) {
  if (ptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess) return check_launch("cudaIpcCloseMemHandle");
  return TTS_OK;
}

static int peer_table(int32_t* const* flags, int N, PeerI& f) {
  for (int q = 0; q < N; ++q) {
    TTS_REQUIRE(flags[q], "null peer flag pointer");
    f.p[q] = flags[q];
  }
  return TTS_OK;
}

static int peer_sync(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch, int sig, int wait,
                     void* stream) {
  TTS_REQUIRE(flags && epoch && N >= 1 && N <= PEER_MAX && rank >= 0 && rank < N && (phase == 0 || phase == 1),
              "bad peer barrier arguments");
  PeerI f = {};
  if (int rc = peer_table(flags, N, f)) return rc;
  k_peer_sync<<<1, 32, 0, as_stream(stream)>>>(f, flags[rank], rank, N, phase, epoch, sig, wait);
  return check_launch("peer_sync");
}

extern "C" int tts_peer_barrier(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch, void* stream) {
  return peer_sync(flags, rank, N, phase, epoch, 1, 1, stream);
}

extern "C" int tts_peer_signal(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch, void* stream) {
  return peer_sync(flags, rank, N, phase, epoch, 1, 0, stream);
}

extern "C" int tts_peer_wait(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch, void* stream) {
  return peer_sync(flags, rank, N, phase, epoch, 0, 1, stream);
}

extern "C" int tts_peer_sgld(float* params, int G, double lr_means, float noise_lr, const float* eps_noise,
                             const int32_t* step, uint64_t seed, int32_t* const* flags, int rank, int N, void* stream) {
  TTS_REQUIRE(params && step && flags && G >= 1 && N >= 1 && N <= PEER_MAX && rank >= 0 && rank < N,
              "bad peer SGLD arguments");
  PeerI f = {};
  if (int rc = peer_table(flags, N, f)) return rc;
  k_sgld_peer<<<(G + 255) / 256, 256, 0, as_stream(stream)>>>(params, G, lr_means, noise_lr, eps_noise, step, seed,
                                                              flags[rank], N);
  return check_launch("peer_sgld");
}

extern "C" int tts_adam_peer(float* const* params, const float* const* grads, float* m, float* v, int G, int sh_degree,
                             int rank, int N, const int32_t* step, const double* lr7, double beta1, double beta2,
                             double eps, const float* const* loss, float* loss_total, int32_t* const* flags,
                             void* stream) {
  TTS_REQUIRE(params && grads && loss && m && v && step && lr7 && loss_total && flags, "null pointer");
  TTS_REQUIRE(N >= 1 && N <= PEER_MAX && rank >= 0 && rank < N && G >= 1, "bad peer Adam arguments");
  PeerF P = {};
  PeerCF Gr = {}, L = {};
  for (int q = 0; q < N; ++q) {
    TTS_REQUIRE(params[q] && grads[q] && loss[q], "null peer pointer");
    TTS_REQUIRE(aligned16(params[q]) && aligned16(grads[q]), "peer buffers must be 16-byte aligned");
    P.p[q] = params[q];
    Gr.p[q] = grads[q];
    L.p[q] = loss[q];
  }
  TTS_REQUIRE(aligned16(m) && aligned16(v), "moments must be 16-byte aligned");
  // torch skips parameters without a gradient: the colour rest trains only with SH on
  const long long n = sh_degree > 0 ? 59LL * G : 14LL * G;
  const long long chunk = ((n + N - 1) / N + 3) / 4 * 4;
  const long long lo = std::min(n, (long long)rank * chunk), hi = std::min(n, lo + chunk);
  cudaStream_t st = as_stream(stream);
  long long blocks = (hi - lo) / 4 / 256 + 1;
  if (blocks > 148 * 8) blocks = 148 * 8;
  PeerI f = {};
  if (int rc = peer_table(flags, N, f)) return rc;
  k_adam_peer<<<(unsigned)blocks, 256, 0, st>>>(P, Gr, m, v, G, lo, hi, N, rank, N - 1, step, lr7, beta1, beta2, eps,
                                                L, loss_total, f, params[rank], flags[rank]);
  return check_launch("adam_peer");
}
