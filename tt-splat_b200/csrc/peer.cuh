// NVLink peer-memory flags of the multi-GPU optimizer step (shared by the peer kernels and the
// relocation kernel, which waits for the step's phase 1 before its SGLD phase).
#pragma once
#include "common.cuh"

namespace tts {

constexpr int PEER_MAX = 8;
constexpr int STATUS_PEER_TIMEOUT = 4;

struct PeerF {
  float* p[PEER_MAX];
};
struct PeerCF {
  const float* p[PEER_MAX];
};
struct PeerI {
  int* p[PEER_MAX];
};

// Flags: flags_r[phase * PEER_MAX + q] on rank r holds the last epoch rank q reached in `phase`;
// flags_r[2 * PEER_MAX] counts the finished blocks of this rank's Adam kernel.
constexpr int FLAG_COUNTER = 2 * PEER_MAX;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Store `epoch` into every rank's flag slot for (phase, rank) with system-scope release
// semantics: this thread's earlier writes, and those ordered before them, are visible to any
// thread that acquires the flag.
__device__ __forceinline__ void peer_signal(PeerI flags, int rank, int N, int phase, int epoch) {
#pragma unroll
  for (int q = 0; q < PEER_MAX; ++q)
    if (q < N) st_release_sys(flags.p[q] + phase * PEER_MAX + rank, epoch);
}

// Wait (one thread, iteration limit) until all N ranks reached `epoch` in `phase` (acquire).
// Returns false, after recording the timeout in the status word, when a rank never arrived.
__device__ __forceinline__ bool peer_wait(const int* mine, int N, int phase, int epoch) {
  for (int q = 0; q < N; ++q) {
    const int* src = mine + phase * PEER_MAX + q;
    int it = 0;
    while (ld_acquire_sys(src) < epoch) {
      if (++it > (1 << 22)) {
        atomicOr(&g_status, STATUS_PEER_TIMEOUT);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

}  // namespace tts
