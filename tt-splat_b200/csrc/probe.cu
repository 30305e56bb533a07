// FP32 FMA-pipe throughput probe: the roofline denominator of the FP32-bound tile kernels
// (the render forward and backward run their (pixel, slot) loops as packed fma.rn.f32x2).
// Every thread runs PROBE_CHAINS independent packed-FMA chains, enough to cover the pipe's
// latency, over `iters` rounds; the grid fills every SM several times over.  One fma.rn.f32x2
// is 4 flops (two lanes, multiply + add), so a launch performs
//   blocks x PROBE_THREADS x iters x PROBE_CHAINS x 4 flops,
// which the caller divides by the launch's event-timed duration.
#include "common.cuh"

namespace tts {

constexpr int PROBE_THREADS = 256;
constexpr int PROBE_CHAINS = 8;

__global__ void __launch_bounds__(PROBE_THREADS) k_fma_probe(int iters, float seed, float* __restrict__ out) {
  f32x2 acc[PROBE_CHAINS];
  const f32x2 a = mk2(0.999f, 0.998f), b = mk2(seed * 1e-3f, seed * 2e-3f);
#pragma unroll
  for (int c = 0; c < PROBE_CHAINS; ++c) acc[c] = mk2(seed + c, seed - c);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < PROBE_CHAINS; ++c) acc[c] = fma2(a, acc[c], b);
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < PROBE_CHAINS; ++c) s += hsum2(acc[c]);
  out[blockIdx.x * PROBE_THREADS + threadIdx.x] = s;   // keeps the chains alive
}

}  // namespace tts

using namespace tts;

extern "C" long long tts_fma_probe_flops(int blocks, int iters) {
  if (blocks < 1 || iters < 1) return 0;
  return (long long)blocks * PROBE_THREADS * iters * PROBE_CHAINS * 4LL;
}

extern "C" int tts_fma_probe(int blocks, int iters, float* out, void* stream) {
  TTS_REQUIRE(blocks >= 1 && iters >= 1 && out, "bad probe arguments");
  k_fma_probe<<<(unsigned)blocks, PROBE_THREADS, 0, as_stream(stream)>>>(iters, 1.0f, out);
  return check_launch("fma_probe");
}
