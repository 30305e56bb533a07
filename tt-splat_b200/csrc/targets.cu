// 8-bit training images on the device: the dataset loaders' [0, 1] floats are x / 255 of 8-bit
// pixels (spike/data.py reads PNG/JPEG frames), so a train step can keep its target images as
// uint8 (a quarter of the bytes to upload and hold) and expand them to the fp32 targets the loss
// reads, x / 255 correctly rounded: bit-identical to numpy's float32(x) / float32(255).
#include "common.cuh"

namespace tts {

// 16 bytes per thread and iteration: one 16-byte load, four 16-byte stores.
__global__ void __launch_bounds__(256) k_unit_from_u8(const uint4* __restrict__ src, long long n16,
                                                      float4* __restrict__ dst) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
    const uint4 w = __ldg(src + i);
    const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
      dst[4 * i + k] = make_float4(unit_from_byte(words[k] & 0xffu), unit_from_byte((words[k] >> 8) & 0xffu),
                                   unit_from_byte((words[k] >> 16) & 0xffu), unit_from_byte(words[k] >> 24));
  }
}

__global__ void k_unit_from_u8_tail(const uint8_t* __restrict__ src, long long beg, long long n, float* __restrict__ dst) {
  const long long i = beg + threadIdx.x;
  if (i < n) dst[i] = unit_from_byte(src[i]);
}

}  // namespace tts

using namespace tts;

extern "C" int tts_unit_from_u8(const uint8_t* src, long long n, float* dst, void* stream) {
  TTS_REQUIRE(n >= 0 && (n == 0 || (src && dst)), "bad unit_from_u8 arguments");
  TTS_REQUIRE(aligned16(src) && aligned16(dst), "src and dst must be 16-byte aligned");
  if (n == 0) return TTS_OK;
  cudaStream_t st = as_stream(stream);
  const long long n16 = n / 16;
  if (n16 > 0) {
    long long blocks = (n16 + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    k_unit_from_u8<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const uint4*>(src), n16,
                                                     reinterpret_cast<float4*>(dst));
  }
  if (n % 16) k_unit_from_u8_tail<<<1, 32, 0, st>>>(src, n16 * 16, n, dst);
  return check_launch("unit_from_u8");
}
