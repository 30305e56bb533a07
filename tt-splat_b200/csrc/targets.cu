// 8-bit training images on the device: the dataset loaders' [0, 1] floats are x / 255 of 8-bit
// pixels (spike/data.py reads PNG/JPEG frames), so a train step can keep its target images as
// uint8 (a quarter of the bytes to upload and hold) and expand them to the fp32 targets the loss
// reads, x / 255 correctly rounded: bit-identical to numpy's float32(x) / float32(255).
#include "common.cuh"

namespace tts {

// Four bytes in, one float4 out per thread and iteration: a warp reads 128 contiguous bytes and
// writes 512 contiguous bytes.
__global__ void __launch_bounds__(256) k_unit_from_u8(const uchar4* __restrict__ src, long long n4,
                                                      float4* __restrict__ dst) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const uchar4 b = __ldg(src + i);
    dst[i] = make_float4(unit_from_byte(b.x), unit_from_byte(b.y), unit_from_byte(b.z), unit_from_byte(b.w));
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
  const long long n4 = n / 4;
  if (n4 > 0) {
    long long blocks = (n4 + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_unit_from_u8<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const uchar4*>(src), n4,
                                                     reinterpret_cast<float4*>(dst));
  }
  if (n % 4) k_unit_from_u8_tail<<<1, 32, 0, st>>>(src, n4 * 4, n, dst);
  return check_launch("unit_from_u8");
}
