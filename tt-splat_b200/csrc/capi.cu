// C ABI plumbing: version, thread-local error strings, the device status word.
#include <cstdio>
#include <string>

#include "common.cuh"

namespace tts {

__device__ int g_status = 0;

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TTS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return TTS_OK;
}

}  // namespace tts

extern "C" int tts_version(void) { return 1; }

extern "C" const char* tts_last_error(void) { return tts::t_last_error.c_str(); }

extern "C" int tts_read_status(int* status_host) {
  int zero = 0;
  if (cudaMemcpyFromSymbol(status_host, tts::g_status, sizeof(int)) != cudaSuccess) return tts::check_launch("read status");
  if (cudaMemcpyToSymbol(tts::g_status, &zero, sizeof(int)) != cudaSuccess) return tts::check_launch("clear status");
  return TTS_OK;
}
