// rt_api.cu — library-wide entry points: ABI version, thread-local error text, the sticky device
// status word and the cached SM count.
#include <cstdlib>
#include <mutex>

#include "rt_common.cuh"

namespace rt {

static thread_local char t_error[512] = {0};

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return RT_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = getenv("RT_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

bool staged_enabled() {
  static const bool on = [] {
    const char *v = getenv("RT_ROW_STAGED");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}
bool pair_enabled() {
  static const bool on = [] {
    const char *v = getenv("RT_GEMM_PAIR");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

}  // namespace rt

using namespace rt;

extern "C" int rt_abi_version(void) { return RT_ABI_VERSION; }

extern "C" const char *rt_last_error(void) { return t_error; }

extern "C" int rt_device_status(uint32_t *out, int clear, void *stream) {
  if (out == nullptr) return fail(RT_ERR_INVALID_ARGUMENT, "rt_device_status: null output");
  cudaStream_t s = as_stream(stream);
  uint32_t value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, g_status, sizeof(value), 0,
                                            cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e != cudaSuccess) return fail(RT_ERR_CUDA, "rt_device_status: %s", cudaGetErrorString(e));
  *out = value;
  return RT_OK;
}

extern "C" int rt_sm_count(int *out) {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(RT_ERR_CUDA, "rt_sm_count: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(RT_ERR_UNSUPPORTED, "rt_sm_count: device %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int v = 0;
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(RT_ERR_CUDA, "rt_sm_count: %s", cudaGetErrorString(e));
    cached[dev] = v;
  }
  *out = cached[dev];
  return RT_OK;
}
