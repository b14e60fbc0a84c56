// Host-side status plumbing of the C ABI: last-error text per host thread and
// the device status word that bounded waits and index checks set.
#include <mutex>

#include "common.cuh"

namespace sc {

// One word per device; kernels get its address as an argument.
__device__ unsigned int g_device_status = 0;

namespace {
thread_local int t_last_code = SC_OK;
thread_local char t_last_text[512] = "";

constexpr int kMaxDevices = 64;
unsigned int* g_status_addr[kMaxDevices] = {};
std::mutex g_status_mutex;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  t_last_code = code;
  va_list args;
  va_start(args, fmt);
  vsnprintf(t_last_text, sizeof(t_last_text), fmt, args);
  va_end(args);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(SC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return SC_OK;
}

unsigned int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (g_status_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_addr[dev] = static_cast<unsigned int*>(p);
  }
  return g_status_addr[dev];
}

}  // namespace sc

extern "C" int sc_version(void) { return 100; }

extern "C" int sc_last_error(char* buf, int n) {
  if (buf != nullptr && n > 0) snprintf(buf, (size_t)n, "%s", sc::t_last_text);
  return sc::t_last_code;
}

extern "C" int sc_device_status(unsigned int* status, void* stream) {
  if (status == nullptr) return sc::set_error(SC_ERR_INVALID, "sc_device_status: null output");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int* word = sc::device_status_word();
  if (word == nullptr)
    return sc::set_error(SC_ERR_CUDA, "sc_device_status: no device status word");
  cudaError_t err =
      cudaMemcpyAsync(status, word, sizeof(unsigned int), cudaMemcpyDeviceToHost, s);
  if (err == cudaSuccess) err = cudaMemsetAsync(word, 0, sizeof(unsigned int), s);
  if (err == cudaSuccess) err = cudaStreamSynchronize(s);
  if (err != cudaSuccess)
    return sc::set_error(SC_ERR_CUDA, "sc_device_status: %s", cudaGetErrorString(err));
  return SC_OK;
}
