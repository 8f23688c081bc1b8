// Library-level C ABI: version, error channel, device status word.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace b2 {

namespace {
thread_local char g_last_error[1024] = "";
std::mutex g_handler_mu;
b2_error_handler_func g_handler = nullptr;
void* g_handler_data = nullptr;

constexpr int kMaxDevices = 64;
unsigned* g_status[kMaxDevices] = {};
std::mutex g_status_mu;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  b2_error_handler_func h;
  void* d;
  {
    std::lock_guard<std::mutex> lk(g_handler_mu);
    h = g_handler;
    d = g_handler_data;
  }
  if (h) h(g_last_error, d);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return B2_OK;
  return set_error(B2_ERR_CUDA, "[%s] CUDA error: %s", what, cudaGetErrorString(e));
}

// The status word is a module-scope device variable (one per device that
// loads the library, zero at load); its address is looked up once per device
// and cached for the life of the process, so the library is not meant to be
// used across a cudaDeviceReset (which unloads the module and invalidates
// every cached device address: the status word, the static decode scratch,
// the SiLU table).
__device__ unsigned g_status_word = 0u;

unsigned* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    g_status[dev] = static_cast<unsigned*>(p);
  }
  return g_status[dev];
}

// Opt a kernel into `bytes` of dynamic shared memory on the current device.
// The limit is the device's opt-in maximum minus the kernel's static shared
// memory.  Cached per (kernel, device).
int ensure_dynamic_smem(const void* fn, size_t bytes, const char* what) {
  static std::mutex mu;
  static const void* fns[64] = {};
  static size_t done[64][kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(B2_ERR_CUDA, "[%s] cannot query the current device", what);
  std::lock_guard<std::mutex> lk(mu);
  int slot = -1;
  for (int i = 0; i < 64; ++i) {
    if (fns[i] == fn) { slot = i; break; }
    if (!fns[i]) { fns[i] = fn; slot = i; break; }
  }
  if (slot >= 0 && done[slot][dev] >= bytes) return B2_OK;
  cudaFuncAttributes attr;
  cudaError_t e = cudaFuncGetAttributes(&attr, fn);
  if (e != cudaSuccess) return check_cuda(e, what);
  int optin = 0;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return check_cuda(e, what);
  const size_t limit = (size_t)optin - attr.sharedSizeBytes;
  if (bytes > limit)
    return set_error(B2_ERR_UNSUPPORTED, "[%s] needs %zu bytes of shared memory (limit %zu)", what, bytes, limit);
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)limit);
  if (e != cudaSuccess) return check_cuda(e, what);
  if (slot >= 0) done[slot][dev] = limit;
  return B2_OK;
}

}  // namespace b2

extern "C" {

const char* b2_version(void) { return "b2moe 0.1.0 (sm_100a)"; }

const char* b2_last_error(void) { return b2::g_last_error; }

void b2_set_error_handler(b2_error_handler_func handler, void* data) {
  std::lock_guard<std::mutex> lk(b2::g_handler_mu);
  b2::g_handler = handler;
  b2::g_handler_data = data;
}

int b2_device_status(unsigned* status, b2_stream_t stream) {
  B2_REQUIRE(status != nullptr, "[b2_device_status] status pointer is NULL");
  unsigned* d = b2::device_status_ptr();
  if (!d) return b2::set_error(B2_ERR_CUDA, "[b2_device_status] status word unavailable");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned h = 0;
  int rc = b2::check_cuda(cudaMemcpyAsync(&h, d, sizeof(unsigned), cudaMemcpyDeviceToHost, s),
                          "b2_device_status");
  if (rc) return rc;
  rc = b2::check_cuda(cudaMemsetAsync(d, 0, sizeof(unsigned), s), "b2_device_status");
  if (rc) return rc;
  rc = b2::check_cuda(cudaStreamSynchronize(s), "b2_device_status");
  if (rc) return rc;
  *status = h;
  return B2_OK;
}

}  // extern "C"
