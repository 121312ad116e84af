// Library-wide entry points: error channel, ABI version, device error word.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

thread_local char g_last_error[1024] = {0};

// One word per device (module globals are instantiated per device context).
// Kernels OR DeviceErrorBits into it when a bounded wait gives up.
__device__ unsigned int g_device_error_word;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned int* g_err_addr[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};
int g_cc_major[kMaxDevices] = {0};

}  // namespace

namespace w8a8 {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = 0; }

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

unsigned int* device_error_word() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {
    fail(W8A8_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_error_word);
    if (e != cudaSuccess) {
      fail(W8A8_ERR_CUDA, "cudaGetSymbolAddress(error word) failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    g_err_addr[dev] = static_cast<unsigned int*>(p);
  }
  return g_err_addr[dev];
}

static void fill_device_facts(int dev) {
  if (g_sm_count[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) g_sm_count[dev] = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess) g_cc_major[dev] = v;
  }
}

int sm_count() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  fill_device_facts(dev);
  return g_sm_count[dev];
}

int device_cc_major() {
  int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  fill_device_facts(dev);
  return g_cc_major[dev];
}

}  // namespace w8a8

extern "C" {

const char* w8a8_last_error(void) { return g_last_error; }

int w8a8_abi_version(void) { return 1; }

int w8a8_device_error(int* code, int clear) {
  W8A8_REQUIRE(code != nullptr, W8A8_ERR_INVALID_ARG, "w8a8_device_error: code is null");
  unsigned int* addr = w8a8::device_error_word();
  if (!addr) return W8A8_ERR_CUDA;
  W8A8_CUDA_TRY(cudaDeviceSynchronize());
  unsigned int v = 0;
  W8A8_CUDA_TRY(cudaMemcpy(&v, addr, sizeof(v), cudaMemcpyDeviceToHost));
  if (clear) {
    unsigned int z = 0;
    W8A8_CUDA_TRY(cudaMemcpy(addr, &z, sizeof(z), cudaMemcpyHostToDevice));
  }
  *code = static_cast<int>(v);
  return W8A8_OK;
}

}  // extern "C"
