// Library-wide C ABI pieces: error reporting, device error word, SM count.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {
thread_local char t_last_error[512] = "";
__device__ int g_device_error = 0;

constexpr int kMaxDevices = 64;
int* g_err_ptr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
std::mutex g_mu;
}  // namespace

int csahca_set_cuda_error(cudaError_t e, const char* what) {
  std::snprintf(t_last_error, sizeof(t_last_error), "CUDA error %d (%s) in %s", int(e), cudaGetErrorString(e), what);
  return CSAHCA_ECUDA;
}

int csahca_set_arg_error(const char* msg) {
  std::snprintf(t_last_error, sizeof(t_last_error), "%s", msg);
  return CSAHCA_EINVAL;
}

int csahca_set_unsupported(const char* msg) {
  std::snprintf(t_last_error, sizeof(t_last_error), "%s", msg);
  return CSAHCA_EUNSUPPORTED;
}

int* csahca_device_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int csahca_num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

extern "C" const char* csahca_last_error(void) { return t_last_error; }

extern "C" const char* csahca_version(void) { return "csahca_b200 0.1.0 (sm_100a)"; }

extern "C" int csahca_read_device_error(int* code) {
  if (code == nullptr) return csahca_set_arg_error("code must not be NULL");
  *code = 0;
  int* p = csahca_device_error_ptr();
  if (p == nullptr) return csahca_set_cuda_error(cudaErrorInvalidDevice, "cudaGetSymbolAddress");
  CSAHCA_RETURN_IF_CUDA(cudaDeviceSynchronize());
  CSAHCA_RETURN_IF_CUDA(cudaMemcpy(code, p, sizeof(int), cudaMemcpyDeviceToHost));
  const int zero = 0;
  CSAHCA_RETURN_IF_CUDA(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
  return CSAHCA_OK;
}
