// Library-wide C ABI entry points: version, error reporting, device fault word.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace b200 {

__device__ int g_device_flags = 0;

static thread_local std::string t_last_error;

void set_last_error(const std::string& msg) { t_last_error = msg; }

int fail_arg(const char* what) {
  set_last_error(std::string("bad argument: ") + what);
  return B200_ERR_ARG;
}

int fail_unsupported(const char* what) {
  set_last_error(std::string("unsupported: ") + what);
  return B200_UNSUPPORTED;
}

int fail_cuda(cudaError_t err, const char* where) {
  set_last_error(std::string("CUDA error ") + cudaGetErrorName(err) + " (" +
                 cudaGetErrorString(err) + ") at " + where);
  return -(1000 + static_cast<int>(err));
}

int* device_flags_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_flags) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

int max_smem_optin() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 227 * 1024;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 227 * 1024;
  return n;
}

}  // namespace b200

extern "C" {

int b200_version(void) { return 10000; }

const char* b200_last_error(void) { return b200::t_last_error.c_str(); }

int b200_sm_count(void) { return b200::sm_count(); }

int b200_read_device_flags(void* stream, int* flags_out) {
  if (!flags_out) return b200::fail_arg("flags_out is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int zero = 0;
  B200_CUDA_CHECK(cudaMemcpyFromSymbolAsync(flags_out, b200::g_device_flags, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, s));
  B200_CUDA_CHECK(cudaMemcpyToSymbolAsync(b200::g_device_flags, &zero, sizeof(int), 0,
                                          cudaMemcpyHostToDevice, s));
  B200_CUDA_CHECK(cudaStreamSynchronize(s));
  return B200_OK;
}

}  // extern "C"
