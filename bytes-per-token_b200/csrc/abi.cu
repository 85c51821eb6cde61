// Status reporting shared by every entry point: the thread-local error message, the device-side error flag,
// and small cached device properties.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace bpt {

__device__ int g_device_error = 0;

namespace {
thread_local char t_message[512] = "";
}

int set_error(int status, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(t_message, sizeof(t_message), fmt, args);
  va_end(args);
  return status;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(BPT_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return BPT_OK;
}

int num_sms() {
  // Per device; a process drives at most a handful of GPUs.
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

void* tensor_map_encoder() {
  static void* fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return p;
  }();
  return fn;
}

int set_max_smem(const void* kernel, int bytes) {
  if (bytes <= 48 * 1024) return BPT_OK;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess)
    return set_error(BPT_ERR_CUDA, "cannot reserve %d bytes of shared memory: %s", bytes, cudaGetErrorString(err));
  return BPT_OK;
}

}  // namespace bpt

extern "C" int bpt_abi_version(void) { return BPT_ABI_VERSION; }

extern "C" const char* bpt_last_error(void) { return bpt::t_message; }

extern "C" int bpt_device_error(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  int value = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbol(&value, bpt::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (value != 0) cudaMemcpyToSymbol(bpt::g_device_error, &zero, sizeof(int));
  return value;
}
