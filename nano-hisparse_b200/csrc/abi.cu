// Library information, error reporting and the mapped-host alias query of the
// libhisparse C ABI (declarations in include/hisparse.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace hs {

namespace {
thread_local char g_error[512] = "";
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
}  // namespace

int set_error(int status, const char *fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
  return status;
}

int check_launch(const char *what) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(HS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return HS_OK;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int reserve_smem(const void *func, size_t bytes, const char *what) {
  if (bytes <= 48 * 1024) return HS_OK;
  struct Entry {
    const void *func;
    int device;
    size_t bytes;
  };
  static std::mutex lock;
  static Entry table[256];
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> guard(lock);
  for (int i = 0; i < used; ++i)
    if (table[i].func == func && table[i].device == dev && table[i].bytes >= bytes) return HS_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return set_error(HS_ERR_CUDA, "%s: cannot reserve %zu bytes of shared memory", what, bytes);
  }
  for (int i = 0; i < used; ++i)
    if (table[i].func == func && table[i].device == dev) {
      table[i].bytes = bytes;
      return HS_OK;
    }
  if (used < 256) table[used++] = Entry{func, dev, bytes};
  return HS_OK;
}

}  // namespace hs

extern "C" int hs_version(void) { return HS_ABI_VERSION; }

extern "C" const char *hs_status_string(int status) {
  switch (status) {
    case HS_OK: return "ok";
    case HS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case HS_ERR_UNSUPPORTED: return "unsupported";
    case HS_ERR_WORKSPACE: return "workspace too small";
    case HS_ERR_CUDA: return "CUDA error";
    case HS_ERR_NOT_MAPPED: return "host memory is not mapped for the device";
  }
  return "unknown status";
}

extern "C" const char *hs_last_error(void) { return hs::g_error; }

// Replaces MappedHost (nano_hisparse/row_kernels.py:10-32): the reference asks
// the driver for CU_POINTER_ATTRIBUTE_DEVICE_POINTER of a torch-pinned tensor.
extern "C" int hs_host_device_pointer(const void *host, void **device_alias) {
  if (!host || !device_alias)
    return hs::set_error(HS_ERR_INVALID_ARGUMENT, "host alias: null pointer");
  cudaPointerAttributes attr{};
  const cudaError_t err = cudaPointerGetAttributes(&attr, host);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return hs::set_error(HS_ERR_NOT_MAPPED, "cannot map pinned host allocation to CUDA: %s",
                         cudaGetErrorString(err));
  }
  if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
    return hs::set_error(HS_ERR_NOT_MAPPED, "row gather requires pinned host backing");
  *device_alias = attr.devicePointer;
  return HS_OK;
}
