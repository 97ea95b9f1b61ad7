// Library-wide entry points: errors, version, device checks and device status, and the CUDA
// IPC mapping of an output buffer into the other ranks' address spaces.
#include <cudaTypedefs.h>

#include "kab_host.h"

#include <cstring>
#include <mutex>
#include <vector>

namespace kab {

namespace {
thread_local std::string t_error;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(KAB_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return KAB_OK;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

}  // namespace kab

extern "C" {

const char* kab_last_error(void) { return kab::t_error.c_str(); }

int kab_abi_version(void) { return KAB_ABI_VERSION; }

int kab_device_check(int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0)
    return kab::fail(KAB_EUNSUPPORTED, "no CUDA device");
  if (device < 0 || device >= count)
    return kab::fail(KAB_EINVAL, "device %d out of range (%d devices)", device, count);
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10 || minor != 0)
    return kab::fail(KAB_EUNSUPPORTED,
                     "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                     major, minor);
  return KAB_OK;
}

int kab_device_status(unsigned* bits, int clear, void* stream) {
  KAB_REQUIRE(bits != nullptr, "bits is null");
  const cudaStream_t s = kab::as_stream(stream);
  unsigned v = kab::gemm_device_status(clear != 0, s) | kab::attention_device_status(clear != 0, s);
  const cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return kab::fail(KAB_ECUDA, "device status: %s", cudaGetErrorString(e));
  *bits = v;
  return KAB_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == KAB_IPC_HANDLE_BYTES, "IPC handle size");

int kab_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  KAB_REQUIRE(ptr != nullptr && handle != nullptr && offset != nullptr, "null pointer");
  static PFN_cuMemGetAddressRange_v3020 range = nullptr;
  if (range == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return kab::fail(KAB_EUNSUPPORTED, "cuMemGetAddressRange is unavailable");
    range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return kab::fail(KAB_EINVAL, "not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return kab::fail(KAB_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof h);
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return KAB_OK;
}

int kab_ipc_open(const void* handle, void** base) {
  KAB_REQUIRE(handle != nullptr && base != nullptr, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return kab::fail(KAB_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return KAB_OK;
}

int kab_ipc_close(void* base) {
  KAB_REQUIRE(base != nullptr, "null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return kab::fail(KAB_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return KAB_OK;
}

}  // extern "C"
