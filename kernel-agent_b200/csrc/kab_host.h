// Host-side helpers shared by the library's translation units: the thread-local error
// message, argument checks and CUDA error mapping.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/kab.h"

namespace kab {

// Records the message of a failing call (kab_last_error) and returns `code`.
int fail(int code, const char* fmt, ...);
// KAB_OK, or KAB_ECUDA with the runtime's message when the last launch failed.
int check_launch(const char* what);
// The number of SMs of the current device (cached per device).
int sm_count();
// True when `p` is a multiple of `bytes`.
inline bool aligned(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline int dtype_bytes(int dtype) { return dtype == KAB_F32 ? 4 : 2; }
inline bool valid_dtype(int dtype) {
  return dtype == KAB_F32 || dtype == KAB_BF16 || dtype == KAB_F16;
}

// Per-translation-unit device status readers (each TU with waiting kernels owns a word).
unsigned gemm_device_status(bool clear, cudaStream_t stream);
unsigned attention_device_status(bool clear, cudaStream_t stream);

}  // namespace kab

#define KAB_REQUIRE(cond, ...)                         \
  do {                                                 \
    if (!(cond)) return ::kab::fail(KAB_EINVAL, __VA_ARGS__); \
  } while (0)
