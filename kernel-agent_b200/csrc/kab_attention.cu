// FP8 attention prefill: device status word of this translation unit.
#include "kab_host.h"

namespace kab {
__device__ unsigned g_attention_status = 0;

unsigned attention_device_status(bool clear, cudaStream_t stream) {
  unsigned v = 0;
  cudaMemcpyFromSymbolAsync(&v, g_attention_status, sizeof v, 0, cudaMemcpyDeviceToHost, stream);
  cudaStreamSynchronize(stream);
  if (clear) {
    const unsigned zero = 0;
    cudaMemcpyToSymbolAsync(g_attention_status, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, stream);
  }
  return v;
}
}  // namespace kab
