// placeholder, replaced by the tcgen05 kernel
#include "scan_common.cuh"
namespace m3 {
// Device error word: set by any bounded wait that gave up (read with m3_device_error()).
__device__ int g_device_error = 0;
int read_device_error(int clear) {
  int host = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&host, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return host;
}
bool scan_umma_supported(const m3_scan_args&) { return false; }
cudaError_t launch_scan_umma(const m3_scan_args&, cudaStream_t) { return cudaErrorNotSupported; }
}
