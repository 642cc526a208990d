// m3_scan_fwd_noalloc: the chunked-SSD forward for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc (or any allocating routine) at the point where
// they run the scan: a runtime that owns every byte of device memory through its own pool, a
// plugin loaded into a process whose allocator it must not touch, or a code path that runs while
// allocation is forbidden. m3_scan_fwd needs a float32 workspace that the caller normally
// allocates; this entry point instead uses a fixed scratch array that lives in the library's own
// device image (kNoAllocWorkspaceBytes per GPU that loads the library, held until process exit).
//
// The caller still provides every input and output tensor. Calls share the one scratch array, so
// calls on the same device that overlap on the GPU (different streams, no ordering between them)
// race on it; calls on one stream are ordered and safe. The scratch needs no clearing: the
// pre-pass writes every element it later reads.
#include <mutex>
#include <string>

#include "common.cuh"

namespace {

constexpr int64_t kNoAllocWorkspaceBytes = M3_NOALLOC_WORKSPACE_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocWorkspaceBytes / sizeof(float)];

std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current). Looked up once per
// device; the name g_noalloc_scratch in host code is only a host-side stand-in, never an address.
float* scratch_for(int device) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_scratch_ptr[device] = static_cast<float*>(ptr);
  }
  return g_scratch_ptr[device];
}

}  // namespace

namespace m3 {
int report_error(int code, const char* msg);
bool scan_umma_supported(const m3_scan_args& a);
int scan_umma_segments(const m3_scan_args& a);
}

extern "C" int m3_scan_fwd_noalloc(const m3_scan_args* args, void* stream) {
  if (args == nullptr) return m3_scan_fwd(nullptr, stream);  // reports the null argument
  m3_scan_args a = *args;
  int device = a.device;
  if (device >= 0) {
    if (device >= kMaxDevices || cudaSetDevice(device) != cudaSuccess) {
      return m3::report_error(M3_ERR_CUDA, "m3_scan_fwd_noalloc: cannot select the device");
    }
  } else if (cudaGetDevice(&device) != cudaSuccess || device >= kMaxDevices) {
    return m3::report_error(M3_ERR_CUDA, "m3_scan_fwd_noalloc: cannot query the current device");
  }
  a.workspace = m3_tensor{};
  int64_t need = m3_scan_workspace_bytes(&a);
  if (need < 0) return (int)(-need);
  // A sequence split into segments keeps per-segment records in the scratch too; when they do not
  // fit, scan in fewer segments (the results then agree with m3_scan_fwd within rounding).
  if (need > kNoAllocWorkspaceBytes && m3::scan_umma_supported(a)) {
    for (int n = m3::scan_umma_segments(a) - 1; n >= 1 && need > kNoAllocWorkspaceBytes; --n) {
      a.segments = n;
      need = m3_scan_workspace_bytes(&a);
    }
  }
  if (need > kNoAllocWorkspaceBytes) {
    const std::string msg = "m3_scan_fwd_noalloc: these sizes need " + std::to_string(need) +
                            " bytes of scratch, above the fixed limit of " +
                            std::to_string(kNoAllocWorkspaceBytes) +
                            " bytes (reduce batch x length, or use m3_scan_fwd with a caller workspace)";
    return m3::report_error(M3_ERR_SHAPE, msg.c_str());
  }
  if (need > 0) {
    float* scratch = scratch_for(device);
    if (scratch == nullptr) {
      return m3::report_error(M3_ERR_CUDA, "m3_scan_fwd_noalloc: cudaGetSymbolAddress failed");
    }
    a.workspace.data = scratch;
    a.workspace.dtype = M3_F32;
    a.workspace.ndim = 1;
    a.workspace.stride[0] = 1;
  }
  return m3_scan_fwd(&a, stream);
}
