// Projections of a decode step: y = x W^T (nn.Linear without bias) for a few rows of x (one row
// per decoded sequence), W [O][I] in the activation dtype. At batch 1 the in_proj / out_proj of a
// step are pure weight streams (59 MB and 26 MB per layer for d_model 2560); this kernel reads each
// weight row once with 16-byte loads, keeps every lane's loads of a block in flight before the
// multiply-adds, and accumulates in FP32 (bf16 x bf16 products are exact), rounding y once to the
// activation dtype as the library GEMM does. x is staged in shared memory. One warp per output
// row; 8 warps per CTA.
#include <string>

#include "common.cuh"

namespace m3 {

int report_error(int code, const char* msg);

namespace {

constexpr int kGemvThreads = 256;
constexpr int kRowsPerWarp = 1;
constexpr int kUnroll = 10;  // 256-element blocks whose loads are issued together (I <= 2560: all)

template <typename T> __device__ __forceinline__ void fma8(float& acc, uint4 w, uint4 x) {
  const T* we = reinterpret_cast<const T*>(&w);
  const T* xe = reinterpret_cast<const T*>(&x);
#pragma unroll
  for (int e = 0; e < 8; ++e) acc = fmaf(to_f(we[e]), to_f(xe[e]), acc);
}

template <typename T, int M>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const m3_gemv_args a) {
  extern __shared__ __align__(16) uint8_t gsm[];
  T* xs = reinterpret_cast<T*>(gsm);  // [M][I]
  const int I = (int)a.in_dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Launched as a programmatic dependent of the kernel before it in a decode step: release the next
  // kernel, pull this warp's weight rows (never written by any kernel) towards L2 while the
  // previous kernel finishes, then wait for it before touching x or y.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  {
    const int64_t op = ((int64_t)blockIdx.x * (kGemvThreads / 32) + warp) * kRowsPerWarp;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
      if (op + r < a.out_dim) {
        const T* row = static_cast<const T*>(a.w.data) + (op + r) * a.w.stride[0];
        for (int i = 64 * lane; i < I; i += 64 * 32)  // one 128-byte line per lane and step
          asm volatile("prefetch.global.L2 [%0];" ::"l"(row + i));
      }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const T* xp = static_cast<const T*>(a.x.data);
  for (int c = threadIdx.x; c < M * (I / 8); c += kGemvThreads) {
    const int m = c / (I / 8), i = 8 * (c % (I / 8));
    *reinterpret_cast<uint4*>(xs + m * I + i) = *reinterpret_cast<const uint4*>(xp + m * a.x.stride[0] + i);
  }
  __syncthreads();
  const int64_t o0 = ((int64_t)blockIdx.x * (kGemvThreads / 32) + warp) * kRowsPerWarp;
  if (o0 >= a.out_dim) return;
  const T* wp = static_cast<const T*>(a.w.data);
  const T* wr[kRowsPerWarp];
  bool ok[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    ok[r] = o0 + r < a.out_dim;
    wr[r] = wp + (ok[r] ? o0 + r : o0) * a.w.stride[0];
  }
  float acc[kRowsPerWarp][M];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;
  for (int base = 8 * lane; base < I; base += 256 * kUnroll) {
    uint4 w[kUnroll][kRowsPerWarp];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        const int i = base + 256 * u;
        w[u][r] = i < I ? __ldcs(reinterpret_cast<const uint4*>(wr[r] + i)) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = base + 256 * u;
      if (i < I) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * I + i);
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r) fma8<T>(acc[r][m], w[u][r], xv);
        }
      }
    }
  }
  T* yp = static_cast<T*>(a.y.data);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[r][m]);
      if (lane == 0 && ok[r]) yp[m * a.y.stride[0] + (o0 + r) * a.y.stride[1]] = from_f<T>(v);
    }
}

template <typename T, int M> cudaError_t launch_m(const m3_gemv_args& a, cudaStream_t stream) {
  const size_t smem = (size_t)M * a.in_dim * sizeof(T);
  cudaError_t e = cudaFuncSetAttribute(gemv_kernel<T, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t per_cta = (kGemvThreads / 32) * kRowsPerWarp;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.out_dim + per_cta - 1) / per_cta));
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<T, M>, a);
}

template <typename T> cudaError_t launch_t(const m3_gemv_args& a, cudaStream_t stream) {
  switch (a.rows) {
    case 1: return launch_m<T, 1>(a, stream);
    case 2: return launch_m<T, 2>(a, stream);
    case 3: return launch_m<T, 3>(a, stream);
    default: return launch_m<T, 4>(a, stream);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace m3

extern "C" int m3_gemv(const m3_gemv_args* args, void* stream) {
  if (args == nullptr) return m3::report_error(M3_ERR_ARGUMENT, "null argument struct");
  const m3_gemv_args& a = *args;
  if (a.rows < 1 || a.rows > 4 || a.out_dim <= 0 || a.in_dim <= 0 || a.in_dim % 8 != 0 || a.in_dim > 16384)
    return m3::report_error(M3_ERR_SHAPE, "m3_gemv: 1 to 4 rows, in_dim a positive multiple of 8 (<= 16384)");
  if (!a.x.data || !a.w.data || !a.y.data || a.x.dtype == M3_F32 || a.w.dtype != a.x.dtype || a.y.dtype != a.x.dtype)
    return m3::report_error(M3_ERR_DTYPE, "m3_gemv: x, w and y must share one 16-bit dtype");
  if (a.x.stride[1] != 1 || a.w.stride[1] != 1 || !m3::aligned16(a.x.data) || !m3::aligned16(a.w.data) ||
      a.x.stride[0] % 8 != 0 || a.w.stride[0] % 8 != 0)
    return m3::report_error(M3_ERR_LAYOUT, "m3_gemv: x and w rows must be contiguous and 16-byte aligned");
  if (a.device >= 0 && cudaSetDevice(a.device) != cudaSuccess)
    return m3::report_error(M3_ERR_CUDA, "m3_gemv: cannot select the device");
  const cudaError_t e = a.x.dtype == M3_BF16 ? m3::launch_t<__nv_bfloat16>(a, static_cast<cudaStream_t>(stream))
                                             : m3::launch_t<__half>(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return m3::report_error(M3_ERR_CUDA, (std::string("m3_gemv launch failed: ") + cudaGetErrorString(e)).c_str());
  return M3_OK;
}
