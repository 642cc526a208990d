// Residual add + RMSNorm between Mamba-3 blocks, one pass over the residual stream.
//
// The reference block is `hidden + mixer(norm(hidden))` (mamba3/model.py:487-520) with
// `norm(x) = F.rms_norm(x, w.to(x.dtype), eps).to(x.dtype)`, and under bf16 autocast the next
// in_proj then casts that fp32 result to bf16. Done as three PyTorch kernels that is a read and a
// write of the fp32 residual for the add, another read for the norm and a read / write for the
// cast. Here one kernel reads the residual and the mixer output once, writes the updated residual
// and writes the normalised row directly in the dtype its consumer reads:
//   r     = x (+ m)                      (fp32 arithmetic, r stored to out_x when given)
//   out_n = round(r * rsqrt(mean(r^2) + eps) * round(w))   (round: to out_n's dtype; w to x's dtype)
// One warp per row; rows whose elements are contiguous and 16-byte aligned take a float4 path.
#include "common.cuh"

namespace m3 {

int report_error(int code, const char* msg);

namespace {

constexpr int kNormThreads = 256;  // 8 rows per CTA

// Generic path: any dtypes and strides.
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(const m3_norm_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int D = a.dim;
  const int64_t xo = row * a.x.stride[0], mo = row * a.m.stride[0];
  float ss = 0.0f;
  // a 16-bit residual stream holds the rounded sum (the reference adds in that dtype)
  auto resid = [&](int i) {
    float r = ld_t(a.x, xo + i * a.x.stride[1]);
    if (a.m.data) {
      r += ld_t(a.m, mo + i * a.m.stride[1]);
      if (a.x.dtype == M3_BF16) r = rnd<__nv_bfloat16>(r);
      else if (a.x.dtype == M3_F16) r = rnd<__half>(r);
    }
    return r;
  };
  for (int i = lane; i < D; i += 32) {
    const float r = resid(i);
    ss += r * r;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / D + a.eps);
  for (int i = lane; i < D; i += 32) {
    const float r = resid(i);
    if (a.out_x.data) st_t(a.out_x, row * a.out_x.stride[0] + i * a.out_x.stride[1], r);
    // the weight is cast to the residual's dtype first (F.rms_norm(x, w.to(x.dtype)))
    float w = ld_t(a.w, i * a.w.stride[0]);
    if (a.x.dtype == M3_BF16) w = rnd<__nv_bfloat16>(w);
    else if (a.x.dtype == M3_F16) w = rnd<__half>(w);
    st_t(a.out_n, row * a.out_n.stride[0] + i * a.out_n.stride[1], r * inv * w);
  }
}

// Few rows (a decode step: one row per sequence): one CTA of kNormThreads per row, any dtypes.
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_rowblock(const m3_norm_args a) {
  __shared__ float part[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const int D = a.dim, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t xo = row * a.x.stride[0], mo = row * a.m.stride[0];
  auto resid = [&](int i) {
    float r = ld_t(a.x, xo + i * a.x.stride[1]);
    if (a.m.data) {
      r += ld_t(a.m, mo + i * a.m.stride[1]);
      if (a.x.dtype == M3_BF16) r = rnd<__nv_bfloat16>(r);
      else if (a.x.dtype == M3_F16) r = rnd<__half>(r);
    }
    return r;
  };
  float ss = 0.0f;
  for (int i = tid; i < D; i += kNormThreads) {
    const float r = resid(i);
    ss += r * r;
  }
  ss = warp_sum(ss);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += part[w];
  const float inv = rsqrtf(tot / D + a.eps);
  for (int i = tid; i < D; i += kNormThreads) {
    const float r = resid(i);
    if (a.out_x.data) st_t(a.out_x, row * a.out_x.stride[0] + i * a.out_x.stride[1], r);
    float w = ld_t(a.w, i * a.w.stride[0]);
    if (a.x.dtype == M3_BF16) w = rnd<__nv_bfloat16>(w);
    else if (a.x.dtype == M3_F16) w = rnd<__half>(w);
    st_t(a.out_n, row * a.out_n.stride[0] + i * a.out_n.stride[1], r * inv * w);
  }
}

// Few rows of one 16-bit dtype T throughout (x, m, out_x, out_n, w: a bf16 / fp16 model's decode
// step): one CTA per row, each thread holding up to kRowChunks 16-byte chunks of the row in
// registers; every load is issued before the block reduction, the row is read once.
constexpr int kRowChunks = 4;  // dim <= 4 * 8 * 256 = 8192
template <typename T>
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_row16(const m3_norm_args a) {
  __shared__ float part[kNormThreads / 32];
  // programmatic dependent of the projection before it: release the next kernel, wait for the
  // previous one before reading anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t row = blockIdx.x;
  const int D = a.dim, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* xp = static_cast<const T*>(a.x.data) + row * a.x.stride[0];
  const T* mp = a.m.data ? static_cast<const T*>(a.m.data) + row * a.m.stride[0] : nullptr;
  const T* wp = static_cast<const T*>(a.w.data);
  float r[kRowChunks][8];
  uint4 wv[kRowChunks];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = 8 * (tid + kNormThreads * c);
    uint4 xv = make_uint4(0u, 0u, 0u, 0u), mv = xv;
    wv[c] = xv;
    if (i < D) {
      xv = *reinterpret_cast<const uint4*>(xp + i);
      if (mp) mv = *reinterpret_cast<const uint4*>(mp + i);
      wv[c] = *reinterpret_cast<const uint4*>(wp + i);
    }
    const T* xe = reinterpret_cast<const T*>(&xv);
    const T* me = reinterpret_cast<const T*>(&mv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // the residual stream holds the rounded sum (the reference adds in this dtype)
      r[c][e] = mp ? rnd<T>(to_f(xe[e]) + to_f(me[e])) : to_f(xe[e]);
      ss += r[c][e] * r[c][e];
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += part[w];
  const float inv = rsqrtf(tot / D + a.eps);
  T* op = a.out_x.data ? static_cast<T*>(a.out_x.data) + row * a.out_x.stride[0] : nullptr;
  T* np = static_cast<T*>(a.out_n.data) + row * a.out_n.stride[0];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = 8 * (tid + kNormThreads * c);
    if (i >= D) continue;
    T xo[8], no[8];
    const T* we = reinterpret_cast<const T*>(&wv[c]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      xo[e] = from_f<T>(r[c][e]);
      no[e] = from_f<T>(r[c][e] * inv * to_f(we[e]));
    }
    if (op) *reinterpret_cast<uint4*>(op + i) = *reinterpret_cast<const uint4*>(xo);
    *reinterpret_cast<uint4*>(np + i) = *reinterpret_cast<const uint4*>(no);
  }
}

// Vector path: fp32 residual, dim % 128 == 0, contiguous 16-byte aligned rows; m and out_n 16-bit
// (TM / TN) or fp32. Each lane owns float4 groups lane, lane + 32, ... (NV of them, up to 16).
template <typename TM, typename TN, int NV>
__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_vec(const m3_norm_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const float* xp = static_cast<const float*>(a.x.data) + row * a.x.stride[0];
  const TM* mp = static_cast<const TM*>(a.m.data) + row * a.m.stride[0];
  float4 r[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) r[v] = reinterpret_cast<const float4*>(xp)[lane + 32 * v];
  if (a.m.data) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int e = 4 * (lane + 32 * v);
      r[v].x += to_f(mp[e]);
      r[v].y += to_f(mp[e + 1]);
      r[v].z += to_f(mp[e + 2]);
      r[v].w += to_f(mp[e + 3]);
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int v = 0; v < NV; ++v) ss += r[v].x * r[v].x + r[v].y * r[v].y + r[v].z * r[v].z + r[v].w * r[v].w;
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / a.dim + a.eps);
  if (a.out_x.data) {
    float* op = static_cast<float*>(a.out_x.data) + row * a.out_x.stride[0];
#pragma unroll
    for (int v = 0; v < NV; ++v) reinterpret_cast<float4*>(op)[lane + 32 * v] = r[v];
  }
  const float* wp = static_cast<const float*>(a.w.data);
  TN* np = static_cast<TN*>(a.out_n.data) + row * a.out_n.stride[0];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int e = 4 * (lane + 32 * v);
    const float4 w = reinterpret_cast<const float4*>(wp)[lane + 32 * v];
    np[e] = from_f<TN>(r[v].x * inv * w.x);
    np[e + 1] = from_f<TN>(r[v].y * inv * w.y);
    np[e + 2] = from_f<TN>(r[v].z * inv * w.z);
    np[e + 3] = from_f<TN>(r[v].w * inv * w.w);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename TM, typename TN>
cudaError_t launch_vec(const m3_norm_args& a, dim3 grid, cudaStream_t stream) {
  switch (a.dim / 128) {
    case 1: residual_rmsnorm_vec<TM, TN, 1><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 2: residual_rmsnorm_vec<TM, TN, 2><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 4: residual_rmsnorm_vec<TM, TN, 4><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 8: residual_rmsnorm_vec<TM, TN, 8><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 12: residual_rmsnorm_vec<TM, TN, 12><<<grid, kNormThreads, 0, stream>>>(a); break;
    case 16: residual_rmsnorm_vec<TM, TN, 16><<<grid, kNormThreads, 0, stream>>>(a); break;
    default: residual_rmsnorm_kernel<<<grid, kNormThreads, 0, stream>>>(a); break;
  }
  return cudaGetLastError();
}

template <typename TM>
cudaError_t launch_vec_n(const m3_norm_args& a, dim3 grid, cudaStream_t stream) {
  switch (a.out_n.dtype) {
    case M3_BF16: return launch_vec<TM, __nv_bfloat16>(a, grid, stream);
    case M3_F16: return launch_vec<TM, __half>(a, grid, stream);
    default: return launch_vec<TM, float>(a, grid, stream);
  }
}

bool is_float(int d) { return d == M3_F32 || d == M3_F16 || d == M3_BF16; }

}  // namespace
}  // namespace m3

extern "C" int m3_residual_rmsnorm(const m3_norm_args* args, void* stream) {
  using namespace m3;
  if (args == nullptr) return report_error(M3_ERR_ARGUMENT, "null argument struct");
  const m3_norm_args& a = *args;
  if (a.rows < 0 || a.dim <= 0) return report_error(M3_ERR_SHAPE, "rows must be >= 0 and dim positive");
  if (!a.x.data || !a.w.data || !a.out_n.data)
    return report_error(M3_ERR_ARGUMENT, "x, w and out_n are required");
  if (!is_float(a.x.dtype) || !is_float(a.w.dtype) || !is_float(a.out_n.dtype) ||
      (a.m.data && !is_float(a.m.dtype)) || (a.out_x.data && a.out_x.dtype != a.x.dtype))
    return report_error(M3_ERR_DTYPE, "unsupported dtype (out_x must match x)");
  if (a.x.ndim != 2 || a.out_n.ndim != 2 || a.w.ndim != 1 || (a.m.data && a.m.ndim != 2) ||
      (a.out_x.data && a.out_x.ndim != 2))
    return report_error(M3_ERR_SHAPE, "x, m, out_x, out_n are [rows, dim] and w is [dim]");
  if (a.out_n.data == a.x.data || (a.m.data && a.out_n.data == a.m.data))
    return report_error(M3_ERR_LAYOUT, "out_n must not alias x or m");
  if (a.device >= 0 && cudaSetDevice(a.device) != cudaSuccess)
    return report_error(M3_ERR_CUDA, "cudaSetDevice failed");
  if (a.rows == 0) return M3_OK;
  const dim3 grid((unsigned)((a.rows + kNormThreads / 32 - 1) / (kNormThreads / 32)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto rowvec = [](const m3_tensor& t, int elem) {
    return t.stride[1] == 1 && aligned16(t.data) && (t.stride[0] * elem) % 16 == 0;
  };
  const int msz = a.m.dtype == M3_F32 ? 4 : 2, nsz = a.out_n.dtype == M3_F32 ? 4 : 2;
  const bool vec = a.dim % 128 == 0 && a.dim <= 2048 && a.x.dtype == M3_F32 && a.w.dtype == M3_F32 &&
                   a.w.stride[0] == 1 && aligned16(a.w.data) && rowvec(a.x, 4) && rowvec(a.out_n, nsz) &&
                   (!a.m.data || (a.m.stride[1] == 1 && (reinterpret_cast<uintptr_t>(a.m.data) % (4 * msz)) == 0 &&
                                  (a.m.stride[0] * msz) % (4 * msz) == 0)) &&
                   (!a.out_x.data || rowvec(a.out_x, 4));
  cudaError_t e;
  const bool one16 = a.x.dtype != M3_F32 && a.w.dtype == a.x.dtype && a.out_n.dtype == a.x.dtype &&
                     (!a.m.data || a.m.dtype == a.x.dtype) && a.dim % 8 == 0 && a.dim <= 8 * kNormThreads * kRowChunks &&
                     a.w.stride[0] == 1 && aligned16(a.w.data) && rowvec(a.x, 2) && rowvec(a.out_n, 2) &&
                     (!a.m.data || rowvec(a.m, 2)) && (!a.out_x.data || rowvec(a.out_x, 2));
  if (a.rows < 8 * 148 && one16) {  // a 16-bit model's decode step
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.rows);
    cfg.blockDim = dim3(kNormThreads);
    cfg.stream = st;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    e = a.x.dtype == M3_BF16 ? cudaLaunchKernelEx(&cfg, residual_rmsnorm_row16<__nv_bfloat16>, a)
                             : cudaLaunchKernelEx(&cfg, residual_rmsnorm_row16<__half>, a);
  } else if (a.rows < 8 * 148) {  // too few rows for a warp each to fill the GPU
    residual_rmsnorm_rowblock<<<(unsigned)a.rows, kNormThreads, 0, st>>>(a);
    e = cudaGetLastError();
  } else if (vec) {
    switch (a.m.data ? a.m.dtype : M3_BF16) {
      case M3_BF16: e = launch_vec_n<__nv_bfloat16>(a, grid, st); break;
      case M3_F16: e = launch_vec_n<__half>(a, grid, st); break;
      default: e = launch_vec_n<float>(a, grid, st); break;
    }
  } else {
    residual_rmsnorm_kernel<<<grid, kNormThreads, 0, st>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return report_error(M3_ERR_CUDA, "residual_rmsnorm launch failed");
  return M3_OK;
}
