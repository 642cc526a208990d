// Training kernels of the chunked SSD core: a forward that keeps the state at every chunk start,
// and its backward (the gradients autograd takes through mamba3/ops.py:716-816 in the reference's
// training path, whose GEMMs are the _BmmFloat products of ops.py:202-250).
//
// Core op, per (batch, head); rows i = (token t, rank r) flattened, chunks of kRows rows
// (kRows / R tokens); cum = inclusive cumsum of adt inside the chunk:
//   y_i     = e^{cum_t} (S_c q_i) + sum_j Wt_ij v_j,   Wt_ij = L_ts (q_i . k_j),
//             L_ts = e^{cum_t - cum_s} (s < t), diag_t (s = t), 0 (s > t)
//   S_{c+1} = e^{cum_last} S_c + sum_j e^{cum_last - cum_s} v_j k_j^T          (S: [P, N])
// q, k (k already times the trapezoid scale), v (rank values) are float32 here; the bias, rotation,
// scale, D skip, SiLU gate and rank sum around the core stay differentiable PyTorch ops.
//
// Backward, chunks in reverse with dS = dLoss/dS_{c+1} resident in shared memory:
//   dq_i = e^{cum_t} S_c^T dy_i + sum_j M_ij k_j,        M_ij = L_ts (dy_i . v_j)
//   dk_j = T_s dS^T v_j + sum_i M_ij q_i,                T_s = e^{cum_last - cum_s}
//   dv_j = T_s dS k_j + sum_i Wt_ij dy_i
//   dS_c = e^{cum_last} dS + sum_i e^{cum_t} dy_i q_i^T
//   dcum_t: e^{cum_t} dy_i . (S_c q_i); +- L_ts (q_i . k_j)(dy_i . v_j) for s < t;
//           e^{cum_last} <dS, S_c> + T_s v_j . (dS k_j) on the last token, - T_s v_j . (dS k_j) on s
//   ddiag_t = sum over same-token pairs (q_i . k_j)(dy_i . v_j);  dadt = reverse cumsum of dcum.
// One CTA (256 threads) per (batch, head); FP32 CUDA-core arithmetic from shared memory.
#include <string>

#include "common.cuh"

namespace m3 {
namespace ssdt {

constexpr int kRows = 32;      // rows per chunk
constexpr int kThreads = 256;
constexpr int kMaxN = 128, kMaxP = 64;

struct Smem {
  int N, P;
  int ldn, ldp;  // padded row strides (N + 1, P + 1): conflict-free column walks
  float *S, *dS, *Q, *K, *V, *dY, *A, *W, *M, *red;
};

__host__ __device__ inline size_t smem_floats(int N, int P, bool bwd) {
  const size_t st = (size_t)P * (N + 1);
  const size_t rows = (size_t)kRows * (N + 1) * 2 + (size_t)kRows * (P + 1) * 2;
  const size_t sq = (size_t)kRows * (kRows + 1) * 3;
  return st * (bwd ? 2 : 1) + rows + sq + 6 * kRows;  // red: cum, e^cum, T, dcum, ddiag, scalars
}

__device__ inline Smem carve(float* base, int N, int P, bool bwd) {
  Smem s;
  s.N = N, s.P = P, s.ldn = N + 1, s.ldp = P + 1;
  float* p = base;
  s.S = p, p += (size_t)P * s.ldn;
  s.dS = bwd ? p : nullptr;
  if (bwd) p += (size_t)P * s.ldn;
  s.Q = p, p += kRows * s.ldn;
  s.K = p, p += kRows * s.ldn;
  s.V = p, p += kRows * s.ldp;
  s.dY = p, p += kRows * s.ldp;
  s.A = p, p += kRows * (kRows + 1);
  s.W = p, p += kRows * (kRows + 1);
  s.M = p, p += kRows * (kRows + 1);
  s.red = p;  // [6][kRows]: cum, e^{cum}, T, dcum, ddiag, scalars
  return s;
}

// Row (t, r) of a [B, L, H, R, X] tensor.
__device__ __forceinline__ const float* row_ptr(const m3_tensor& t, int b, int tok, int h, int r) {
  return static_cast<const float*>(t.data) + b * t.stride[0] + (int64_t)tok * t.stride[1] + h * t.stride[2] +
         r * t.stride[3];
}
__device__ __forceinline__ float* row_ptr_w(const m3_tensor& t, int b, int tok, int h, int r) {
  return static_cast<float*>(t.data) + b * t.stride[0] + (int64_t)tok * t.stride[1] + h * t.stride[2] +
         r * t.stride[3];
}

// Loads the chunk's rows [row0, row0 + rows) of a [B, L, H, R, X] tensor into dst [kRows][ld]
// (rows past the end zero).
__device__ inline void load_rows(float* dst, int ld, const m3_tensor& t, int b, int h, int R, int row0, int rows,
                                 int X) {
  for (int o = threadIdx.x; o < kRows * X; o += kThreads) {
    const int i = o / X, x = o % X;
    float v = 0.0f;
    if (i < rows) {
      const int row = row0 + i;
      v = row_ptr(t, b, row / R, h, row % R)[x * t.stride[4]];
    }
    dst[i * ld + x] = v;
  }
}

// Per-token scalars of the chunk (warp 0): cum (inclusive), e^{cum}, e^{cum_last - cum}; returns
// nothing, fills red[0..2][token].
__device__ inline void chunk_scalars(const Smem& s, const m3_tensor& adt, int b, int h, int t0, int ntok) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float a = lane < ntok ? static_cast<const float*>(adt.data)[b * adt.stride[0] + (int64_t)(t0 + lane) *
                                                                          adt.stride[1] + h * adt.stride[2]]
                                : 0.0f;
    const float cum = warp_incl_scan(a, lane);
    const float last = __shfl_sync(0xffffffffu, cum, max(ntok - 1, 0));
    s.red[lane] = cum;
    s.red[kRows + lane] = lane < ntok ? expf(cum) : 0.0f;
    s.red[2 * kRows + lane] = lane < ntok ? expf(last - cum) : 0.0f;
  }
}

__device__ __forceinline__ float diag_of(const m3_tensor& d, int b, int t, int h) {
  return static_cast<const float*>(d.data)[b * d.stride[0] + (int64_t)t * d.stride[1] + h * d.stride[2]];
}

// Lower-triangular token weights L_ts (including diag_t on s == t).
__device__ __forceinline__ float lweight(const Smem& s, int t, int u, float dg) {
  return u < t ? expf(s.red[t] - s.red[u]) : (u == t ? dg : 0.0f);
}

__global__ void __launch_bounds__(kThreads) ssd_fwd_kernel(const m3_ssd_args a) {
  extern __shared__ float smem[];
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int N = a.d_state, P = a.head_dim, R = a.rank, L = a.length;
  const Smem s = carve(smem, N, P, false);
  const int tok_per = kRows / R;
  const int nchunk = (L + tok_per - 1) / tok_per;
  // initial state
  for (int o = tid; o < P * N; o += kThreads) {
    const int p = o / N, n = o % N;
    float v = 0.0f;
    if (a.initial_state.data) {
      const m3_tensor& t = a.initial_state;
      v = static_cast<const float*>(t.data)[b * t.stride[0] + h * t.stride[1] + p * t.stride[2] + n * t.stride[3]];
    }
    s.S[p * s.ldn + n] = v;
  }
  for (int c = 0; c < nchunk; ++c) {
    const int t0 = c * tok_per, ntok = min(tok_per, L - t0), rows = ntok * R;
    __syncthreads();
    // keep S_c for the backward
    {
      const m3_tensor& cs = a.chunk_states;
      float* dst = static_cast<float*>(cs.data) + b * cs.stride[0] + h * cs.stride[1] + (int64_t)c * cs.stride[2];
      for (int o = tid; o < P * N; o += kThreads) {
        const int p = o / N, n = o % N;
        dst[p * cs.stride[3] + n * cs.stride[4]] = s.S[p * s.ldn + n];
      }
    }
    load_rows(s.Q, s.ldn, a.q, b, h, R, t0 * R, rows, N);
    load_rows(s.K, s.ldn, a.k, b, h, R, t0 * R, rows, N);
    load_rows(s.V, s.ldp, a.v, b, h, R, t0 * R, rows, P);
    chunk_scalars(s, a.adt, b, h, t0, ntok);
    __syncthreads();
    // Wt = L o (Q K^T)
    for (int o = tid; o < kRows * kRows; o += kThreads) {
      const int i = o / kRows, j = o % kRows;
      float w = 0.0f;
      if (i < rows && j < rows) {
        const int ti = i / R, tj = j / R;
        const float lw = lweight(s, ti, tj, tj == ti ? diag_of(a.diag, b, t0 + ti, h) : 0.0f);
        if (lw != 0.0f) {
          float acc = 0.0f;
          for (int n = 0; n < N; ++n) acc = fmaf(s.Q[i * s.ldn + n], s.K[j * s.ldn + n], acc);
          w = lw * acc;
        }
      }
      s.W[i * (kRows + 1) + j] = w;
    }
    __syncthreads();
    // y_i = e^{cum_t} S_c q_i + sum_j Wt_ij v_j
    for (int o = tid; o < rows * P; o += kThreads) {
      const int i = o / P, p = o % P;
      float inter = 0.0f;
      for (int n = 0; n < N; ++n) inter = fmaf(s.S[p * s.ldn + n], s.Q[i * s.ldn + n], inter);
      float intra = 0.0f;
      for (int j = 0; j <= min(rows - 1, (i / R + 1) * R - 1); ++j)
        intra = fmaf(s.W[i * (kRows + 1) + j], s.V[j * s.ldp + p], intra);
      const int row = t0 * R + i;
      row_ptr_w(a.y, b, row / R, h, row % R)[p * a.y.stride[4]] = s.red[kRows + i / R] * inter + intra;
    }
    __syncthreads();
    // S_{c+1} = e^{cum_last} S_c + sum_j T_s v_j k_j^T
    const float lam = expf(s.red[ntok - 1]);
    for (int o = tid; o < P * N; o += kThreads) {
      const int p = o / N, n = o % N;
      float acc = 0.0f;
      for (int j = 0; j < rows; ++j) acc = fmaf(s.red[2 * kRows + j / R] * s.V[j * s.ldp + p], s.K[j * s.ldn + n], acc);
      s.S[p * s.ldn + n] = fmaf(lam, s.S[p * s.ldn + n], acc);
    }
  }
  __syncthreads();
  const m3_tensor& fs = a.final_state;
  for (int o = tid; o < P * N; o += kThreads) {
    const int p = o / N, n = o % N;
    static_cast<float*>(fs.data)[b * fs.stride[0] + h * fs.stride[1] + p * fs.stride[2] + n * fs.stride[3]] =
        s.S[p * s.ldn + n];
  }
}

__global__ void __launch_bounds__(kThreads) ssd_bwd_kernel(const m3_ssd_args a) {
  extern __shared__ float smem[];
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31;
  const int N = a.d_state, P = a.head_dim, R = a.rank, L = a.length;
  const Smem s = carve(smem, N, P, true);
  const int tok_per = kRows / R;
  const int nchunk = (L + tok_per - 1) / tok_per;
  float* dcum = s.red + 3 * kRows;     // [kRows] per token
  float* ddg = s.red + 4 * kRows;      // [kRows] per token (diag gradient)
  float* scal = s.red + 5 * kRows;     // [0]: <dS, S_c>
  // dS = gradient of the final state
  for (int o = tid; o < P * N; o += kThreads) {
    const int p = o / N, n = o % N;
    float v = 0.0f;
    if (a.dfinal.data) {
      const m3_tensor& t = a.dfinal;
      v = static_cast<const float*>(t.data)[b * t.stride[0] + h * t.stride[1] + p * t.stride[2] + n * t.stride[3]];
    }
    s.dS[p * s.ldn + n] = v;
  }
  for (int c = nchunk - 1; c >= 0; --c) {
    const int t0 = c * tok_per, ntok = min(tok_per, L - t0), rows = ntok * R;
    __syncthreads();
    {
      const m3_tensor& cs = a.chunk_states;
      const float* src = static_cast<const float*>(cs.data) + b * cs.stride[0] + h * cs.stride[1] +
                         (int64_t)c * cs.stride[2];
      for (int o = tid; o < P * N; o += kThreads) {
        const int p = o / N, n = o % N;
        s.S[p * s.ldn + n] = src[p * cs.stride[3] + n * cs.stride[4]];
      }
    }
    load_rows(s.Q, s.ldn, a.q, b, h, R, t0 * R, rows, N);
    load_rows(s.K, s.ldn, a.k, b, h, R, t0 * R, rows, N);
    load_rows(s.V, s.ldp, a.v, b, h, R, t0 * R, rows, P);
    load_rows(s.dY, s.ldp, a.dy, b, h, R, t0 * R, rows, P);
    chunk_scalars(s, a.adt, b, h, t0, ntok);
    if (tid < kRows) dcum[tid] = ddg[tid] = 0.0f;
    if (tid == 0) scal[0] = 0.0f;
    __syncthreads();
    // A = Q K^T, B = dY V^T; Wt = L o A, M = L o B; the decay and diagonal gradients of each pair.
    for (int o = tid; o < kRows * kRows; o += kThreads) {
      const int i = o / kRows, j = o % kRows;
      float wt = 0.0f, m = 0.0f;
      if (i < rows && j < rows && j / R <= i / R) {
        const int ti = i / R, tj = j / R;
        float qa = 0.0f, bb = 0.0f;
        for (int n = 0; n < N; ++n) qa = fmaf(s.Q[i * s.ldn + n], s.K[j * s.ldn + n], qa);
        for (int p = 0; p < P; ++p) bb = fmaf(s.dY[i * s.ldp + p], s.V[j * s.ldp + p], bb);
        if (tj == ti) {
          const float dg = diag_of(a.diag, b, t0 + ti, h);
          wt = dg * qa;
          m = dg * bb;
          atomicAdd(&ddg[ti], qa * bb);
        } else {
          const float lw = expf(s.red[ti] - s.red[tj]);
          wt = lw * qa;
          m = lw * bb;
          const float g = lw * qa * bb;
          atomicAdd(&dcum[ti], g);
          atomicAdd(&dcum[tj], -g);
        }
      }
      s.W[i * (kRows + 1) + j] = wt;
      s.M[i * (kRows + 1) + j] = m;
    }
    // <dS, S_c> (for the e^{cum_last} factor of the carried state)
    {
      float acc = 0.0f;
      for (int o = tid; o < P * N; o += kThreads) {
        const int p = o / N, n = o % N;
        acc = fmaf(s.dS[p * s.ldn + n], s.S[p * s.ldn + n], acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) atomicAdd(&scal[0], acc);
    }
    __syncthreads();
    // dq_i = e^{cum_t} S_c^T dy_i + sum_j M_ij k_j ; dk_j = T_s dS^T v_j + sum_i M_ij q_i
    for (int o = tid; o < rows * N; o += kThreads) {
      const int i = o / N, n = o % N;
      const int ti = i / R;
      float inter = 0.0f, sv = 0.0f;
      for (int p = 0; p < P; ++p) {
        inter = fmaf(s.S[p * s.ldn + n], s.dY[i * s.ldp + p], inter);
        sv = fmaf(s.dS[p * s.ldn + n], s.V[i * s.ldp + p], sv);
      }
      float dq = s.red[kRows + ti] * inter, dk = s.red[2 * kRows + ti] * sv;
      for (int j = 0; j < rows; ++j) {
        dq = fmaf(s.M[i * (kRows + 1) + j], s.K[j * s.ldn + n], dq);  // M_ij (zero above the token)
        dk = fmaf(s.M[j * (kRows + 1) + i], s.Q[j * s.ldn + n], dk);  // M_ji: rows j at or after i
      }
      const int row = t0 * R + i;
      row_ptr_w(a.dq, b, row / R, h, row % R)[n * a.dq.stride[4]] = dq;
      row_ptr_w(a.dk, b, row / R, h, row % R)[n * a.dk.stride[4]] = dk;
    }
    // dv_j = T_s dS k_j + sum_i Wt_ij dy_i ; dcum from the state term (v_j . dS k_j) and the inter
    // term (dy_i . S_c q_i)
    for (int o = tid; o < kRows * P; o += kThreads) {
      const int j = o / P, p = o % P;
      float dv = 0.0f, sdot = 0.0f, idot = 0.0f;
      if (j < rows) {
        const int tj = j / R;
        float dsk = 0.0f, sq = 0.0f;
        for (int n = 0; n < N; ++n) {
          dsk = fmaf(s.dS[p * s.ldn + n], s.K[j * s.ldn + n], dsk);
          sq = fmaf(s.S[p * s.ldn + n], s.Q[j * s.ldn + n], sq);
        }
        const float T = s.red[2 * kRows + tj];
        dv = T * dsk;
        for (int i = tj * R; i < rows; ++i) dv = fmaf(s.W[i * (kRows + 1) + j], s.dY[i * s.ldp + p], dv);
        sdot = T * s.V[j * s.ldp + p] * dsk;
        idot = s.red[kRows + tj] * s.dY[j * s.ldp + p] * sq;
        const int row = t0 * R + j;
        row_ptr_w(a.dv, b, row / R, h, row % R)[p * a.dv.stride[4]] = dv;
      }
      // rows j of one warp share j when P >= 32 (P a multiple of 32): reduce over the warp's p
      const float contrib = idot - sdot;  // on token tj
      const float last = sdot;            // on the last token
      if (P % 32 == 0) {
        const float c1 = warp_sum(contrib), c2 = warp_sum(last);
        if (lane == 0 && j < rows) {
          atomicAdd(&dcum[j / R], c1);
          atomicAdd(&dcum[ntok - 1], c2);
        }
      } else if (j < rows) {
        atomicAdd(&dcum[j / R], contrib);
        atomicAdd(&dcum[ntok - 1], last);
      }
    }
    __syncthreads();
    // dS_c = e^{cum_last} dS + sum_i e^{cum_t} dy_i q_i^T
    const float lam = expf(s.red[ntok - 1]);
    for (int o = tid; o < P * N; o += kThreads) {
      const int p = o / N, n = o % N;
      float acc = 0.0f;
      for (int i = 0; i < rows; ++i) acc = fmaf(s.red[kRows + i / R] * s.dY[i * s.ldp + p], s.Q[i * s.ldn + n], acc);
      s.dS[p * s.ldn + n] = fmaf(lam, s.dS[p * s.ldn + n], acc);
    }
    // dadt = reverse cumsum of dcum (with e^{cum_last} <dS, S_c> on the last token); ddiag
    if (tid < 32) {
      float v = lane < ntok ? dcum[lane] + (lane == ntok - 1 ? lam * scal[0] : 0.0f) : 0.0f;
      // reverse inclusive scan: sum over tokens u >= lane
      for (int off = 1; off < 32; off <<= 1) {
        const float nb = __shfl_down_sync(0xffffffffu, v, off);
        if (lane + off < 32) v += nb;
      }
      if (lane < ntok) {
        const m3_tensor& da = a.dadt;
        static_cast<float*>(da.data)[b * da.stride[0] + (int64_t)(t0 + lane) * da.stride[1] + h * da.stride[2]] = v;
        const m3_tensor& dd = a.ddiag;
        static_cast<float*>(dd.data)[b * dd.stride[0] + (int64_t)(t0 + lane) * dd.stride[1] + h * dd.stride[2]] =
            ddg[lane];
      }
    }
  }
  __syncthreads();
  if (a.dinitial.data) {
    const m3_tensor& t = a.dinitial;
    for (int o = tid; o < P * N; o += kThreads) {
      const int p = o / N, n = o % N;
      static_cast<float*>(t.data)[b * t.stride[0] + h * t.stride[1] + p * t.stride[2] + n * t.stride[3]] =
          s.dS[p * s.ldn + n];
    }
  }
}

}  // namespace ssdt

int report_error(int code, const char* msg);

static int ssd_check(const m3_ssd_args* args, bool bwd) {
  if (args == nullptr) return report_error(M3_ERR_ARGUMENT, "null argument struct");
  const m3_ssd_args& a = *args;
  if (a.batch <= 0 || a.length <= 0 || a.heads <= 0) return report_error(M3_ERR_SHAPE, "batch, length and heads must be positive");
  if (a.rank != 1 && a.rank != 2 && a.rank != 4 && a.rank != 8) return report_error(M3_ERR_SHAPE, "rank must be 1, 2, 4 or 8");
  if (a.d_state <= 0 || a.d_state > ssdt::kMaxN || a.head_dim <= 0 || a.head_dim > ssdt::kMaxP)
    return report_error(M3_ERR_SHAPE, "training kernels serve d_state <= 128 and head_dim <= 64");
  const m3_tensor* need[] = {&a.q, &a.k, &a.v, &a.adt, &a.diag, &a.chunk_states};
  for (const m3_tensor* t : need)
    if (t->data == nullptr || t->dtype != M3_F32) return report_error(M3_ERR_ARGUMENT, "q, k, v, adt, diag and chunk_states must be float32 tensors");
  if (a.initial_state.data && a.initial_state.dtype != M3_F32) return report_error(M3_ERR_ARGUMENT, "initial_state must be float32");
  if (!bwd) {
    if (!a.y.data || !a.final_state.data || a.y.dtype != M3_F32 || a.final_state.dtype != M3_F32)
      return report_error(M3_ERR_ARGUMENT, "y and final_state must be float32 outputs");
  } else {
    const m3_tensor* outs[] = {&a.dy, &a.dq, &a.dk, &a.dv, &a.dadt, &a.ddiag};
    for (const m3_tensor* t : outs)
      if (t->data == nullptr || t->dtype != M3_F32) return report_error(M3_ERR_ARGUMENT, "dy, dq, dk, dv, dadt and ddiag must be float32 tensors");
    if ((a.dfinal.data && a.dfinal.dtype != M3_F32) || (a.dinitial.data && a.dinitial.dtype != M3_F32))
      return report_error(M3_ERR_ARGUMENT, "dfinal and dinitial must be float32");
  }
  return M3_OK;
}

static int ssd_launch(const m3_ssd_args* args, void* stream, bool bwd) {
  const int rc = ssd_check(args, bwd);
  if (rc != M3_OK) return rc;
  const m3_ssd_args& a = *args;
  if (a.device >= 0 && cudaSetDevice(a.device) != cudaSuccess) return report_error(M3_ERR_CUDA, "cannot select the device");
  const size_t smem = ssdt::smem_floats(a.d_state, a.head_dim, bwd) * sizeof(float);
  auto kern = bwd ? ssdt::ssd_bwd_kernel : ssdt::ssd_fwd_kernel;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    kern<<<dim3(a.heads, a.batch), ssdt::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return report_error(M3_ERR_CUDA, (std::string("training kernel launch failed: ") + cudaGetErrorString(e)).c_str());
  return M3_OK;
}

}  // namespace m3

extern "C" {

int m3_ssd_chunk_rows(void) { return m3::ssdt::kRows; }

int m3_ssd_train_fwd(const m3_ssd_args* args, void* stream) { return m3::ssd_launch(args, stream, false); }

int m3_ssd_train_bwd(const m3_ssd_args* args, void* stream) { return m3::ssd_launch(args, stream, true); }

}  // extern "C"
