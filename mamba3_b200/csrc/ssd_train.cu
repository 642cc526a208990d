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
// Backward, with G_c = dLoss/dS_{c+1} (the gradient of chunk c's end state):
//   dq_i = e^{cum_t} S_c^T dy_i + sum_j M_ij k_j,        M_ij = L_ts (dy_i . v_j)
//   dk_j = T_s G_c^T v_j + sum_i M_ij q_i,               T_s = e^{cum_last - cum_s}
//   dv_j = T_s G_c k_j + sum_i Wt_ij dy_i
//   dS_c = e^{cum_last} G_c + sum_i e^{cum_t} dy_i q_i^T  (= G_{c-1})
//   dcum_t: e^{cum_t} dy_i . (S_c q_i); +- L_ts (q_i . k_j)(dy_i . v_j) for s < t;
//           e^{cum_last} <G_c, S_c> + T_s v_j . (G_c k_j) on the last token, - T_s v_j . (G_c k_j) on s
//   ddiag_t = sum over same-token pairs (q_i . k_j)(dy_i . v_j);  dadt = reverse cumsum of dcum.
//
// Chunk-parallel schedule (only the two carries are sequential, as elementwise scans):
//   forward:  chunk_delta (per chunk: sum_j T_s v_j k_j^T and e^{cum_last})
//             -> state_scan (per (batch, head): S_{c+1} = e^{cum_last} S_c + delta_c, S_c kept)
//             -> chunk_output (per chunk: y)
//   backward: chunk_delta (per chunk: sum_i e^{cum_t} dy_i q_i^T)
//             -> grad_scan (per (batch, head), reverse: G_c kept, <G_c, S_c>)
//             -> chunk_grads (per chunk: dq, dk, dv, dadt, ddiag)
// Per-chunk kernels: one CTA (256 threads) per (chunk, head, batch), FP32 CUDA-core products from
// shared memory, each thread accumulating a register tile with 128-bit shared loads.
#include <string>

#include "common.cuh"

namespace m3 {
namespace ssdt {

constexpr int kRows = 32;  // rows per chunk
constexpr int kThreads = 256;
constexpr int kMaxN = 128, kMaxP = 64;

// Offset of row (t, r) of a [B, L, H, R, X] tensor.
__device__ __forceinline__ int64_t row_off(const m3_tensor& t, int b, int tok, int h, int r) {
  return b * t.stride[0] + (int64_t)tok * t.stride[1] + h * t.stride[2] + r * t.stride[3];
}

// Loads rows [row0, row0 + rows) (flattened (token, rank)) of a [B, L, H, R, X] float tensor with
// contiguous, 16-byte aligned rows into dst [kRows][ld], scaled per row by scale[row / R] when given;
// rows past `rows` are zero. One warp per row, 16-byte loads (X <= 128).
__device__ inline void load_rows(float* dst, int ld, const m3_tensor& t, int b, int h, int R, int row0, int rows,
                                 int X, const float* scale = nullptr) {
  const float* base = static_cast<const float*>(t.data);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < kRows; i += kThreads / 32) {
    if (4 * lane >= X) continue;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < rows) {
      const int row = row0 + i;
      v = *reinterpret_cast<const float4*>(base + row_off(t, b, row / R, h, row % R) + 4 * lane);
      if (scale) {
        const float f = scale[i / R];
        v.x *= f, v.y *= f, v.z *= f, v.w *= f;
      }
    }
    *reinterpret_cast<float4*>(dst + i * ld + 4 * lane) = v;
  }
}

// Per-token scalars of a chunk (warp 0): red[0..] cum, red[32..] e^{cum}, red[64..] e^{cum_last - cum}
// (zero past the sequence end).
__device__ inline void chunk_scalars(float* red, const m3_tensor& adt, int b, int h, int t0, int ntok) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float a = lane < ntok ? static_cast<const float*>(adt.data)[b * adt.stride[0] + (int64_t)(t0 + lane) *
                                                                          adt.stride[1] + h * adt.stride[2]]
                                : 0.0f;
    const float cum = warp_incl_scan(a, lane);
    const float last = __shfl_sync(0xffffffffu, cum, max(ntok - 1, 0));
    red[lane] = cum;
    red[kRows + lane] = lane < ntok ? expf(cum) : 0.0f;
    red[2 * kRows + lane] = lane < ntok ? expf(last - cum) : 0.0f;
  }
}

// Register-tiled product: acc[t][u] += sum_k A(mi(t), k) B(k, nj(u)) over k in [0, K) (K a multiple
// of 4). A is stored k-major (A(m, k) = A[k * lda + m]) when AK, else m-major (A[m * lda + k]); B
// likewise with BK (B(k, n) = B[k * ldb + n]) or n-major (B[n * ldb + k]). Tile indices: a k-major
// operand is read in 16-byte groups, mi(t) = mb + (t / 4) ms + t % 4; an m-major one row by row,
// mi(t) = mb + t ms (nj likewise). Threads of a warp take adjacent mb / nb, so their 16-byte shared
// loads fall on adjacent addresses (k-major) or on rows one padded stride apart (m-/n-major):
// no bank conflicts.
template <int TM, int TN, bool AK, bool BK>
__device__ __forceinline__ void mm(float (&acc)[TM][TN], const float* A, int lda, const float* B, int ldb, int K,
                                   int mb, int ms, int nb, int ns) {
  static_assert(!AK || TM % 4 == 0, "k-major A is read in groups of four");
  static_assert(!BK || TN % 4 == 0, "k-major B is read in groups of four");
  for (int k = 0; k < K; k += 4) {
    float a[4][TM], bb[4][TN];
    if constexpr (AK) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int t = 0; t < TM; t += 4) {
          const float4 v = *reinterpret_cast<const float4*>(A + (k + kk) * lda + mb + (t / 4) * ms);
          a[kk][t] = v.x, a[kk][t + 1] = v.y, a[kk][t + 2] = v.z, a[kk][t + 3] = v.w;
        }
    } else {
#pragma unroll
      for (int t = 0; t < TM; ++t) {
        const float4 v = *reinterpret_cast<const float4*>(A + (mb + t * ms) * lda + k);
        a[0][t] = v.x, a[1][t] = v.y, a[2][t] = v.z, a[3][t] = v.w;
      }
    }
    if constexpr (BK) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int u = 0; u < TN; u += 4) {
          const float4 v = *reinterpret_cast<const float4*>(B + (k + kk) * ldb + nb + (u / 4) * ns);
          bb[kk][u] = v.x, bb[kk][u + 1] = v.y, bb[kk][u + 2] = v.z, bb[kk][u + 3] = v.w;
        }
    } else {
#pragma unroll
      for (int u = 0; u < TN; ++u) {
        const float4 v = *reinterpret_cast<const float4*>(B + (nb + u * ns) * ldb + k);
        bb[0][u] = v.x, bb[1][u] = v.y, bb[2][u] = v.z, bb[3][u] = v.w;
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int t = 0; t < TM; ++t)
#pragma unroll
        for (int u = 0; u < TN; ++u) acc[t][u] = fmaf(a[kk][t], bb[kk][u], acc[t][u]);
  }
}

// Tile index of element t: grouped (k-major reads) or row-wise.
__device__ __forceinline__ int gidx(int base, int stride, int t) { return base + (t >> 2) * stride + (t & 3); }
__device__ __forceinline__ int ridx(int base, int stride, int t) { return base + t * stride; }

template <int TM, int TN> __device__ __forceinline__ void zero(float (&acc)[TM][TN]) {
#pragma unroll
  for (int t = 0; t < TM; ++t)
#pragma unroll
    for (int u = 0; u < TN; ++u) acc[t][u] = 0.0f;
}

// Padded shared row strides (multiples of 4 floats; the +4 staggers rows across banks).
__host__ __device__ constexpr int ldn(int N) { return N + 4; }
__host__ __device__ constexpr int ldp(int P) { return P + 4; }
constexpr int kLdr = kRows + 4;

struct Geo {
  int N, P, R, L, tok_per, nchunk;
};
__device__ __forceinline__ Geo geo(const m3_ssd_args& a) {
  Geo g;
  g.N = a.d_state, g.P = a.head_dim, g.R = a.rank, g.L = a.length;
  g.tok_per = kRows / g.R;
  g.nchunk = (g.L + g.tok_per - 1) / g.tok_per;
  return g;
}

// Chunk-state buffer [B][H][nchunk][P][N] (contiguous).
__device__ __forceinline__ float* chunk_slot(const m3_ssd_args& a, const Geo& g, int b, int h, int c) {
  return static_cast<float*>(a.chunk_states.data) + (((int64_t)b * a.heads + h) * g.nchunk + c) * g.P * g.N;
}

__device__ __forceinline__ float diag_at(const m3_ssd_args& a, int b, int t, int h) {
  return static_cast<const float*>(a.diag.data)[b * a.diag.stride[0] + (int64_t)t * a.diag.stride[1] +
                                                h * a.diag.stride[2]];
}

// delta_c = sum_j w_j x_j y_j^T over the chunk rows ([P][N]) into `out`, with x = v (w = T_s) for the
// forward or x = dy (w = e^{cum_t}) for the backward, y = k or q. Also writes e^{cum_last} to lam.
// Thread tile: 4 p x 8 n (two groups of four columns N / 2 apart).
__global__ void __launch_bounds__(kThreads) chunk_delta_kernel(const m3_ssd_args a, int bwd, float* out, float* lam) {
  extern __shared__ float smem[];
  const Geo g = geo(a);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t0 = c * g.tok_per, ntok = min(g.tok_per, g.L - t0), rows = ntok * g.R;
  float* X = smem;                    // [kRows][ldp]
  float* Y = X + kRows * ldp(g.P);    // [kRows][ldn]
  float* red = Y + kRows * ldn(g.N);  // [3][kRows]
  chunk_scalars(red, a.adt, b, h, t0, ntok);
  __syncthreads();
  load_rows(X, ldp(g.P), bwd ? a.dy : a.v, b, h, g.R, t0 * g.R, rows, g.P, red + (bwd ? kRows : 2 * kRows));
  load_rows(Y, ldn(g.N), bwd ? a.q : a.k, b, h, g.R, t0 * g.R, rows, g.N);
  __syncthreads();
  float* dst = out + (((int64_t)b * a.heads + h) * g.nchunk + c) * g.P * g.N;
  const int cn = g.N / 8;  // threads along n
  for (int tile = threadIdx.x; tile < (g.P / 4) * cn; tile += kThreads) {
    const int mb = (tile / cn) * 4, nb = (tile % cn) * 4, ns = 4 * cn;
    float acc[4][8];
    zero(acc);
    mm<4, 8, true, true>(acc, X, ldp(g.P), Y, ldn(g.N), kRows, mb, 0, nb, ns);
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int q = 0; q < 2; ++q)
        *reinterpret_cast<float4*>(dst + (mb + t) * g.N + nb + q * ns) =
            make_float4(acc[t][4 * q], acc[t][4 * q + 1], acc[t][4 * q + 2], acc[t][4 * q + 3]);
  }
  if (threadIdx.x == 0) lam[((int64_t)b * a.heads + h) * g.nchunk + c] = expf(red[ntok - 1]);
}

// Loads rows [row0, row0 + rows) of a [B, L, H, R, X] float tensor transposed into dst [X][ld]
// (dst[x * ld + i]); rows past `rows` are zero.
__device__ inline void load_rows_t(float* dst, int ld, const m3_tensor& t, int b, int h, int R, int row0, int rows,
                                   int X) {
  const float* base = static_cast<const float*>(t.data);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = warp; i < kRows; i += kThreads / 32) {
    if (4 * lane >= X) continue;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < rows) {
      const int row = row0 + i;
      v = *reinterpret_cast<const float4*>(base + row_off(t, b, row / R, h, row % R) + 4 * lane);
    }
    dst[(4 * lane) * ld + i] = v.x;
    dst[(4 * lane + 1) * ld + i] = v.y;
    dst[(4 * lane + 2) * ld + i] = v.z;
    dst[(4 * lane + 3) * ld + i] = v.w;
  }
}

// Forward carry, per (batch, head): slot c holds delta_c on entry and S_c on exit;
// S_{c+1} = lam_c S_c + delta_c; the last S is the final state. Thread: float4 groups
// e = 4 (tid + 256 q); the next chunk's deltas are loaded before the current chunk is stored.
constexpr int kMaxPer = kMaxN * kMaxP / (kThreads * 4);  // float4 groups per thread

__global__ void __launch_bounds__(kThreads) state_scan_kernel(const m3_ssd_args a, const float* lam) {
  const Geo g = geo(a);
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int PN = g.P * g.N;
  const float* lp = lam + ((int64_t)b * a.heads + h) * g.nchunk;
  float4 s[kMaxPer], d[kMaxPer];
#pragma unroll
  for (int q = 0; q < kMaxPer; ++q) {
    const int e = (tid + q * kThreads) * 4;
    s[q] = d[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < PN) {
      if (a.initial_state.data) {
        const int p = e / g.N, n = e % g.N;
        const m3_tensor& t = a.initial_state;
        const float* src = static_cast<const float*>(t.data) + b * t.stride[0] + h * t.stride[1] + p * t.stride[2];
        s[q] = make_float4(src[n * t.stride[3]], src[(n + 1) * t.stride[3]], src[(n + 2) * t.stride[3]],
                           src[(n + 3) * t.stride[3]]);
      }
      d[q] = *reinterpret_cast<const float4*>(chunk_slot(a, g, b, h, 0) + e);
    }
  }
  for (int c = 0; c < g.nchunk; ++c) {
    float4 nx[kMaxPer];
    float* slot = chunk_slot(a, g, b, h, c);
    const bool more = c + 1 < g.nchunk;
    const float* next = more ? chunk_slot(a, g, b, h, c + 1) : slot;
    const float l = lp[c];
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) {
      const int e = (tid + q * kThreads) * 4;
      nx[q] = (e < PN && more) ? *reinterpret_cast<const float4*>(next + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) {
      const int e = (tid + q * kThreads) * 4;
      if (e < PN) {
        *reinterpret_cast<float4*>(slot + e) = s[q];
        s[q] = make_float4(fmaf(l, s[q].x, d[q].x), fmaf(l, s[q].y, d[q].y), fmaf(l, s[q].z, d[q].z),
                           fmaf(l, s[q].w, d[q].w));
        d[q] = nx[q];
      }
    }
  }
  const m3_tensor& f = a.final_state;
#pragma unroll
  for (int q = 0; q < kMaxPer; ++q) {
    const int e = (tid + q * kThreads) * 4;
    if (e < PN) {
      const int p = e / g.N, n = e % g.N;
      float* dst = static_cast<float*>(f.data) + b * f.stride[0] + h * f.stride[1] + p * f.stride[2];
      dst[n * f.stride[3]] = s[q].x, dst[(n + 1) * f.stride[3]] = s[q].y;
      dst[(n + 2) * f.stride[3]] = s[q].z, dst[(n + 3) * f.stride[3]] = s[q].w;
    }
  }
}

// y_i = e^{cum_t} S_c q_i + sum_j Wt_ij v_j per chunk. Row tiles i = im + 16 t; columns p = in + (P/4) u.
__global__ void __launch_bounds__(kThreads) chunk_output_kernel(const m3_ssd_args a) {
  extern __shared__ float smem[];
  const Geo g = geo(a);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int t0 = c * g.tok_per, ntok = min(g.tok_per, g.L - t0), rows = ntok * g.R, R = g.R;
  const int LN = ldn(g.N);
  float* S = smem;                // [P][LN]
  float* Q = S + g.P * LN;        // [kRows][LN]
  float* K = Q + kRows * LN;      // [kRows][LN]
  float* Vt = K + kRows * LN;     // [P][kLdr]   v transposed
  float* W = Vt + g.P * kLdr;     // [kRows][kLdr]
  float* red = W + kRows * kLdr;  // [3][kRows]
  chunk_scalars(red, a.adt, b, h, t0, ntok);
  {
    const float* src = chunk_slot(a, g, b, h, c);
    for (int e = tid * 4; e < g.P * g.N; e += kThreads * 4)
      *reinterpret_cast<float4*>(S + (e / g.N) * LN + e % g.N) = *reinterpret_cast<const float4*>(src + e);
  }
  load_rows(Q, LN, a.q, b, h, R, t0 * R, rows, g.N);
  load_rows(K, LN, a.k, b, h, R, t0 * R, rows, g.N);
  load_rows_t(Vt, kLdr, a.v, b, h, R, t0 * R, rows, g.P);
  __syncthreads();
  // W = L o (Q K^T): 2 x 2 tiles, i = im + 16 t, j = in + 16 u
  {
    const int im = tid / 16, in = tid % 16;
    float acc[2][2];
    zero(acc);
    mm<2, 2, false, false>(acc, Q, LN, K, LN, g.N, im, 16, in, 16);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = im + 16 * t, j = in + 16 * u, ti = i / R, tj = j / R;
        float w = 0.0f;
        if (i < rows && j < rows && tj <= ti)
          w = (tj < ti ? expf(red[ti] - red[tj]) : diag_at(a, b, t0 + ti, h)) * acc[t][u];
        W[i * kLdr + j] = w;
      }
  }
  __syncthreads();
  // y = e^{cum} (Q S^T) + W V: 2 x 4 tiles over [kRows][P]
  const int cn = g.P / 4;
  for (int tile = tid; tile < 16 * cn; tile += kThreads) {
    const int im = tile / cn, in = tile % cn;
    float inter[2][4], intra[2][4];
    zero(inter);
    zero(intra);
    mm<2, 4, false, false>(inter, Q, LN, S, LN, g.N, im, 16, in, cn);
    mm<2, 4, false, false>(intra, W, kLdr, Vt, kLdr, kRows, im, 16, in, cn);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int i = im + 16 * t;
      if (i >= rows) continue;
      const int row = t0 * R + i;
      float* dst = static_cast<float*>(a.y.data) + row_off(a.y, b, row / R, h, row % R);
      const float e = red[kRows + i / R];
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[(in + cn * u) * a.y.stride[4]] = fmaf(e, inter[t][u], intra[t][u]);
    }
  }
}

// Backward carry, per (batch, head), chunks in reverse: slot c holds sum_i e^{cum_t} dy_i q_i^T on
// entry and G_c = dLoss/dS_{c+1} on exit; dS_c = lam_c G_c + delta_c. Also <G_c, S_c> per chunk
// (into gs) and the gradient of the initial state.
__global__ void __launch_bounds__(kThreads) grad_scan_kernel(const m3_ssd_args a, float* grads, const float* lam,
                                                             float* gs) {
  const Geo g = geo(a);
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int PN = g.P * g.N;
  const int64_t base = ((int64_t)b * a.heads + h) * g.nchunk;
  __shared__ float part[kThreads / 32];
  float4 d[kMaxPer], dl[kMaxPer], st4[kMaxPer];  // carry; this chunk's delta and S_c
#pragma unroll
  for (int q = 0; q < kMaxPer; ++q) {
    const int e = (tid + q * kThreads) * 4;
    d[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < PN && a.dfinal.data) {
      const int p = e / g.N, n = e % g.N;
      const m3_tensor& t = a.dfinal;
      const float* src = static_cast<const float*>(t.data) + b * t.stride[0] + h * t.stride[1] + p * t.stride[2];
      d[q] = make_float4(src[n * t.stride[3]], src[(n + 1) * t.stride[3]], src[(n + 2) * t.stride[3]],
                         src[(n + 3) * t.stride[3]]);
    }
  }
  auto fetch = [&](int c, float4* dlt, float4* stc) {
    const float* slot = grads + (base + c) * PN;
    const float* st = chunk_slot(a, g, b, h, c);
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) {
      const int e = (tid + q * kThreads) * 4;
      dlt[q] = stc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < PN) {
        dlt[q] = *reinterpret_cast<const float4*>(slot + e);
        stc[q] = *reinterpret_cast<const float4*>(st + e);
      }
    }
  };
  fetch(g.nchunk - 1, dl, st4);
  for (int c = g.nchunk - 1; c >= 0; --c) {
    float dot = 0.0f;
    const float l = lam[base + c];
    float* slot = grads + (base + c) * PN;
    float4 ndl[kMaxPer], nst[kMaxPer];
    if (c > 0) fetch(c - 1, ndl, nst);
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) {
      const int e = (tid + q * kThreads) * 4;
      if (e < PN) {
        *reinterpret_cast<float4*>(slot + e) = d[q];
        const float4 s = st4[q], delta = dl[q];
        dot += d[q].x * s.x + d[q].y * s.y + d[q].z * s.z + d[q].w * s.w;
        d[q] = make_float4(fmaf(l, d[q].x, delta.x), fmaf(l, d[q].y, delta.y), fmaf(l, d[q].z, delta.z),
                           fmaf(l, d[q].w, delta.w));
      }
      if (c > 0) dl[q] = ndl[q], st4[q] = nst[q];
    }
    dot = warp_sum(dot);
    if ((tid & 31) == 0) part[tid >> 5] = dot;
    __syncthreads();
    if (tid == 0) {
      float s = 0.0f;
      for (int w = 0; w < kThreads / 32; ++w) s += part[w];
      gs[base + c] = s;
    }
    __syncthreads();
  }
  if (a.dinitial.data) {
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) {
      const int e = (tid + q * kThreads) * 4;
      if (e < PN) {
        const int p = e / g.N, n = e % g.N;
        const m3_tensor& t = a.dinitial;
        float* dst = static_cast<float*>(t.data) + b * t.stride[0] + h * t.stride[1] + p * t.stride[2];
        dst[n * t.stride[3]] = d[q].x, dst[(n + 1) * t.stride[3]] = d[q].y;
        dst[(n + 2) * t.stride[3]] = d[q].z, dst[(n + 3) * t.stride[3]] = d[q].w;
      }
    }
  }
}

// Per-chunk gradients. Phase 1 (S_c in shared memory): scores, M, M^T, W^T, the pair terms of
// dcum / ddiag, dq and the inter term of dcum. Phase 2 (G_c replaces S_c): dk, dv and the state
// terms of dcum. Row tiles i (or j) = im + 16 t; columns n = 4 in + 64 (u / 4) + u % 4 (grouped) or
// p = in + (P/4) u (row-wise).
__global__ void __launch_bounds__(kThreads) chunk_grads_kernel(const m3_ssd_args a, const float* grads,
                                                               const float* gs) {
  extern __shared__ float smem[];
  const Geo g = geo(a);
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z, tid = threadIdx.x;
  const int t0 = c * g.tok_per, ntok = min(g.tok_per, g.L - t0), rows = ntok * g.R, R = g.R;
  const int LN = ldn(g.N), LP = ldp(g.P);
  float* S = smem;                 // [P][LN]: S_c, then G_c
  float* Q = S + g.P * LN;         // [kRows][LN]
  float* K = Q + kRows * LN;       // [kRows][LN]
  float* V = K + kRows * LN;       // [kRows][LP]
  float* dY = V + kRows * LP;      // [kRows][LP]
  float* dYt = dY + kRows * LP;    // [P][kLdr]
  float* M = dYt + g.P * kLdr;     // [kRows][kLdr]  L o (dY V^T)
  float* Mt = M + kRows * kLdr;    // [kRows][kLdr]  its transpose
  float* Wt = Mt + kRows * kLdr;   // [kRows][kLdr]  (L o (Q K^T))^T
  float* red = Wt + kRows * kLdr;  // cum, e^cum, T, dcum, ddiag  [5][kRows]
  float* dcum = red + 3 * kRows;
  float* ddg = red + 4 * kRows;
  const int64_t bh = (int64_t)b * a.heads + h;
  chunk_scalars(red, a.adt, b, h, t0, ntok);
  if (tid < kRows) dcum[tid] = ddg[tid] = 0.0f;
  {
    const float* src = chunk_slot(a, g, b, h, c);
    for (int e = tid * 4; e < g.P * g.N; e += kThreads * 4)
      *reinterpret_cast<float4*>(S + (e / g.N) * LN + e % g.N) = *reinterpret_cast<const float4*>(src + e);
  }
  load_rows(Q, LN, a.q, b, h, R, t0 * R, rows, g.N);
  load_rows(K, LN, a.k, b, h, R, t0 * R, rows, g.N);
  load_rows(V, LP, a.v, b, h, R, t0 * R, rows, g.P);
  load_rows(dY, LP, a.dy, b, h, R, t0 * R, rows, g.P);
  load_rows_t(dYt, kLdr, a.dy, b, h, R, t0 * R, rows, g.P);
  __syncthreads();
  // scores A = Q K^T and B = dY V^T (2 x 2 tiles): Wt, M, Mt, pair terms of dcum / ddiag
  {
    const int im = tid / 16, in = tid % 16;
    float qa[2][2], bb[2][2];
    zero(qa);
    zero(bb);
    mm<2, 2, false, false>(qa, Q, LN, K, LN, g.N, im, 16, in, 16);
    mm<2, 2, false, false>(bb, dY, LP, V, LP, g.P, im, 16, in, 16);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = im + 16 * t, j = in + 16 * u, ti = i / R, tj = j / R;
        float w = 0.0f, m = 0.0f;
        if (i < rows && j < rows && tj <= ti) {
          if (tj == ti) {
            const float dg = diag_at(a, b, t0 + ti, h);
            w = dg * qa[t][u];
            m = dg * bb[t][u];
            atomicAdd(&ddg[ti], qa[t][u] * bb[t][u]);
          } else {
            const float lw = expf(red[ti] - red[tj]);
            w = lw * qa[t][u];
            m = lw * bb[t][u];
            const float gp = w * bb[t][u];
            atomicAdd(&dcum[ti], gp);
            atomicAdd(&dcum[tj], -gp);
          }
        }
        Wt[j * kLdr + i] = w;
        M[i * kLdr + j] = m;
        Mt[j * kLdr + i] = m;
      }
  }
  __syncthreads();
  const int cn8 = g.N / 8, cn4 = g.P / 4;
  // dq = e^{cum} (dY S) + M K: 2 x 8 tiles over [kRows][N]
  for (int tile = tid; tile < 16 * cn8; tile += kThreads) {
    const int im = tile / cn8, nb = (tile % cn8) * 4, ns = 4 * cn8;
    float inter[2][8], intra[2][8];
    zero(inter);
    zero(intra);
    mm<2, 8, false, true>(inter, dY, LP, S, LN, g.P, im, 16, nb, ns);
    mm<2, 8, false, true>(intra, M, kLdr, K, LN, kRows, im, 16, nb, ns);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int i = im + 16 * t;
      if (i >= rows) continue;
      const int row = t0 * R + i;
      float* dst = static_cast<float*>(a.dq.data) + row_off(a.dq, b, row / R, h, row % R);
      const float e = red[kRows + i / R];
#pragma unroll
      for (int u = 0; u < 8; ++u) dst[gidx(nb, ns, u) * a.dq.stride[4]] = fmaf(e, inter[t][u], intra[t][u]);
    }
  }
  // inter term of dcum: e^{cum_t} dy_i . (S q_i): (Q S^T) in 2 x 4 tiles over [kRows][P]
  for (int tile = tid; tile < 16 * cn4; tile += kThreads) {
    const int im = tile / cn4, in = tile % cn4;
    float sq[2][4];
    zero(sq);
    mm<2, 4, false, false>(sq, Q, LN, S, LN, g.N, im, 16, in, cn4);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int i = im + 16 * t;
      float d = 0.0f;
#pragma unroll
      for (int u = 0; u < 4; ++u) d = fmaf(dY[i * LP + in + cn4 * u], sq[t][u], d);
      if (i < rows) atomicAdd(&dcum[i / R], red[kRows + i / R] * d);
    }
  }
  __syncthreads();
  // Phase 2: G_c = dLoss/dS_{c+1} replaces S_c
  {
    const float* src = grads + (bh * g.nchunk + c) * g.P * g.N;
    for (int e = tid * 4; e < g.P * g.N; e += kThreads * 4)
      *reinterpret_cast<float4*>(S + (e / g.N) * LN + e % g.N) = *reinterpret_cast<const float4*>(src + e);
  }
  __syncthreads();
  // dk = T (V G) + M^T Q: 2 x 8 tiles over [kRows][N]
  for (int tile = tid; tile < 16 * cn8; tile += kThreads) {
    const int im = tile / cn8, nb = (tile % cn8) * 4, ns = 4 * cn8;
    float st[2][8], pr[2][8];
    zero(st);
    zero(pr);
    mm<2, 8, false, true>(st, V, LP, S, LN, g.P, im, 16, nb, ns);
    mm<2, 8, false, true>(pr, Mt, kLdr, Q, LN, kRows, im, 16, nb, ns);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int j = im + 16 * t;
      if (j >= rows) continue;
      const int row = t0 * R + j;
      float* dst = static_cast<float*>(a.dk.data) + row_off(a.dk, b, row / R, h, row % R);
      const float T = red[2 * kRows + j / R];
#pragma unroll
      for (int u = 0; u < 8; ++u) dst[gidx(nb, ns, u) * a.dk.stride[4]] = fmaf(T, st[t][u], pr[t][u]);
    }
  }
  // dv = T (K G^T) + Wt dY^T... per element: T (G k_j)[p] + sum_i Wt_ji dy_i[p]; 2 x 4 tiles over
  // [kRows][P]; state terms of dcum from v_j . (G k_j)
  for (int tile = tid; tile < 16 * cn4; tile += kThreads) {
    const int im = tile / cn4, in = tile % cn4;
    float gk[2][4], pr[2][4];
    zero(gk);
    zero(pr);
    mm<2, 4, false, false>(gk, K, LN, S, LN, g.N, im, 16, in, cn4);
    mm<2, 4, false, false>(pr, Wt, kLdr, dYt, kLdr, kRows, im, 16, in, cn4);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int j = im + 16 * t;
      if (j >= rows) continue;
      const int row = t0 * R + j;
      float* dst = static_cast<float*>(a.dv.data) + row_off(a.dv, b, row / R, h, row % R);
      const float T = red[2 * kRows + j / R];
      float sd = 0.0f;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int pp = in + cn4 * u;
        dst[pp * a.dv.stride[4]] = fmaf(T, gk[t][u], pr[t][u]);
        sd = fmaf(V[j * LP + pp], gk[t][u], sd);
      }
      sd *= T;
      atomicAdd(&dcum[j / R], -sd);
      atomicAdd(&dcum[ntok - 1], sd);
    }
  }
  __syncthreads();
  // dadt = reverse cumsum of dcum (plus e^{cum_last} <G_c, S_c> on the last token); ddiag
  if (tid < 32) {
    const int lane = tid;
    const float lam = expf(red[ntok - 1]);
    float v = lane < ntok ? dcum[lane] + (lane == ntok - 1 ? lam * gs[bh * g.nchunk + c] : 0.0f) : 0.0f;
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

inline size_t delta_smem(int N, int P) { return (size_t)(kRows * ldp(P) + kRows * ldn(N) + 3 * kRows) * 4; }
inline size_t output_smem(int N, int P) {
  return (size_t)(P * ldn(N) + 2 * kRows * ldn(N) + P * kLdr + kRows * kLdr + 3 * kRows) * 4;
}
inline size_t grads_smem(int N, int P) {
  return (size_t)(P * ldn(N) + 2 * kRows * ldn(N) + 2 * kRows * ldp(P) + P * kLdr + 3 * kRows * kLdr + 5 * kRows) *
         4;
}

}  // namespace ssdt

int report_error(int code, const char* msg);

static int ssd_check(const m3_ssd_args* args, bool bwd) {
  if (args == nullptr) return report_error(M3_ERR_ARGUMENT, "null argument struct");
  const m3_ssd_args& a = *args;
  if (a.batch <= 0 || a.length <= 0 || a.heads <= 0)
    return report_error(M3_ERR_SHAPE, "batch, length and heads must be positive");
  if (a.rank != 1 && a.rank != 2 && a.rank != 4 && a.rank != 8)
    return report_error(M3_ERR_SHAPE, "rank must be 1, 2, 4 or 8");
  if (a.d_state <= 0 || a.d_state > ssdt::kMaxN || a.head_dim <= 0 || a.head_dim > ssdt::kMaxP ||
      a.d_state % 8 != 0 || a.head_dim % 8 != 0)
    return report_error(M3_ERR_SHAPE, "training kernels serve d_state <= 128 and head_dim <= 64, multiples of 8");
  const m3_tensor* need[] = {&a.q, &a.k, &a.v, &a.adt, &a.diag, &a.chunk_states};
  for (const m3_tensor* t : need)
    if (t->data == nullptr || t->dtype != M3_F32)
      return report_error(M3_ERR_ARGUMENT, "q, k, v, adt, diag and chunk_states must be float32 tensors");
  if ((reinterpret_cast<uintptr_t>(a.chunk_states.data) & 15u) != 0)
    return report_error(M3_ERR_LAYOUT, "chunk_states must be 16-byte aligned and contiguous");
  // row tensors: contiguous rows starting on 16-byte boundaries (16-byte loads)
  const m3_tensor* row_tensors[] = {&a.q, &a.k, &a.v, &a.dy};
  for (const m3_tensor* t : row_tensors) {
    if (t->data == nullptr) continue;
    if (t->stride[4] != 1 || (reinterpret_cast<uintptr_t>(t->data) & 15u) != 0 || t->stride[0] % 4 != 0 ||
        t->stride[1] % 4 != 0 || t->stride[2] % 4 != 0 || t->stride[3] % 4 != 0)
      return report_error(M3_ERR_LAYOUT, "q, k, v and dy need contiguous rows on 16-byte boundaries");
  }
  if (a.initial_state.data && a.initial_state.dtype != M3_F32)
    return report_error(M3_ERR_ARGUMENT, "initial_state must be float32");
  if (!bwd) {
    if (!a.y.data || !a.final_state.data || a.y.dtype != M3_F32 || a.final_state.dtype != M3_F32)
      return report_error(M3_ERR_ARGUMENT, "y and final_state must be float32 outputs");
  } else {
    const m3_tensor* outs[] = {&a.dy, &a.dq, &a.dk, &a.dv, &a.dadt, &a.ddiag};
    for (const m3_tensor* t : outs)
      if (t->data == nullptr || t->dtype != M3_F32)
        return report_error(M3_ERR_ARGUMENT, "dy, dq, dk, dv, dadt and ddiag must be float32 tensors");
    if ((a.dfinal.data && a.dfinal.dtype != M3_F32) || (a.dinitial.data && a.dinitial.dtype != M3_F32))
      return report_error(M3_ERR_ARGUMENT, "dfinal and dinitial must be float32");
  }
  if (a.workspace.data == nullptr || a.workspace.dtype != M3_F32 ||
      (reinterpret_cast<uintptr_t>(a.workspace.data) & 15u) != 0)
    return report_error(M3_ERR_ARGUMENT, "a 16-byte aligned float32 workspace of m3_ssd_workspace_bytes() is required");
  return M3_OK;
}

static int64_t ssd_nchunk(const m3_ssd_args& a) {
  const int tok_per = ssdt::kRows / a.rank;
  return (a.length + tok_per - 1) / tok_per;
}

// Scratch floats of a call: per-chunk e^{cum_last} and <G_c, S_c>, then (backward) the gradient slots.
static int64_t ssd_scratch_floats(const m3_ssd_args& a, bool bwd) {
  const int64_t slots = (int64_t)a.batch * a.heads * ssd_nchunk(a);
  const int64_t small = (2 * slots + 3) / 4 * 4;
  return small + (bwd ? slots * a.head_dim * a.d_state : 0);
}

template <typename K> static cudaError_t set_smem(K kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

static int ssd_launch(const m3_ssd_args* args, void* stream_, bool bwd) {
  const int rc = ssd_check(args, bwd);
  if (rc != M3_OK) return rc;
  const m3_ssd_args& a = *args;
  if (a.device >= 0 && cudaSetDevice(a.device) != cudaSuccess)
    return report_error(M3_ERR_CUDA, "cannot select the device");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int N = a.d_state, P = a.head_dim;
  const int64_t nchunk = ssd_nchunk(a);
  const int64_t slots = (int64_t)a.batch * a.heads * nchunk;
  float* ws = static_cast<float*>(a.workspace.data);
  float* lam = ws;
  float* gs = ws + slots;
  float* grads = ws + (2 * slots + 3) / 4 * 4;
  const dim3 chunk_grid((unsigned)nchunk, a.heads, a.batch), bh_grid(a.heads, a.batch);
  cudaError_t e = set_smem(ssdt::chunk_delta_kernel, ssdt::delta_smem(N, P));
  if (!bwd) {
    if (e == cudaSuccess) e = set_smem(ssdt::chunk_output_kernel, ssdt::output_smem(N, P));
    if (e == cudaSuccess) {
      ssdt::chunk_delta_kernel<<<chunk_grid, ssdt::kThreads, ssdt::delta_smem(N, P), stream>>>(
          a, 0, static_cast<float*>(a.chunk_states.data), lam);
      ssdt::state_scan_kernel<<<bh_grid, ssdt::kThreads, 0, stream>>>(a, lam);
      ssdt::chunk_output_kernel<<<chunk_grid, ssdt::kThreads, ssdt::output_smem(N, P), stream>>>(a);
      e = cudaGetLastError();
    }
  } else {
    if (e == cudaSuccess) e = set_smem(ssdt::chunk_grads_kernel, ssdt::grads_smem(N, P));
    if (e == cudaSuccess) {
      ssdt::chunk_delta_kernel<<<chunk_grid, ssdt::kThreads, ssdt::delta_smem(N, P), stream>>>(a, 1, grads, lam);
      ssdt::grad_scan_kernel<<<bh_grid, ssdt::kThreads, 0, stream>>>(a, grads, lam, gs);
      ssdt::chunk_grads_kernel<<<chunk_grid, ssdt::kThreads, ssdt::grads_smem(N, P), stream>>>(a, grads, gs);
      e = cudaGetLastError();
    }
  }
  if (e != cudaSuccess)
    return report_error(M3_ERR_CUDA, (std::string("training kernel launch failed: ") + cudaGetErrorString(e)).c_str());
  return M3_OK;
}

}  // namespace m3

extern "C" {

int m3_ssd_chunk_rows(void) { return m3::ssdt::kRows; }

int64_t m3_ssd_workspace_bytes(const m3_ssd_args* args, int backward) {
  if (args == nullptr) return -m3::report_error(M3_ERR_ARGUMENT, "null argument struct");
  if (args->batch <= 0 || args->length <= 0 || args->heads <= 0 || args->rank <= 0)
    return -m3::report_error(M3_ERR_SHAPE, "batch, length, heads and rank must be positive");
  return m3::ssd_scratch_floats(*args, backward != 0) * (int64_t)sizeof(float);
}

int m3_ssd_train_fwd(const m3_ssd_args* args, void* stream) { return m3::ssd_launch(args, stream, false); }

int m3_ssd_train_bwd(const m3_ssd_args* args, void* stream) { return m3::ssd_launch(args, stream, true); }

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Training prelude: group expansion, bias, rotation and trapezoid scale of q / k
// (mamba3/ops.py:35-84 rotate_qk, ops.py:665-676 / 719-745 bias and k * scale), fused into one
// pass that writes the float32 core operands, and its backward. One warp per (batch, token, head);
// lane l owns columns n = 4 l .. 4 l + 3 of every rank's row: a SISO rotation pair (2m, 2m + 1) is
// lane-local, a MIMO pair (m, 2S + m) sits in lanes l and l + S / 2 (one shuffle).
// The activation-dtype rounding of every step follows the reference's tensor ops.
// ---------------------------------------------------------------------------------------------
namespace m3 {
namespace ssdt {

template <typename T> struct PreludeLane {
  const m3_prelude_args& a;
  int b, t, h, g, lane, n0, S;
  bool active, mimo;
  __device__ PreludeLane(const m3_prelude_args& a_, int b_, int t_, int h_, int lane_)
      : a(a_), b(b_), t(t_), h(h_), lane(lane_) {
    g = h / (a.heads / a.groups);
    n0 = 4 * lane;
    active = n0 < a.d_state;
    S = a.phase.data ? a.num_angles : 0;
    mimo = a.mimo_rotation != 0;
  }
  // lane holding the rotation partner of this lane's columns (MIMO), else this lane
  __device__ int partner() const {
    if (!mimo || S == 0) return lane;
    if (n0 < S) return lane + S / 2;  // columns n + 2S, same slot
    if (n0 >= 2 * S && n0 < 3 * S) return lane - S / 2;
    return lane;
  }
  // angle index of slot j (or -1: not rotated); first: this element is the pair's first member
  __device__ int angle(int j, bool& first) const {
    const int n = n0 + j;
    first = true;
    if (S == 0) return -1;
    if (!mimo) {
      first = (n & 1) == 0;
      return (n >> 1) < S ? (n >> 1) : -1;
    }
    if (n < S) return n;
    if (n >= 2 * S && n < 3 * S) {
      first = false;
      return n - 2 * S;
    }
    return -1;
  }
  __device__ float phase_at(int m) const {
    const m3_tensor& p = a.phase;
    return static_cast<const float*>(p.data)[b * p.stride[0] + (int64_t)t * p.stride[1] + h * p.stride[2] +
                                             m * p.stride[3]];
  }
  // biased, unrotated q (which = 0) or k (1) of rank r, rounded to T
  __device__ void biased(int which, int r, float (&x)[4]) const {
    const m3_tensor& src = which ? a.k : a.q;
    const m3_tensor& bias = which ? a.k_bias : a.q_bias;
    const int64_t base = b * src.stride[0] + (int64_t)t * src.stride[1] + g * src.stride[2] + r * src.stride[3];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[j] = 0.0f;
      if (active) {
        x[j] = ld_t(src, base + (n0 + j) * src.stride[4]);
        if (bias.data)
          x[j] = rnd<T>(x[j] + rnd<T>(ld_t(bias, h * bias.stride[0] + r * bias.stride[1] + (n0 + j) * bias.stride[2])));
      }
    }
  }
};

template <typename T>
__global__ void __launch_bounds__(128) prelude_fwd_kernel(const m3_prelude_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.batch * a.length * a.heads) return;
  const int h = (int)(wid % a.heads), t = (int)((wid / a.heads) % a.length), b = (int)(wid / ((int64_t)a.heads * a.length));
  PreludeLane<T> pl(a, b, t, h, lane);
  const int src = pl.partner();
  float cs[4], sn[4];
  int ang[4];
  bool first[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ang[j] = pl.active ? pl.angle(j, first[j]) : -1;
    cs[j] = 1.0f, sn[j] = 0.0f;
    if (ang[j] >= 0) {
      float s_, c_;
      sincosf(pl.phase_at(ang[j]), &s_, &c_);
      cs[j] = rnd<T>(c_), sn[j] = rnd<T>(s_);
    }
  }
  const float sc = rnd<T>(static_cast<const float*>(a.scale.data)[b * a.scale.stride[0] + (int64_t)t * a.scale.stride[1] +
                                                                   h * a.scale.stride[2]]);
  for (int which = 0; which < 2; ++which) {
    for (int r = 0; r < a.rank; ++r) {
      float x[4], o[4];
      pl.biased(which, r, x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // partner element: same lane (SISO, slot j ^ 1) or the partner lane, slot j (MIMO)
        const float other = pl.mimo ? __shfl_sync(0xffffffffu, x[j], src) : x[j ^ 1];
        o[j] = x[j];
        if (ang[j] >= 0) {
          const float av = first[j] ? x[j] : other, bv = first[j] ? other : x[j];
          o[j] = first[j] ? rnd<T>(rnd<T>(av * cs[j]) - rnd<T>(bv * sn[j]))
                          : rnd<T>(rnd<T>(av * sn[j]) + rnd<T>(bv * cs[j]));
        }
        if (which) o[j] = rnd<T>(o[j] * sc);
      }
      if (pl.active) {
        const m3_tensor& dst = which ? a.kc : a.qf;
        *reinterpret_cast<float4*>(static_cast<float*>(dst.data) + b * dst.stride[0] + (int64_t)t * dst.stride[1] +
                                   h * dst.stride[2] + r * dst.stride[3] + pl.n0) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) prelude_bwd_kernel(const m3_prelude_args a) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.batch * a.length * a.heads) return;
  const int h = (int)(wid % a.heads), t = (int)((wid / a.heads) % a.length), b = (int)(wid / ((int64_t)a.heads * a.length));
  PreludeLane<T> pl(a, b, t, h, lane);
  const int src = pl.partner();
  float cs[4], sn[4], ce[4], se[4], dph[4];
  int ang[4];
  bool first[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    ang[j] = pl.active ? pl.angle(j, first[j]) : -1;
    cs[j] = ce[j] = 1.0f, sn[j] = se[j] = 0.0f, dph[j] = 0.0f;
    if (ang[j] >= 0) {
      sincosf(pl.phase_at(ang[j]), &se[j], &ce[j]);
      cs[j] = rnd<T>(ce[j]), sn[j] = rnd<T>(se[j]);
    }
  }
  const float sc = rnd<T>(static_cast<const float*>(a.scale.data)[b * a.scale.stride[0] + (int64_t)t * a.scale.stride[1] +
                                                                   h * a.scale.stride[2]]);
  float dsc = 0.0f;
  for (int which = 0; which < 2; ++which) {
    const m3_tensor& din = which ? a.dkc : a.dqf;
    const m3_tensor& dout = which ? a.dkb : a.dqb;
    for (int r = 0; r < a.rank; ++r) {
      float x[4], d[4] = {0.f, 0.f, 0.f, 0.f};
      pl.biased(which, r, x);
      if (pl.active) {
        const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(din.data) + b * din.stride[0] +
                                                          (int64_t)t * din.stride[1] + h * din.stride[2] +
                                                          r * din.stride[3] + pl.n0);
        d[0] = v.x, d[1] = v.y, d[2] = v.z, d[3] = v.w;
      }
      float rot[4];
      // forward rotated values (for the scale gradient) and the gradient before the scale
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float other = pl.mimo ? __shfl_sync(0xffffffffu, x[j], src) : x[j ^ 1];
        rot[j] = x[j];
        if (ang[j] >= 0) {
          const float av = first[j] ? x[j] : other, bv = first[j] ? other : x[j];
          rot[j] = first[j] ? rnd<T>(rnd<T>(av * cs[j]) - rnd<T>(bv * sn[j]))
                            : rnd<T>(rnd<T>(av * sn[j]) + rnd<T>(bv * cs[j]));
        }
      }
      if (which) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          dsc = fmaf(d[j], rot[j], dsc);
          d[j] *= sc;
        }
      }
      // rotation backward: out1 = a c - b s, out2 = a s + b c
      float g[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float xo = pl.mimo ? __shfl_sync(0xffffffffu, x[j], src) : x[j ^ 1];
        const float dother = pl.mimo ? __shfl_sync(0xffffffffu, d[j], src) : d[j ^ 1];
        g[j] = d[j];
        if (ang[j] >= 0) {
          const float av = first[j] ? x[j] : xo, bv = first[j] ? xo : x[j];
          const float d1 = first[j] ? d[j] : dother, d2 = first[j] ? dother : d[j];
          g[j] = first[j] ? d1 * cs[j] + d2 * sn[j] : -d1 * sn[j] + d2 * cs[j];
          if (first[j]) dph[j] += (d1 * av + d2 * bv) * (-se[j]) + (d2 * av - d1 * bv) * ce[j];
        }
      }
      if (pl.active) {
        *reinterpret_cast<float4*>(static_cast<float*>(dout.data) + b * dout.stride[0] + (int64_t)t * dout.stride[1] +
                                   h * dout.stride[2] + r * dout.stride[3] + pl.n0) = make_float4(g[0], g[1], g[2], g[3]);
      }
    }
  }
  if (a.dphase.data) {
    const m3_tensor& p = a.dphase;
    float* dp = static_cast<float*>(p.data) + b * p.stride[0] + (int64_t)t * p.stride[1] + h * p.stride[2];
    // every angle m < S has exactly one first member (column 2m SISO, m MIMO): its lane writes it
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (ang[j] >= 0 && first[j]) dp[ang[j] * p.stride[3]] = dph[j];
  }
  dsc = warp_sum(dsc);
  if (lane == 0) {
    const m3_tensor& s = a.dscale;
    static_cast<float*>(s.data)[b * s.stride[0] + (int64_t)t * s.stride[1] + h * s.stride[2]] = dsc;
  }
}

}  // namespace ssdt

static int prelude_launch(const m3_prelude_args* args, void* stream, bool bwd) {
  if (args == nullptr) return report_error(M3_ERR_ARGUMENT, "null argument struct");
  const m3_prelude_args& a = *args;
  if (a.batch <= 0 || a.length <= 0 || a.heads <= 0 || a.groups <= 0 || a.heads % a.groups != 0 || a.rank <= 0)
    return report_error(M3_ERR_SHAPE, "batch, length, heads, groups and rank must be positive (heads divisible by groups)");
  if (a.d_state <= 0 || a.d_state > 128 || a.d_state % 4 != 0)
    return report_error(M3_ERR_SHAPE, "the prelude kernels serve d_state <= 128, a multiple of 4");
  if (a.phase.data && (a.num_angles <= 0 || (a.mimo_rotation ? (a.num_angles % 4 != 0 || 4 * a.num_angles > a.d_state)
                                                             : 2 * a.num_angles > a.d_state)))
    return report_error(M3_ERR_SHAPE, "angle count does not fit the state width (MIMO: a multiple of 4)");
  if (!a.q.data || !a.k.data || !a.scale.data || a.scale.dtype != M3_F32 || a.q.dtype != a.k.dtype)
    return report_error(M3_ERR_ARGUMENT, "q, k (same dtype) and a float32 scale are required");
  if ((a.q_bias.data == nullptr) != (a.k_bias.data == nullptr))
    return report_error(M3_ERR_ARGUMENT, "q_bias and k_bias must be given together");
  if (a.phase.data && a.phase.dtype != M3_F32) return report_error(M3_ERR_ARGUMENT, "phase must be float32");
  const m3_tensor* rows[] = {bwd ? &a.dqf : &a.qf, bwd ? &a.dkc : &a.kc, bwd ? &a.dqb : &a.qf, bwd ? &a.dkb : &a.kc};
  for (const m3_tensor* r : rows)
    if (!r->data || r->dtype != M3_F32 || r->stride[4] != 1 || (reinterpret_cast<uintptr_t>(r->data) & 15u) ||
        r->stride[0] % 4 || r->stride[1] % 4 || r->stride[2] % 4 || r->stride[3] % 4)
      return report_error(M3_ERR_LAYOUT, "float32 [B,L,H,R,N] rows must be contiguous and 16-byte aligned");
  if (bwd && (!a.dscale.data || a.dscale.dtype != M3_F32)) return report_error(M3_ERR_ARGUMENT, "dscale (float32) is required");
  if (a.device >= 0 && cudaSetDevice(a.device) != cudaSuccess) return report_error(M3_ERR_CUDA, "cannot select the device");
  const int64_t warps = (int64_t)a.batch * a.length * a.heads;
  const unsigned grid = (unsigned)((warps + 3) / 4);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a.q.dtype) {
    case M3_BF16:
      bwd ? ssdt::prelude_bwd_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a)
          : ssdt::prelude_fwd_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a);
      break;
    case M3_F16:
      bwd ? ssdt::prelude_bwd_kernel<__half><<<grid, 128, 0, st>>>(a) : ssdt::prelude_fwd_kernel<__half><<<grid, 128, 0, st>>>(a);
      break;
    default:
      bwd ? ssdt::prelude_bwd_kernel<float><<<grid, 128, 0, st>>>(a) : ssdt::prelude_fwd_kernel<float><<<grid, 128, 0, st>>>(a);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(M3_ERR_CUDA, (std::string("prelude launch failed: ") + cudaGetErrorString(e)).c_str());
  return M3_OK;
}

}  // namespace m3

extern "C" {
int m3_ssd_prelude_fwd(const m3_prelude_args* args, void* stream) { return m3::prelude_launch(args, stream, false); }
int m3_ssd_prelude_bwd(const m3_prelude_args* args, void* stream) { return m3::prelude_launch(args, stream, true); }
}
