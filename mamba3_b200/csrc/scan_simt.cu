// Chunked Mamba-3 SSD forward on CUDA cores (FP32 arithmetic).
//
// This kernel serves every shape and dtype (it is the FP32 path, and the path for state widths
// and head dims the tensor-core kernel is not built for). One CTA owns one (batch, head) pair and
// walks the sequence one tile of ROWS flattened (token, rank) rows at a time, carrying the FP32
// state [P, N] in shared memory:
//   y_i   = e^{cum_i} (q_i . S^T) + sum_{j <= i} (q_i . k_j scale_j) L_ij v_j + D v_i,
//   y     = sum_r mo_r silu(z mz_r) y_(t,r)
//   S'    = e^{cum_last} S + sum_j v_j e^{cum_last - cum_j} (k_j scale_j)^T
// with L_ij = e^{cum_i - cum_j} below the diagonal and gamma/scale on same-token pairs
// (mamba3/ops.py:716-816; the fused reference kernels are mamba3/_triton.py:74-413).
// In bf16/fp16 mode the activation-dtype roundings of the reference are reproduced with rnd<T>.
#include "scan_common.cuh"

namespace m3 {

struct SimtLayout {
  int NP, PP, WP;
  size_t q, k, v, v2, y, w, st, ph, scal, seg, carry, total;
};

__host__ __device__ inline SimtLayout simt_layout(int rows, int tok, int N, int P, int S) {
  SimtLayout L;
  L.NP = N + 1;
  L.PP = P + 1;
  L.WP = rows + 1;
  size_t o = 0;
  L.q = o; o += (size_t)rows * L.NP;
  L.k = o; o += (size_t)rows * L.NP;
  L.v = o; o += (size_t)rows * L.PP;
  L.v2 = o; o += (size_t)rows * L.PP;
  L.y = o; o += (size_t)rows * L.PP;
  L.w = o; o += (size_t)rows * L.WP;
  L.st = o; o += (size_t)P * L.NP;
  L.ph = o; o += (size_t)tok * (S + 1);
  L.scal = o; o += 7 * 128 + 8;
  L.seg = o; o += 768;
  L.carry = o; o += 2 * 128;
  L.total = o * sizeof(float);
  return L;
}

template <typename T, int R, int ROWS>
__global__ void __launch_bounds__(256) scan_simt_kernel(const m3_scan_args a) {
  constexpr int TOK = ROWS / R;
  const int h = blockIdx.x, b = blockIdx.y;
  const int N = a.d_state, P = a.head_dim, S = a.num_angles, L = a.length;
  const int g = h / (a.heads / a.groups);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const SimtLayout lay = simt_layout(ROWS, TOK, N, P, S);
  const int NP = lay.NP, PP = lay.PP, WP = lay.WP;
  extern __shared__ float smem[];
  float* sQ = smem + lay.q;
  float* sK = smem + lay.k;
  float* sV = smem + lay.v;
  float* sV2 = smem + lay.v2;
  float* sY = smem + lay.y;
  float* sW = smem + lay.w;
  float* sS = smem + lay.st;
  float* sPh = smem + lay.ph;
  float* scal = smem + lay.scal;
  TileScalars ts{scal, scal + 128, scal + 256, scal + 384, scal + 512, scal + 640, scal + 7 * 128};
  float* seg = smem + lay.seg;
  float* carry_off = smem + lay.carry;
  float* carry_loc = carry_off + 128;
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;

  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const T* vp = static_cast<const T*>(a.value.data);
  const T* zp = static_cast<const T*>(a.gate.data);
  T* yp = static_cast<T*>(a.y.data);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);

  // ---- initial state (+ endpoint-cache contribution, mamba3/ops.py:679-686) ----
  float c0 = 0.0f;
  if (a.initial_k.data) {
    float dt0, adt0;
    const int t_first = scan_token(a, 0);
    load_dt_adt(a, b, t_first, h, dt0, adt0);
    c0 = dt0 * (1.0f - sigmoidf_(load_trap(a, b, t_first, h)));
  }
  for (int i = tid; i < P * N; i += blockDim.x) {
    const int p = i / N, n = i % N;
    float s = 0.0f;
    if (a.initial_state.data) {
      const m3_tensor& t = a.initial_state;
      s = ld_t(t, b * t.stride[0] + h * t.stride[1] + p * t.stride[2] + n * t.stride[3]);
    }
    if (a.initial_k.data) {
      const m3_tensor& ik = a.initial_k;
      const m3_tensor& iv = a.initial_value;
      const float v = ld_t(iv, b * iv.stride[0] + h * iv.stride[1] + p * iv.stride[2]);
      float acc = 0.0f;
      for (int r = 0; r < R; ++r) {
        float vr = v;
        if (R > 1) vr = rnd<T>(v * rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] +
                                                       p * a.mimo_x.stride[2])));
        acc += vr * ld_t(ik, b * ik.stride[0] + h * ik.stride[1] + r * ik.stride[2] + n * ik.stride[3]);
      }
      s += c0 * acc;
    }
    sS[p * NP + n] = s;
  }
  if (tid < S) {
    float off = 0.0f;
    if (a.initial_phase.data) {
      const m3_tensor& t = a.initial_phase;
      off = ld_t(t, b * t.stride[0] + h * t.stride[1] + tid * t.stride[2]);
    }
    carry_off[tid] = off;
    carry_loc[tid] = 0.0f;
  }
  __syncthreads();

  for (int t0 = 0; t0 < L; t0 += TOK) {
    const int nt = min(TOK, L - t0);
    float last_decay;
    tile_scalars(a, b, h, t0, nt, TOK, ts, last_decay);
    if (has_phase) tile_phase(a, b, h, t0, nt, TOK, ts.dt, sPh, S + 1, carry_off, carry_loc, seg);

    // ---- stage q, k (norm, bias, rotation, scale) and v rows ----
    for (int row = warp; row < ROWS; row += 8) {
      const int j = row / R, r = row % R;
      float* qrow = sQ + row * NP;
      float* krow = sK + row * NP;
      if (j >= nt) {
        for (int n = lane; n < N; n += 32) { qrow[n] = 0.0f; krow[n] = 0.0f; }
        for (int p = lane; p < P; p += 32) { sV[row * PP + p] = 0.0f; sV2[row * PP + p] = 0.0f; }
        continue;
      }
      const int t = scan_token(a, t0 + j);
      const int64_t qb = b * a.q.stride[0] + (int64_t)t * a.q.stride[1] + g * a.q.stride[2] + r * a.q.stride[3];
      const int64_t kb = b * a.k.stride[0] + (int64_t)t * a.k.stride[1] + g * a.k.stride[2] + r * a.k.stride[3];
      float sq = 0.0f, sk = 0.0f;
      for (int n = lane; n < N; n += 32) {
        const float x = to_f(qp[qb + n * a.q.stride[4]]);
        const float y = to_f(kp[kb + n * a.k.stride[4]]);
        qrow[n] = x;
        krow[n] = y;
        sq += x * x;
        sk += y * y;
      }
      float rq = 1.0f, rk = 1.0f;
      if (a.q_norm_w.data) {
        rq = rsqrtf(warp_sum(sq) / N + a.norm_eps);
        rk = rsqrtf(warp_sum(sk) / N + a.norm_eps);
      }
      for (int n = lane; n < N; n += 32) {
        float x = qrow[n], y = krow[n];
        if (a.q_norm_w.data) {
          x = rnd<T>(x * rq * rnd<T>(ld_t(a.q_norm_w, n * a.q_norm_w.stride[0])));
          y = rnd<T>(y * rk * rnd<T>(ld_t(a.k_norm_w, n * a.k_norm_w.stride[0])));
        }
        if (a.q_bias.data) {
          x = rnd<T>(x + rnd<T>(ld_t(a.q_bias, h * a.q_bias.stride[0] + r * a.q_bias.stride[1] +
                                                   n * a.q_bias.stride[2])));
          y = rnd<T>(y + rnd<T>(ld_t(a.k_bias, h * a.k_bias.stride[0] + r * a.k_bias.stride[1] +
                                                   n * a.k_bias.stride[2])));
        }
        qrow[n] = x;
        krow[n] = y;
      }
      __syncwarp();
      if (has_phase) {
        // SISO pairs (2m, 2m+1); MIMO pairs (m, 2S + m) — mamba3/ops.py:62-82.
        for (int m = lane; m < S; m += 32) {
          const int e0 = a.mimo_rotation ? m : 2 * m;
          const int e1 = a.mimo_rotation ? m + 2 * S : 2 * m + 1;
          float sn, cs;
          sincosf(sPh[j * (S + 1) + m], &sn, &cs);
          cs = rnd<T>(cs);
          sn = rnd<T>(sn);
          float x0 = qrow[e0], x1 = qrow[e1];
          qrow[e0] = rnd<T>(rnd<T>(x0 * cs) - rnd<T>(x1 * sn));
          qrow[e1] = rnd<T>(rnd<T>(x0 * sn) + rnd<T>(x1 * cs));
          x0 = krow[e0];
          x1 = krow[e1];
          krow[e0] = rnd<T>(rnd<T>(x0 * cs) - rnd<T>(x1 * sn));
          krow[e1] = rnd<T>(rnd<T>(x0 * sn) + rnd<T>(x1 * cs));
        }
        __syncwarp();
      }
      const bool last = (t0 + j == L - 1);
      const float sc = ts.scale[j];
      for (int n = lane; n < N; n += 32) {
        const float y = krow[n];
        if (last && a.final_k.data) {
          const m3_tensor& fk = a.final_k;
          static_cast<T*>(fk.data)[b * fk.stride[0] + h * fk.stride[1] + r * fk.stride[2] + n * fk.stride[3]] =
              from_f<T>(y);
        }
        krow[n] = rnd<T>(y * sc);
      }
      const int64_t vb = b * a.value.stride[0] + (int64_t)t * a.value.stride[1] + h * a.value.stride[2];
      const float ed = ts.edec[j];
      for (int p = lane; p < P; p += 32) {
        float v = to_f(vp[vb + p * a.value.stride[3]]);
        if (R > 1)
          v = rnd<T>(v * rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] +
                                             p * a.mimo_x.stride[2])));
        sV[row * PP + p] = v;
        sV2[row * PP + p] = rnd<T>(v * ed);
      }
    }
    __syncthreads();

    // ---- masked, decayed scores W = (Q K^T) o L, rounded to the activation dtype ----
    for (int idx = tid; idx < ROWS * ROWS; idx += blockDim.x) {
      const int i = idx / ROWS, jj = idx % ROWS;
      const int ti = i / R, tj = jj / R;
      float w = 0.0f;
      if (tj <= ti && ti < nt) {
        const float* qi = sQ + i * NP;
        const float* kj = sK + jj * NP;
        float dot = 0.0f;
        for (int n = 0; n < N; ++n) dot += qi[n] * kj[n];
        const float dec = (tj == ti) ? ts.diag[ti] : expf(ts.cum[ti] - ts.cum[tj]);
        w = rnd<T>(dot * dec);
      }
      sW[i * WP + jj] = w;
    }
    __syncthreads();

    // ---- outputs: inter (old state) + intra + D skip, SiLU gate ----
    for (int idx = tid; idx < ROWS * P; idx += blockDim.x) {
      const int i = idx / P, p = idx % P;
      const int ti = i / R, r = i % R;
      float y = 0.0f;
      if (ti < nt) {
        const float* qi = sQ + i * NP;
        const float* sp = sS + p * NP;
        float inter = 0.0f;
        for (int n = 0; n < N; ++n) inter += qi[n] * rnd<T>(sp[n]);
        float intra = 0.0f;
        const float* wi = sW + i * WP;
        for (int jj = 0; jj <= (ti + 1) * R - 1; ++jj) intra += wi[jj] * sV[jj * PP + p];
        const float v = sV[i * PP + p];
        y = ts.ecum[ti] * inter + intra + Dh * v;
        const int t = scan_token(a, t0 + ti);
        float z = to_f(zp[b * a.gate.stride[0] + (int64_t)t * a.gate.stride[1] + h * a.gate.stride[2] +
                          p * a.gate.stride[3]]);
        if (R > 1)
          z = rnd<T>(z * rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] +
                                             p * a.mimo_z.stride[2])));
        y *= siluf_(z);
        if (R > 1)
          y *= ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
      }
      sY[i * PP + p] = y;
    }
    __syncthreads();
    for (int idx = tid; idx < TOK * P; idx += blockDim.x) {
      const int j = idx / P, p = idx % P;
      if (j < nt) {
        float y = 0.0f;
        for (int r = 0; r < R; ++r) y += sY[(j * R + r) * PP + p];
        const int t = scan_token(a, t0 + j);
        yp[b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2] + p * a.y.stride[3]] = from_f<T>(y);
      }
    }
    // ---- state carry: S = e^{cum_last} S + V2^T K ----
    for (int idx = tid; idx < P * N; idx += blockDim.x) {
      const int p = idx / N, n = idx % N;
      float acc = 0.0f;
      for (int i = 0; i < nt * R; ++i) acc += sV2[i * PP + p] * sK[i * NP + n];
      sS[p * NP + n] = last_decay * sS[p * NP + n] + acc;
    }
    if (t0 + TOK >= L && a.final_phase.data && has_phase) {
      for (int s = tid; s < S; s += blockDim.x) {
        const m3_tensor& fp = a.final_phase;
        static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + s * fp.stride[2]] =
            sPh[(nt - 1) * (S + 1) + s];
      }
    }
    __syncthreads();
  }

  for (int i = tid; i < P * N; i += blockDim.x) {
    const int p = i / N, n = i % N;
    const m3_tensor& fs = a.final_state;
    static_cast<float*>(fs.data)[b * fs.stride[0] + h * fs.stride[1] + p * fs.stride[2] + n * fs.stride[3]] =
        sS[p * NP + n];
  }
}

template <typename T, int R>
static cudaError_t launch_simt_r(const m3_scan_args& a, cudaStream_t stream) {
  const int N = a.d_state, P = a.head_dim, S = a.num_angles;
  dim3 grid(a.heads, a.batch);
  auto try_rows = [&](auto rows_tag) -> cudaError_t {
    constexpr int ROWS = decltype(rows_tag)::value;
    const SimtLayout lay = simt_layout(ROWS, ROWS / R, N, P, S);
    auto kern = scan_simt_kernel<T, R, ROWS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.total);
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, lay.total, stream>>>(a);
    return cudaGetLastError();
  };
  constexpr size_t kMaxSmem = 227 * 1024;
  if (simt_layout(64, 64 / R, N, P, S).total <= kMaxSmem) return try_rows(std::integral_constant<int, 64>{});
  return try_rows(std::integral_constant<int, 32>{});
}

template <typename T>
static cudaError_t launch_simt_t(const m3_scan_args& a, cudaStream_t stream) {
  switch (a.rank) {
    case 1: return launch_simt_r<T, 1>(a, stream);
    case 2: return launch_simt_r<T, 2>(a, stream);
    case 4: return launch_simt_r<T, 4>(a, stream);
    default: return launch_simt_r<T, 8>(a, stream);
  }
}

// Smem bytes the SIMT kernel needs for these sizes (host check before launch).
size_t scan_simt_smem_bytes(int rank, int N, int P, int S) {
  constexpr size_t kMaxSmem = 227 * 1024;
  size_t s = simt_layout(64, 64 / rank, N, P, S).total;
  if (s <= kMaxSmem) return s;
  return simt_layout(32, 32 / rank, N, P, S).total;
}

cudaError_t launch_scan_simt(const m3_scan_args& a, cudaStream_t stream) {
  switch (a.value.dtype) {
    case M3_F32: return launch_simt_t<float>(a, stream);
    case M3_F16: return launch_simt_t<__half>(a, stream);
    default: return launch_simt_t<__nv_bfloat16>(a, stream);
  }
}

}  // namespace m3
