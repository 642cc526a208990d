// Single-token Mamba-3 decode step (SISO and MIMO), memory-bound on the FP32 state.
//
// Math (mamba3/model.py:460-484 and mamba3/ops.py:825-879):
//   phase' = fmod(phase + fmod(pi tanh(angle) dt, 2pi), 2pi);  q, k rotated by phase'
//   alpha = e^{adt}, beta = alpha dt (1 - sigma), gamma = dt sigma
//   S'    = alpha S + beta sum_r (x_prev mx_r) k_prev_r^T + gamma sum_r (x mx_r) k_r^T
//   y     = sum_r mo_r silu(z mz_r) (S' q_r + D x mx_r)
// In bf16/fp16 mode S' is rounded to the activation dtype for the output dot, as in the
// reference (ops.py:866).
//
// Grid (P / rows_per_cta, H, B), 128 threads. Each CTA recomputes the (tiny) phase and rotated
// q/k of its head, then streams its rows of the state exactly once: every state element is read
// and written by the same thread, so out_state may alias state (in-place decoding). Rows are
// split across CTAs so that even batch 1 puts several CTAs on every SM.
#include "common.cuh"

namespace m3 {

constexpr int kStepThreads = 128;

template <typename T, int R, int NPL>
__global__ void __launch_bounds__(kStepThreads) step_kernel(const m3_step_args a, int rows_per_cta) {
  const int h = blockIdx.y, b = blockIdx.z;
  const int p0 = blockIdx.x * rows_per_cta;
  const int N = a.d_state, P = a.head_dim, S = a.num_angles;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  extern __shared__ float sm[];
  float* s_cos = sm;            // S
  float* s_sin = sm + 64;       // S
  float* s_q = sm + 128;        // R * N   rotated q (activation-rounded)
  float* s_k = s_q + R * N;     // R * N   rotated k
  float* s_kp = s_k + R * N;    // R * N   previous rotated k (cache)
  const bool write_small = blockIdx.x == 0;

  const float dtv = ld_t(a.dt, b * a.dt.stride[0] + h * a.dt.stride[1]);
  for (int s = tid; s < S; s += blockDim.x) {
    const float th = ld_t(a.angle_rate, b * a.angle_rate.stride[0] + s * a.angle_rate.stride[1]);
    const float inc = fmodf((kPi * tanhf(th)) * dtv, kTwoPi);
    const float old = ld_t(a.phase, b * a.phase.stride[0] + h * a.phase.stride[1] + s * a.phase.stride[2]);
    const float ph = fmodf(old + inc, kTwoPi);
    if (write_small) {
      const m3_tensor& o = a.out_phase;
      static_cast<float*>(o.data)[b * o.stride[0] + h * o.stride[1] + s * o.stride[2]] = ph;
    }
    float sn, cs;
    sincosf(ph, &sn, &cs);
    s_cos[s] = rnd<T>(cs);
    s_sin[s] = rnd<T>(sn);
  }
  __syncthreads();
  // Rotated q/k: each thread owns rotation pairs (e0, e1) — SISO (2m, 2m+1), MIMO (m, m + N/2)
  // — so the partner element is always in the same thread.
  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const int half = N / 2;
  for (int i = tid; i < R * half; i += blockDim.x) {
    const int r = i / half, m = i % half;
    const int e0 = R > 1 ? m : 2 * m;
    const int e1 = R > 1 ? m + half : 2 * m + 1;
    const int64_t qb = b * a.q.stride[0] + h * a.q.stride[1] + r * a.q.stride[2];
    const int64_t kb = b * a.k.stride[0] + h * a.k.stride[1] + r * a.k.stride[2];
    float q0 = to_f(qp[qb + e0 * a.q.stride[3]]), q1 = to_f(qp[qb + e1 * a.q.stride[3]]);
    float k0 = to_f(kp[kb + e0 * a.k.stride[3]]), k1 = to_f(kp[kb + e1 * a.k.stride[3]]);
    if (a.q_bias.data) {
      const m3_tensor& qb_ = a.q_bias;
      const m3_tensor& kb_ = a.k_bias;
      const int64_t qo = h * qb_.stride[0] + r * qb_.stride[1];
      const int64_t ko = h * kb_.stride[0] + r * kb_.stride[1];
      q0 = rnd<T>(q0 + rnd<T>(ld_t(qb_, qo + e0 * qb_.stride[2])));
      q1 = rnd<T>(q1 + rnd<T>(ld_t(qb_, qo + e1 * qb_.stride[2])));
      k0 = rnd<T>(k0 + rnd<T>(ld_t(kb_, ko + e0 * kb_.stride[2])));
      k1 = rnd<T>(k1 + rnd<T>(ld_t(kb_, ko + e1 * kb_.stride[2])));
    }
    // SISO rotates pairs m < S; MIMO rotates (m, m + 2S) for m < S, and 2S == N/2 there.
    if (m < S) {
      const float cs = s_cos[m], sn = s_sin[m];
      const float nq0 = rnd<T>(rnd<T>(q0 * cs) - rnd<T>(q1 * sn));
      const float nq1 = rnd<T>(rnd<T>(q0 * sn) + rnd<T>(q1 * cs));
      const float nk0 = rnd<T>(rnd<T>(k0 * cs) - rnd<T>(k1 * sn));
      const float nk1 = rnd<T>(rnd<T>(k0 * sn) + rnd<T>(k1 * cs));
      q0 = nq0; q1 = nq1; k0 = nk0; k1 = nk1;
    }
    s_q[r * N + e0] = q0;
    s_q[r * N + e1] = q1;
    s_k[r * N + e0] = k0;
    s_k[r * N + e1] = k1;
    if (write_small) {
      const m3_tensor& o = a.out_k;
      T* op = static_cast<T*>(o.data);
      const int64_t ob = b * o.stride[0] + h * o.stride[1] + r * o.stride[2];
      op[ob + e0 * o.stride[3]] = from_f<T>(k0);
      op[ob + e1 * o.stride[3]] = from_f<T>(k1);
    }
  }
  for (int i = tid; i < R * N; i += blockDim.x) {
    const int r = i / N, n = i % N;
    const m3_tensor& t = a.prev_k;
    s_kp[i] = ld_t(t, b * t.stride[0] + h * t.stride[1] + r * t.stride[2] + n * t.stride[3]);
  }
  const float alpha = expf(ld_t(a.adt, b * a.adt.stride[0] + h * a.adt.stride[1]));
  const float sg = sigmoidf_(ld_t(a.trap, b * a.trap.stride[0] + h * a.trap.stride[1]));
  const float beta = (1.0f - sg) * dtv * alpha;
  const float gamma = sg * dtv;
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  __syncthreads();

  const float* st = static_cast<const float*>(a.state.data);
  float* so = static_cast<float*>(a.out_state.data);
  const int64_t sb = b * a.state.stride[0] + h * a.state.stride[1];
  const int64_t ob = b * a.out_state.stride[0] + h * a.out_state.stride[1];
  const int p_end = min(P, p0 + rows_per_cta);
  const int nwarps = blockDim.x / 32;
  for (int p = p0 + warp; p < p_end; p += nwarps) {
    // Per-row rank values of the current and previous input (activation-rounded, ops.py:193-199).
    const float x = ld_t(a.value, b * a.value.stride[0] + h * a.value.stride[1] + p * a.value.stride[2]);
    const float xp = ld_t(a.prev_value, b * a.prev_value.stride[0] + h * a.prev_value.stride[1] +
                                            p * a.prev_value.stride[2]);
    float xv[R], xpv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (R > 1) {
        const float mx = rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] +
                                                  p * a.mimo_x.stride[2]));
        xv[r] = rnd<T>(x * mx);
        xpv[r] = rnd<T>(xp * mx);
      } else {
        xv[r] = x;
        xpv[r] = xp;
      }
    }
    float sv[NPL];
#pragma unroll
    for (int e = 0; e < NPL; ++e) {
      const int n = lane + 32 * e;
      sv[e] = n < N ? st[sb + p * a.state.stride[2] + n * a.state.stride[3]] : 0.0f;
    }
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll
    for (int e = 0; e < NPL; ++e) {
      const int n = lane + 32 * e;
      if (n < N) {
        float po = 0.0f, co = 0.0f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          po += xpv[r] * s_kp[r * N + n];
          co += xv[r] * s_k[r * N + n];
        }
        const float ns = alpha * sv[e] + beta * po + gamma * co;
        so[ob + p * a.out_state.stride[2] + n * a.out_state.stride[3]] = ns;
        const float nr = rnd<T>(ns);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += nr * s_q[r * N + n];
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
    if (lane == 0) {
      const float z = ld_t(a.gate, b * a.gate.stride[0] + h * a.gate.stride[1] + p * a.gate.stride[2]);
      float y = 0.0f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float o = acc[r] + Dh * xv[r];
        float zr = z;
        if (R > 1)
          zr = rnd<T>(z * rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] +
                                                p * a.mimo_z.stride[2])));
        o *= siluf_(zr);
        if (R > 1)
          o *= ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
        y += o;
      }
      static_cast<T*>(a.y.data)[b * a.y.stride[0] + h * a.y.stride[1] + p * a.y.stride[2]] = from_f<T>(y);
    }
  }
}

template <typename T, int R>
static cudaError_t launch_step_r(const m3_step_args& a, cudaStream_t stream) {
  const int N = a.d_state, P = a.head_dim;
  // Split rows across CTAs until the grid covers every SM a few times.
  int rows = P;
  const long long pairs = (long long)a.batch * a.heads;
  while (rows > 4 && pairs * ((P + rows - 1) / rows) < 4 * 148) rows >>= 1;
  dim3 grid((P + rows - 1) / rows, a.heads, a.batch);
  const size_t smem = (128 + 3 * (size_t)R * N) * sizeof(float);
  auto go = [&](auto kern) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    kern<<<grid, kStepThreads, smem, stream>>>(a, rows);
    return cudaGetLastError();
  };
  if (N <= 32) return go(step_kernel<T, R, 1>);
  if (N <= 64) return go(step_kernel<T, R, 2>);
  if (N <= 128) return go(step_kernel<T, R, 4>);
  return go(step_kernel<T, R, 8>);
}

template <typename T>
static cudaError_t launch_step_t(const m3_step_args& a, cudaStream_t stream) {
  switch (a.rank) {
    case 1: return launch_step_r<T, 1>(a, stream);
    case 2: return launch_step_r<T, 2>(a, stream);
    case 4: return launch_step_r<T, 4>(a, stream);
    default: return launch_step_r<T, 8>(a, stream);
  }
}

cudaError_t launch_step(const m3_step_args& a, cudaStream_t stream) {
  switch (a.value.dtype) {
    case M3_F32: return launch_step_t<float>(a, stream);
    case M3_F16: return launch_step_t<__half>(a, stream);
    default: return launch_step_t<__nv_bfloat16>(a, stream);
  }
}

}  // namespace m3
