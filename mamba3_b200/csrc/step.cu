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
#ifndef M3_STEP_BIG_ROWS
#define M3_STEP_BIG_ROWS 8
#endif
constexpr int kStepBigRows = M3_STEP_BIG_ROWS;  // state rows per warp in the stream pass at large batch

// Per-(batch, head) prologue shared by both step kernels: new phase (written by the CTA with
// write_small), rotated q/k into s_q/s_k (activation-rounded), previous k into s_kp, and the
// scalars alpha, beta, gamma, D. Ends with __syncthreads().
struct StepScalars {
  float alpha, beta, gamma, Dh;
};

// dt and adt of (b, h). Model mode (dt_bias given, mamba3/model.py:195-198): dt holds the raw
// delta logits and adt the raw decay logits; dt = softplus(delta + dt_bias),
// adt = min(-heavy_tail(decay), -1e-4) * dt. Otherwise both are taken as given.
__device__ __forceinline__ void step_dt_adt(const m3_step_args& a, int b, int h, float& dtv, float& adtv) {
  const float d = ld_t(a.dt, b * a.dt.stride[0] + h * a.dt.stride[1]);
  const float g = ld_t(a.adt, b * a.adt.stride[0] + h * a.adt.stride[1]);
  if (a.dt_bias.data) {
    dtv = softplusf_(d + ld_t(a.dt_bias, h * a.dt_bias.stride[0]));
    adtv = fminf(-heavy_tailf(g), -kAFloor) * dtv;
  } else {
    dtv = d;
    adtv = g;
  }
}

// Sum of squares of row r of a [B,H,R,N] tensor over one warp (every lane gets the total).
template <typename T>
__device__ __forceinline__ float row_sumsq(const m3_tensor& t, int b, int h, int r, int N, int lane) {
  const T* p = static_cast<const T*>(t.data) + b * t.stride[0] + h * t.stride[1] + r * t.stride[2];
  float acc = 0.0f;
  for (int n = lane; n < N; n += 32) {
    const float v = to_f(p[n * t.stride[3]]);
    acc += v * v;
  }
  return warp_sum(acc);
}

// RMS-normalised element (F.rms_norm with the weight cast to the activation dtype, one rounding).
template <typename T>
__device__ __forceinline__ float norm_elem(float x, float inv_rms, const m3_tensor& w, int e) {
  return rnd<T>(x * inv_rms * rnd<T>(ld_t(w, e * w.stride[0])));
}

template <typename T, int R>
__device__ __forceinline__ StepScalars step_prologue(const m3_step_args& a, int b, int h, bool write_small, float* sm) {
  // Every global load of the prologue is issued first (one memory round trip), then the math.
  constexpr int kPairIters = R;      // R * (N / 2) <= 128 R pairs for N <= 256, 128 threads
  constexpr int kPrevIters = 2 * R;  // R * N <= 256 R elements
  const int N = a.d_state, S = a.num_angles;
  const int tid = threadIdx.x;
  const int half = N / 2;
  float* s_cos = sm;            // S
  float* s_sin = sm + 64;       // S
  float* s_q = sm + 128;        // R * N   rotated q (activation-rounded)
  float* s_k = s_q + R * N;     // R * N   rotated k
  float* s_kp = s_k + R * N;    // R * N   previous rotated k (cache)
  float* s_rn = s_kp + R * N;   // 2 R     inverse RMS of the q rows, then of the k rows
  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const bool has_norm = a.q_norm_w.data != nullptr;
  if (has_norm) {
    const int warp = tid >> 5, lane = tid & 31;
    for (int j = warp; j < 2 * R; j += kStepThreads / 32) {
      const float ss = row_sumsq<T>(j < R ? a.q : a.k, b, h, j % R, N, lane);
      if (lane == 0) s_rn[j] = rsqrtf(ss / N + a.norm_eps);
    }
    __syncthreads();
  }

  float dtv, adtv;
  step_dt_adt(a, b, h, dtv, adtv);
  const float trapv = ld_t(a.trap, b * a.trap.stride[0] + h * a.trap.stride[1]);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  float th = 0.0f, old = 0.0f;
  if (tid < S) {
    th = ld_t(a.angle_rate, b * a.angle_rate.stride[0] + tid * a.angle_rate.stride[1]);
    old = ld_t(a.phase, b * a.phase.stride[0] + h * a.phase.stride[1] + tid * a.phase.stride[2]);
  }
  // Rotation pairs (e0, e1) — SISO (2m, 2m+1), MIMO (m, m + N/2) — so both elements of a pair
  // are in the same thread.
  float q0[kPairIters], q1[kPairIters], k0[kPairIters], k1[kPairIters];
#pragma unroll
  for (int j = 0; j < kPairIters; ++j) {
    const int i = tid + j * kStepThreads;
    q0[j] = q1[j] = k0[j] = k1[j] = 0.0f;
    if (i < R * half) {
      const int r = i / half, m = i % half;
      const int e0 = R > 1 ? m : 2 * m;
      const int e1 = R > 1 ? m + half : 2 * m + 1;
      const int64_t qb = b * a.q.stride[0] + h * a.q.stride[1] + r * a.q.stride[2];
      const int64_t kb = b * a.k.stride[0] + h * a.k.stride[1] + r * a.k.stride[2];
      q0[j] = to_f(qp[qb + e0 * a.q.stride[3]]);
      q1[j] = to_f(qp[qb + e1 * a.q.stride[3]]);
      k0[j] = to_f(kp[kb + e0 * a.k.stride[3]]);
      k1[j] = to_f(kp[kb + e1 * a.k.stride[3]]);
      if (has_norm) {
        q0[j] = norm_elem<T>(q0[j], s_rn[r], a.q_norm_w, e0);
        q1[j] = norm_elem<T>(q1[j], s_rn[r], a.q_norm_w, e1);
        k0[j] = norm_elem<T>(k0[j], s_rn[R + r], a.k_norm_w, e0);
        k1[j] = norm_elem<T>(k1[j], s_rn[R + r], a.k_norm_w, e1);
      }
      if (a.q_bias.data) {
        const m3_tensor& qb_ = a.q_bias;
        const m3_tensor& kb_ = a.k_bias;
        const int64_t qo = h * qb_.stride[0] + r * qb_.stride[1];
        const int64_t ko = h * kb_.stride[0] + r * kb_.stride[1];
        q0[j] = rnd<T>(q0[j] + rnd<T>(ld_t(qb_, qo + e0 * qb_.stride[2])));
        q1[j] = rnd<T>(q1[j] + rnd<T>(ld_t(qb_, qo + e1 * qb_.stride[2])));
        k0[j] = rnd<T>(k0[j] + rnd<T>(ld_t(kb_, ko + e0 * kb_.stride[2])));
        k1[j] = rnd<T>(k1[j] + rnd<T>(ld_t(kb_, ko + e1 * kb_.stride[2])));
      }
    }
  }
  float kprev[kPrevIters];
#pragma unroll
  for (int j = 0; j < kPrevIters; ++j) {
    const int i = tid + j * kStepThreads;
    kprev[j] = 0.0f;
    if (i < R * N) {
      const int r = i / N, n = i % N;
      const m3_tensor& t = a.prev_k;
      kprev[j] = ld_t(t, b * t.stride[0] + h * t.stride[1] + r * t.stride[2] + n * t.stride[3]);
    }
  }

  if (tid < S) {
    const float inc = fmodf((kPi * tanhf(th)) * dtv, kTwoPi);
    const float ph = fmodf(old + inc, kTwoPi);
    if (write_small) {
      const m3_tensor& o = a.out_phase;
      static_cast<float*>(o.data)[b * o.stride[0] + h * o.stride[1] + tid * o.stride[2]] = ph;
    }
    float sn, cs;
    sincosf(ph, &sn, &cs);
    s_cos[tid] = rnd<T>(cs);
    s_sin[tid] = rnd<T>(sn);
  }
#pragma unroll
  for (int j = 0; j < kPrevIters; ++j) {
    const int i = tid + j * kStepThreads;
    if (i < R * N) s_kp[i] = kprev[j];
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPairIters; ++j) {
    const int i = tid + j * kStepThreads;
    if (i < R * half) {
      const int r = i / half, m = i % half;
      const int e0 = R > 1 ? m : 2 * m;
      const int e1 = R > 1 ? m + half : 2 * m + 1;
      float a0 = q0[j], a1 = q1[j], c0 = k0[j], c1 = k1[j];
      // SISO rotates pairs m < S; MIMO rotates (m, m + 2S) for m < S, and 2S == N/2 there.
      if (m < S) {
        const float cs = s_cos[m], sn = s_sin[m];
        const float nq0 = rnd<T>(rnd<T>(a0 * cs) - rnd<T>(a1 * sn));
        const float nq1 = rnd<T>(rnd<T>(a0 * sn) + rnd<T>(a1 * cs));
        const float nk0 = rnd<T>(rnd<T>(c0 * cs) - rnd<T>(c1 * sn));
        const float nk1 = rnd<T>(rnd<T>(c0 * sn) + rnd<T>(c1 * cs));
        a0 = nq0; a1 = nq1; c0 = nk0; c1 = nk1;
      }
      s_q[r * N + e0] = a0;
      s_q[r * N + e1] = a1;
      s_k[r * N + e0] = c0;
      s_k[r * N + e1] = c1;
      if (write_small) {
        const m3_tensor& o = a.out_k;
        T* op = static_cast<T*>(o.data);
        const int64_t ob = b * o.stride[0] + h * o.stride[1] + r * o.stride[2];
        op[ob + e0 * o.stride[3]] = from_f<T>(c0);
        op[ob + e1 * o.stride[3]] = from_f<T>(c1);
      }
    }
  }
  const float alpha = expf(adtv);
  const float sg = sigmoidf_(trapv);
  const float beta = (1.0f - sg) * dtv * alpha;
  const float gamma = sg * dtv;
  __syncthreads();
  return StepScalars{alpha, beta, gamma, Dh};
}

template <typename T, int R, int NPL>
__global__ void __launch_bounds__(kStepThreads) step_kernel(const m3_step_args a, int rows_per_cta) {
  const int h = blockIdx.y, b = blockIdx.z;
  const int p0 = blockIdx.x * rows_per_cta;
  const int N = a.d_state, P = a.head_dim;
  // Launched as a programmatic dependent of the projection before it: release the next kernel, pull
  // this CTA's state rows towards L2 (a prefetch has no effect on the values read), then wait for
  // the previous kernel before reading any input.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (a.state.stride[3] == 1) {
    const float* sp = static_cast<const float*>(a.state.data) + b * a.state.stride[0] + h * a.state.stride[1];
    for (int i = threadIdx.x; i < rows_per_cta * ((N + 31) / 32); i += blockDim.x) {
      const int p = p0 + i / ((N + 31) / 32), n = 32 * (i % ((N + 31) / 32));
      if (p < P) asm volatile("prefetch.global.L2 [%0];" ::"l"(sp + p * a.state.stride[2] + n));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  extern __shared__ float sm[];
  const float* s_q = sm + 128;
  const float* s_k = s_q + R * N;
  const float* s_kp = s_k + R * N;
  const StepScalars sc = step_prologue<T, R>(a, b, h, blockIdx.x == 0, sm);
  const float alpha = sc.alpha, beta = sc.beta, gamma = sc.gamma, Dh = sc.Dh;

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


// The state is touched exactly once per step: stream it past the caches (evict-first loads and
// stores). Measured on B200 (CUDA-graph replay of one layer, Mamba3(2560) bf16): batch 64 rank 1
// 86.1 -> 70.3 us, batch 256 317.7 -> 292.8 us, batch 64 rank 4 174.2 -> 134.2 us against plain
// loads and stores (which leave the just-written state competing for L2 with the next rows).
__device__ __forceinline__ float4 load_state4(const float* p) {
#ifdef M3_STEP_NO_STREAMING
  return *reinterpret_cast<const float4*>(p);
#else
  return __ldcs(reinterpret_cast<const float4*>(p));
#endif
}
__device__ __forceinline__ void store_state4(float* p, float4 v) {
#ifdef M3_STEP_NO_STREAMING
  *reinterpret_cast<float4*>(p) = v;
#else
  __stcs(reinterpret_cast<float4*>(p), v);
#endif
}

// Two-pass decode for state rows that are contiguous and 16-byte aligned.
//
// Pass 1 (step_prep_kernel, one CTA per (batch, head)): phase advance, rotation of q/k, the new
// phase and rotated-k cache outputs, and the decay scalars, into the workspace:
//   ws[(b H + h) W + ...], W = 2 R N + 4 floats: rotated q [R][N] and rotated k [R][N] in the
//   activation type T (they are T-rounded values; 16-bit halves the stream pass's reads), then, at
//   float 2 R N, alpha, beta,
//   gamma, D.
// Pass 2 (step_stream_kernel): a pure stream over the FP32 state. Lane l of a warp holds the
// float4 groups n = 4 l + 128 v (v < NV); every state row of the CTA, the per-head vectors and the
// per-row inputs are loaded before any arithmetic, so each CTA has all of its HBM reads in flight
// at once; each warp owns RPW consecutive rows.
// One warp per (batch, head); four per CTA. Lane l owns angles l, l + 32 and rotation pairs
// i = l + 32 j; the cos/sin of a pair's angle comes from its owner lane by shuffle.
template <typename T, int R, int NT>
__global__ void __launch_bounds__(kStepThreads) step_prep_kernel(const m3_step_args a) {
  // the stream pass may start now: it loads its state rows before it waits for this grid
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (kStepThreads / 32) + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.batch * a.heads) return;
  const int b = (int)(wid / a.heads), h = (int)(wid % a.heads);
  // NT: d_state known at compile time (0 = read it from the arguments).
  const int N = NT ? NT : a.d_state, S = a.num_angles, half = N / 2;
  float* ws = static_cast<float*>(a.workspace.data) + wid * (2 * R * N + 4);
  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);

  float dtv, adtv;
  step_dt_adt(a, b, h, dtv, adtv);
  const float trapv = ld_t(a.trap, b * a.trap.stride[0] + h * a.trap.stride[1]);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  // Model mode: inverse RMS of q row r and k row r live in lane r (fetched by shuffle).
  const bool has_norm = a.q_norm_w.data != nullptr;
  float my_rq = 1.0f, my_rk = 1.0f;
  if (has_norm) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float sq = row_sumsq<T>(a.q, b, h, r, N, lane);
      const float sk = row_sumsq<T>(a.k, b, h, r, N, lane);
      if (lane == r) {
        my_rq = rsqrtf(sq / N + a.norm_eps);
        my_rk = rsqrtf(sk / N + a.norm_eps);
      }
    }
  }
  float th[2] = {0.f, 0.f}, old[2] = {0.f, 0.f};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int sidx = lane + 32 * u;
    if (sidx < S) {
      th[u] = ld_t(a.angle_rate, b * a.angle_rate.stride[0] + sidx * a.angle_rate.stride[1]);
      old[u] = ld_t(a.phase, b * a.phase.stride[0] + h * a.phase.stride[1] + sidx * a.phase.stride[2]);
    }
  }
  // Rotation pairs (e0, e1): SISO (2m, 2m+1), MIMO (m, m + N/2); processed 4 pairs per lane at a time
  // so that the loads of a batch are in flight together.
  const int npairs = R * half;
  float cs[2] = {1.f, 1.f}, sn[2] = {0.f, 0.f};
  for (int base = 0; base < npairs; base += 128) {
    float q0[4], q1[4], k0[4], k1[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + lane + 32 * u;
      q0[u] = q1[u] = k0[u] = k1[u] = 0.f;
      const int rr = (i < npairs ? i : npairs - 1) / half;
      const float rq = __shfl_sync(0xffffffffu, my_rq, rr), rk = __shfl_sync(0xffffffffu, my_rk, rr);
      if (i < npairs) {
        const int r = i / half, m = i % half;
        const int e0 = R > 1 ? m : 2 * m, e1 = R > 1 ? m + half : 2 * m + 1;
        const int64_t qb = b * a.q.stride[0] + h * a.q.stride[1] + r * a.q.stride[2];
        const int64_t kb = b * a.k.stride[0] + h * a.k.stride[1] + r * a.k.stride[2];
        q0[u] = to_f(qp[qb + e0 * a.q.stride[3]]);
        q1[u] = to_f(qp[qb + e1 * a.q.stride[3]]);
        k0[u] = to_f(kp[kb + e0 * a.k.stride[3]]);
        k1[u] = to_f(kp[kb + e1 * a.k.stride[3]]);
        if (has_norm) {
          q0[u] = norm_elem<T>(q0[u], rq, a.q_norm_w, e0);
          q1[u] = norm_elem<T>(q1[u], rq, a.q_norm_w, e1);
          k0[u] = norm_elem<T>(k0[u], rk, a.k_norm_w, e0);
          k1[u] = norm_elem<T>(k1[u], rk, a.k_norm_w, e1);
        }
        if (a.q_bias.data) {
          const m3_tensor& qb_ = a.q_bias;
          const m3_tensor& kb_ = a.k_bias;
          const int64_t qo = h * qb_.stride[0] + r * qb_.stride[1];
          const int64_t ko = h * kb_.stride[0] + r * kb_.stride[1];
          q0[u] = rnd<T>(q0[u] + rnd<T>(ld_t(qb_, qo + e0 * qb_.stride[2])));
          q1[u] = rnd<T>(q1[u] + rnd<T>(ld_t(qb_, qo + e1 * qb_.stride[2])));
          k0[u] = rnd<T>(k0[u] + rnd<T>(ld_t(kb_, ko + e0 * kb_.stride[2])));
          k1[u] = rnd<T>(k1[u] + rnd<T>(ld_t(kb_, ko + e1 * kb_.stride[2])));
        }
      }
    }
    if (base == 0) {
      // New phase (computed while the first batch of q/k loads is in flight).
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int sidx = lane + 32 * u;
        if (sidx < S) {
          const float inc = fmodf((kPi * tanhf(th[u])) * dtv, kTwoPi);
          const float ph = fmodf(old[u] + inc, kTwoPi);
          const m3_tensor& o = a.out_phase;
          static_cast<float*>(o.data)[b * o.stride[0] + h * o.stride[1] + sidx * o.stride[2]] = ph;
          float s_, c_;
          __sincosf(ph, &s_, &c_);  // |ph| < 2 pi: absolute error ~1e-6
          cs[u] = rnd<T>(c_);
          sn[u] = rnd<T>(s_);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + lane + 32 * u;
      const int m = (i < npairs) ? i % half : 0;
      // cos/sin of angle m live in lane m % 32, slot m / 32 (every lane joins the shuffles).
      const float c0 = __shfl_sync(0xffffffffu, cs[0], m & 31), c1 = __shfl_sync(0xffffffffu, cs[1], m & 31);
      const float s0 = __shfl_sync(0xffffffffu, sn[0], m & 31), s1 = __shfl_sync(0xffffffffu, sn[1], m & 31);
      if (i < npairs) {
        const int r = i / half;
        const int e0 = R > 1 ? m : 2 * m, e1 = R > 1 ? m + half : 2 * m + 1;
        float a0 = q0[u], a1 = q1[u], b0 = k0[u], b1 = k1[u];
        // SISO rotates pairs m < S; MIMO rotates (m, m + 2S) for m < S, and 2S == N/2 there.
        if (m < S) {
          const float c = (m < 32) ? c0 : c1, sv = (m < 32) ? s0 : s1;
          const float nq0 = rnd<T>(rnd<T>(a0 * c) - rnd<T>(a1 * sv));
          const float nq1 = rnd<T>(rnd<T>(a0 * sv) + rnd<T>(a1 * c));
          const float nk0 = rnd<T>(rnd<T>(b0 * c) - rnd<T>(b1 * sv));
          const float nk1 = rnd<T>(rnd<T>(b0 * sv) + rnd<T>(b1 * c));
          a0 = nq0; a1 = nq1; b0 = nk0; b1 = nk1;
        }
        T* wst = reinterpret_cast<T*>(ws);
        wst[r * N + e0] = from_f<T>(a0);
        wst[r * N + e1] = from_f<T>(a1);
        wst[R * N + r * N + e0] = from_f<T>(b0);
        wst[R * N + r * N + e1] = from_f<T>(b1);
        const m3_tensor& o = a.out_k;
        T* op = static_cast<T*>(o.data);
        const int64_t ob = b * o.stride[0] + h * o.stride[1] + r * o.stride[2];
        op[ob + e0 * o.stride[3]] = from_f<T>(b0);
        op[ob + e1 * o.stride[3]] = from_f<T>(b1);
      }
    }
  }
  if (lane == 0) {
    const float alpha = expf(adtv);
    const float sg = sigmoidf_(trapv);
    *reinterpret_cast<float4*>(ws + 2 * R * N) = make_float4(alpha, (1.0f - sg) * dtv * alpha, sg * dtv, Dh);
  }
}

// Unpack eight 16-bit values of a 16-byte word.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 w, float* out) {
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = to_f(e[i]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 w;
  T* e = reinterpret_cast<T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = from_f<T>(v[i]);
  return w;
}

// step_prep_kernel for N = 128 with contiguous, 16-byte aligned 16-bit q / k / out_k rows: the same
// per-element arithmetic, laid out so that each lane owns whole rotation pairs. Unit u (lane u,
// u < 8 R) is row u / 8, pairs m = 8 c .. 8 c + 7 with c = u % 8: SISO elements 16 c .. 16 c + 15
// (pairs (2m, 2m + 1)), MIMO elements 8 c .. 8 c + 7 and 64 + 8 c .. (pairs (m, m + 64)). The RMS
// sums of a row close within its 8 lanes; all row loads and stores are 16-byte vectors.
template <typename T, int R>
__global__ void __launch_bounds__(kStepThreads) step_prep_vec_kernel(const m3_step_args a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int N = 128, kUnits = 8 * R;
  constexpr bool kMimo = R > 1;
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (kStepThreads / 32) + (threadIdx.x >> 5);
  if (wid >= (int64_t)a.batch * a.heads) return;
  const int b = (int)(wid / a.heads), h = (int)(wid % a.heads);
  const int S = a.num_angles;
  float* ws = static_cast<float*>(a.workspace.data) + wid * (2 * R * N + 4);
  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);

  float dtv, adtv;
  step_dt_adt(a, b, h, dtv, adtv);
  const float trapv = ld_t(a.trap, b * a.trap.stride[0] + h * a.trap.stride[1]);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  float th[2] = {0.f, 0.f}, old[2] = {0.f, 0.f};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int sidx = lane + 32 * u;
    if (sidx < S) {
      th[u] = ld_t(a.angle_rate, b * a.angle_rate.stride[0] + sidx * a.angle_rate.stride[1]);
      old[u] = ld_t(a.phase, b * a.phase.stride[0] + h * a.phase.stride[1] + sidx * a.phase.stride[2]);
    }
  }
  // Raw q / k of this lane's units, issued before the phase arithmetic.
  constexpr int kIters = (kUnits + 31) / 32;
  float q[kIters][16], k[kIters][16];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int u = lane + 32 * it, r = min(u, kUnits - 1) / 8, c = u % 8;
    const int64_t qb = b * a.q.stride[0] + h * a.q.stride[1] + r * a.q.stride[2];
    const int64_t kb = b * a.k.stride[0] + h * a.k.stride[1] + r * a.k.stride[2];
    const int o0 = kMimo ? 8 * c : 16 * c, o1 = kMimo ? 64 + 8 * c : 16 * c + 8;
    uint4 w[4] = {};
    if (u < kUnits) {
      w[0] = *reinterpret_cast<const uint4*>(qp + qb + o0);
      w[1] = *reinterpret_cast<const uint4*>(qp + qb + o1);
      w[2] = *reinterpret_cast<const uint4*>(kp + kb + o0);
      w[3] = *reinterpret_cast<const uint4*>(kp + kb + o1);
    }
    unpack8<T>(w[0], q[it]);
    unpack8<T>(w[1], q[it] + 8);
    unpack8<T>(w[2], k[it]);
    unpack8<T>(w[3], k[it] + 8);
  }
  // New phase: lane s owns angles s and s + 32.
  float cs[2] = {1.f, 1.f}, sn[2] = {0.f, 0.f};
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int sidx = lane + 32 * u;
    if (sidx < S) {
      const float inc = fmodf((kPi * tanhf(th[u])) * dtv, kTwoPi);
      const float ph = fmodf(old[u] + inc, kTwoPi);
      const m3_tensor& o = a.out_phase;
      static_cast<float*>(o.data)[b * o.stride[0] + h * o.stride[1] + sidx * o.stride[2]] = ph;
      float s_, c_;
      __sincosf(ph, &s_, &c_);  // |ph| < 2 pi: absolute error ~1e-6
      cs[u] = rnd<T>(c_);
      sn[u] = rnd<T>(s_);
    }
  }
  const bool has_norm = a.q_norm_w.data != nullptr;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int u = lane + 32 * it, r = min(u, kUnits - 1) / 8, c = u % 8;
    const int o0 = kMimo ? 8 * c : 16 * c, o1 = kMimo ? 64 + 8 * c : 16 * c + 8;
    if (has_norm) {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sq += q[it][i] * q[it][i];
        sk += k[it][i] * k[it][i];
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, off);
        sk += __shfl_xor_sync(0xffffffffu, sk, off);
      }
      const float rq = rsqrtf(sq / N + a.norm_eps), rk = rsqrtf(sk / N + a.norm_eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = i < 8 ? o0 + i : o1 + i - 8;
        q[it][i] = norm_elem<T>(q[it][i], rq, a.q_norm_w, e);
        k[it][i] = norm_elem<T>(k[it][i], rk, a.k_norm_w, e);
      }
    }
    if (a.q_bias.data) {
      const m3_tensor& qb_ = a.q_bias;
      const m3_tensor& kb_ = a.k_bias;
      const int64_t qo = h * qb_.stride[0] + r * qb_.stride[1];
      const int64_t ko = h * kb_.stride[0] + r * kb_.stride[1];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = i < 8 ? o0 + i : o1 + i - 8;
        q[it][i] = rnd<T>(q[it][i] + rnd<T>(ld_t(qb_, qo + e * qb_.stride[2])));
        k[it][i] = rnd<T>(k[it][i] + rnd<T>(ld_t(kb_, ko + e * kb_.stride[2])));
      }
    }
    // Rotation of pairs m = 8 c + j < S; (cos, sin) of angle m come from lane m % 32.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = 8 * c + j;
      float cv = __shfl_sync(0xffffffffu, cs[0], m & 31), sv = __shfl_sync(0xffffffffu, sn[0], m & 31);
      if (S > 32) {  // warp-uniform
        const float c1 = __shfl_sync(0xffffffffu, cs[1], m & 31), s1 = __shfl_sync(0xffffffffu, sn[1], m & 31);
        if (m >= 32) {
          cv = c1;
          sv = s1;
        }
      }
      if (m < S) {
        const int i0 = kMimo ? j : 2 * j, i1 = kMimo ? j + 8 : 2 * j + 1;
        const float a0 = q[it][i0], a1 = q[it][i1], b0 = k[it][i0], b1 = k[it][i1];
        q[it][i0] = rnd<T>(rnd<T>(a0 * cv) - rnd<T>(a1 * sv));
        q[it][i1] = rnd<T>(rnd<T>(a0 * sv) + rnd<T>(a1 * cv));
        k[it][i0] = rnd<T>(rnd<T>(b0 * cv) - rnd<T>(b1 * sv));
        k[it][i1] = rnd<T>(rnd<T>(b0 * sv) + rnd<T>(b1 * cv));
      }
    }
    if (u < kUnits) {
      const float* qa = q[it];
      const float* ka = k[it];
      // rotated q / k in the activation type: 8 elements = one 16-byte word per half row
      T* wst = reinterpret_cast<T*>(ws);
      *reinterpret_cast<uint4*>(wst + r * N + o0) = pack8<T>(qa);
      *reinterpret_cast<uint4*>(wst + r * N + o1) = pack8<T>(qa + 8);
      *reinterpret_cast<uint4*>(wst + R * N + r * N + o0) = pack8<T>(ka);
      *reinterpret_cast<uint4*>(wst + R * N + r * N + o1) = pack8<T>(ka + 8);
      const m3_tensor& o = a.out_k;
      T* op = static_cast<T*>(o.data) + b * o.stride[0] + h * o.stride[1] + r * o.stride[2];
      *reinterpret_cast<uint4*>(op + o0) = pack8<T>(ka);
      *reinterpret_cast<uint4*>(op + o1) = pack8<T>(ka + 8);
    }
  }
  if (lane == 0) {
    const float alpha = expf(adtv);
    const float sg = sigmoidf_(trapv);
    *reinterpret_cast<float4*>(ws + 2 * R * N) = make_float4(alpha, (1.0f - sg) * dtv * alpha, sg * dtv, Dh);
  }
}

// Rows of a [B, H, R, N] 16-bit tensor that are contiguous and start on 16-byte boundaries.
static bool rows16(const m3_tensor& t) {
  return t.dtype != M3_F32 && t.stride[3] == 1 && (reinterpret_cast<uintptr_t>(t.data) & 15u) == 0 &&
         t.stride[0] % 8 == 0 && t.stride[1] % 8 == 0 && t.stride[2] % 8 == 0;
}

// Four consecutive activation-type values of a row: packed (two 32-bit words of 16-bit pairs) or
// widened to float. float activations are always held as floats.
template <typename T, bool kPacked> struct Q4 {
  float4 f;
  __device__ __forceinline__ void zero() { f = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (sizeof(T) == 2) {
      const uint2 w = *reinterpret_cast<const uint2*>(p);
      const T* e = reinterpret_cast<const T*>(&w);
      f = make_float4(to_f(e[0]), to_f(e[1]), to_f(e[2]), to_f(e[3]));
    } else {
      f = *reinterpret_cast<const float4*>(p);
    }
  }
  __device__ __forceinline__ void set(float a, float b, float c, float d) { f = make_float4(a, b, c, d); }
  __device__ __forceinline__ float4 get() const { return f; }
};
template <typename T> struct Q4<T, true> {
  uint2 w;
  __device__ __forceinline__ void zero() { w = make_uint2(0u, 0u); }
  __device__ __forceinline__ void load(const T* p) {
    if constexpr (sizeof(T) == 2) {
      w = *reinterpret_cast<const uint2*>(p);
    } else {
      set(p[0], p[1], p[2], p[3]);
    }
  }
  __device__ __forceinline__ void set(float a, float b, float c, float d) {
    T e[4] = {from_f<T>(a), from_f<T>(b), from_f<T>(c), from_f<T>(d)};
    w = *reinterpret_cast<const uint2*>(e);
  }
  __device__ __forceinline__ float4 get() const {
    const T* e = reinterpret_cast<const T*>(&w);
    return make_float4(to_f(e[0]), to_f(e[1]), to_f(e[2]), to_f(e[3]));
  }
};
template <> struct Q4<float, true> : Q4<float, false> {};

template <typename T, int R, int NV, int RPW>
__global__ void __launch_bounds__(kStepThreads) step_stream_kernel(const m3_step_args a, int vec_prev_k) {
  const int h = blockIdx.y, b = blockIdx.z;
  const int N = a.d_state, P = a.head_dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int p0 = blockIdx.x * (RPW * (kStepThreads / 32)) + warp * RPW;
  const float* st = static_cast<const float*>(a.state.data) + b * a.state.stride[0] + h * a.state.stride[1];
  float* so = static_cast<float*>(a.out_state.data) + b * a.out_state.stride[0] + h * a.out_state.stride[1];
  const float* ws = static_cast<const float*>(a.workspace.data) + ((int64_t)b * a.heads + h) * (2 * R * N + 4);
  float4 sv[RPW][NV];
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int n = 4 * lane + 128 * v, p = p0 + rr;
      sv[rr][v] = (p < P && n < N) ? load_state4(st + p * a.state.stride[2] + n) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // Launched as a programmatic dependent of the prep pass: the state rows above do not depend on
  // it, so their loads are in flight before this waits for the prep grid's workspace.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // q, k and the previous k of this lane's four columns: 16-bit values, kept packed (two per word)
  // at rank > 1 to bound registers, widened to float at rank 1.
  Q4<T, (R > 1)> qv[R][NV], kv[R][NV], kpv[R][NV];
  const T* wst = reinterpret_cast<const T*>(ws);
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int n = 4 * lane + 128 * v;
      qv[r][v].zero();
      kv[r][v].zero();
      kpv[r][v].zero();
      if (n < N) {
        qv[r][v].load(wst + r * N + n);
        kv[r][v].load(wst + R * N + r * N + n);
        const m3_tensor& t = a.prev_k;
        const int64_t kb = b * t.stride[0] + h * t.stride[1] + r * t.stride[2];
        if (vec_prev_k) {  // four packed 16-bit values
          kpv[r][v].load(static_cast<const T*>(t.data) + kb + n);
        } else {
          kpv[r][v].set(ld_t(t, kb + n * t.stride[3]), ld_t(t, kb + (n + 1) * t.stride[3]),
                        ld_t(t, kb + (n + 2) * t.stride[3]), ld_t(t, kb + (n + 3) * t.stride[3]));
        }
      }
    }
  }
  const float4 sc = *reinterpret_cast<const float4*>(ws + 2 * R * N);  // alpha, beta, gamma, D
  // Rank-scattered layout (R in {2, 4}, R * RPW <= 32): lane L stands for rank L / G of row L % G
  // (G = 32 / R lanes per rank). It holds that row's x mx_r, xp mx_r, z mz_r and mo_r, hands them to
  // the other lanes by shuffle, receives the row's sum for its rank from a reduce-scatter and runs one
  // (row, rank) epilogue; the ranks are then summed across lane groups.
  constexpr bool kScatter = R > 1 && R * RPW <= 32;
  constexpr int G = 32 / R;
  const int lrow = kScatter ? lane % G : lane, lrank = kScatter ? lane / G : 0;
  float x_l = 0.f, xp_l = 0.f, z_l = 0.f, mo_l = 1.f;
  if (lrow < RPW && p0 + lrow < P) {
    const int p = p0 + lrow;
    x_l = ld_t(a.value, b * a.value.stride[0] + h * a.value.stride[1] + p * a.value.stride[2]);
    xp_l = ld_t(a.prev_value, b * a.prev_value.stride[0] + h * a.prev_value.stride[1] + p * a.prev_value.stride[2]);
    z_l = ld_t(a.gate, b * a.gate.stride[0] + h * a.gate.stride[1] + p * a.gate.stride[2]);
    if (kScatter) {
      const int64_t o = h * a.mimo_x.stride[0] + lrank * a.mimo_x.stride[1] + p * a.mimo_x.stride[2];
      const float mx = rnd<T>(ld_t(a.mimo_x, o));
      x_l = rnd<T>(x_l * mx);
      xp_l = rnd<T>(xp_l * mx);
      z_l = rnd<T>(z_l * rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + lrank * a.mimo_z.stride[1] +
                                              p * a.mimo_z.stride[2])));
      mo_l = ld_t(a.mimo_out, h * a.mimo_out.stride[0] + lrank * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
    }
  }
  float acc_l[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc_l[r] = 0.0f;
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    const int p = p0 + rr;
    if (p >= P) break;  // warp-uniform
    float xv[R], xpv[R];
    if (kScatter) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        xv[r] = __shfl_sync(0xffffffffu, x_l, r * G + rr);
        xpv[r] = __shfl_sync(0xffffffffu, xp_l, r * G + rr);
      }
    } else {
      const float x = __shfl_sync(0xffffffffu, x_l, rr), xp = __shfl_sync(0xffffffffu, xp_l, rr);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (R > 1) {
          const float mx = rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2]));
          xv[r] = rnd<T>(x * mx);
          xpv[r] = rnd<T>(xp * mx);
        } else {
          xv[r] = x;
          xpv[r] = xp;
        }
      }
    }
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int n = 4 * lane + 128 * v;
      if (n < N) {
        float4 po = make_float4(0.f, 0.f, 0.f, 0.f), co = po;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 kp4 = kpv[r][v].get(), k4 = kv[r][v].get();
          po.x += xpv[r] * kp4.x; po.y += xpv[r] * kp4.y;
          po.z += xpv[r] * kp4.z; po.w += xpv[r] * kp4.w;
          co.x += xv[r] * k4.x; co.y += xv[r] * k4.y;
          co.z += xv[r] * k4.z; co.w += xv[r] * k4.w;
        }
        const float4 o = sv[rr][v];
        float4 ns;
        ns.x = sc.x * o.x + sc.y * po.x + sc.z * co.x;
        ns.y = sc.x * o.y + sc.y * po.y + sc.z * co.y;
        ns.z = sc.x * o.z + sc.y * po.z + sc.z * co.z;
        ns.w = sc.x * o.w + sc.y * po.w + sc.z * co.w;
        store_state4(so + p * a.out_state.stride[2] + n, ns);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 q4 = qv[r][v].get();
          acc[r] += rnd<T>(ns.x) * q4.x + rnd<T>(ns.y) * q4.y + rnd<T>(ns.z) * q4.z + rnd<T>(ns.w) * q4.w;
        }
      }
    }
    if (kScatter) {
      // Reduce-scatter: each exchange halves the ranks a lane carries (lanes with bit `off` keep the
      // upper half), then the lanes of a rank group finish the sum; rank r of this row ends in every
      // lane of group r.
#pragma unroll
      for (int cnt = R, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < cnt / 2; ++i) {
          const float send = up ? acc[i] : acc[i + cnt / 2];
          const float keep = up ? acc[i + cnt / 2] : acc[i];
          acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
      if (lrow == rr) acc_l[0] = acc[0];
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        acc[r] = warp_sum(acc[r]);
        if (lane == rr) acc_l[r] = acc[r];  // lane rr finishes row rr below
      }
    }
  }
  // Row epilogues: y = sum_r mo_r silu(z mz_r) (S' q_r + D x mx_r).
  const bool row_ok = lrow < RPW && p0 + lrow < P;
  if (kScatter) {
    float o = row_ok ? (acc_l[0] + sc.w * x_l) * __fdividef(z_l, 1.0f + __expf(-z_l)) * mo_l : 0.0f;
#pragma unroll
    for (int off = G; off < 32; off <<= 1) o += __shfl_xor_sync(0xffffffffu, o, off);
    if (row_ok && lrank == 0)
      static_cast<T*>(a.y.data)[b * a.y.stride[0] + h * a.y.stride[1] + (p0 + lrow) * a.y.stride[2]] = from_f<T>(o);
  } else if (row_ok) {
    const int p = p0 + lane;
    float y = 0.0f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float xr = x_l, zr = z_l;
      if (R > 1) {
        xr = rnd<T>(x_l * rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2])));
        zr = rnd<T>(z_l * rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] + p * a.mimo_z.stride[2])));
      }
      float o = (acc_l[r] + sc.w * xr) * __fdividef(zr, 1.0f + __expf(-zr));
      if (R > 1) o *= ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
      y += o;
    }
    static_cast<T*>(a.y.data)[b * a.y.stride[0] + h * a.y.stride[1] + p * a.y.stride[2]] = from_f<T>(y);
  }
}

// mma.sync m16n8k16 (A row-major, B column-major, 16-bit inputs, FP32 accumulate): d += a b.
template <typename T> __device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                               uint32_t b1);
template <> __device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                                    uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T> __device__ __forceinline__ uint32_t pack_t2(float lo, float hi) {
  T e[2] = {from_f<T>(lo), from_f<T>(hi)};
  return *reinterpret_cast<const uint32_t*>(e);
}

// Stream pass for ranks 2, 4 and 8 (N = 128, P = 64, 16-bit activations) with the rank-structured
// products on the tensor cores. One CTA per (batch, head); warp w owns state rows 16 w .. 16 w + 15,
// held in the m16n8 accumulator layout (lane = 4 g + t: rows g and g + 8, columns 2t, 2t + 1 of
// every 8-column tile). Per 16-column block:
//   U1 = XP KP, U2 = X K       (one m16n8k16 MMA each per 8-column tile; A = the rank values
//                               xp_r[p], x_r[p] with the ranks padded to 16, B = the previous /
//                               current k_r[n] from shared memory)
//   S' = alpha S + beta U1 + gamma U2     (FP32 on the CUDA cores; streamed store)
//   Y += bf16(S') Q            (the two S' tiles are the A operand of one MMA, B = q_r[n])
// The rank values and k are 16-bit values (rounded where the reference rounds them), so every
// product is exact and only the FP32 summation order differs from step_stream_kernel. All of the
// warp's state loads are issued before it waits for the prep pass.
template <typename T, int R>
__global__ void __launch_bounds__(kStepThreads) step_stream_mma_kernel(const m3_step_args a) {
  constexpr int N = 128, KR = 8, LQ = N + 8;
  static_assert(R >= 2 && R <= KR, "ranks 2 .. 8");
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int pr0 = 16 * warp + g, pr1 = pr0 + 8;  // this lane's two state rows
  __shared__ __align__(16) uint16_t kT[N][KR], kpT[N][KR];  // k_r[n], previous k_r[n], transposed
  __shared__ __align__(16) uint16_t qs[KR][LQ];              // q_r[n]
  const float* st = static_cast<const float*>(a.state.data) + b * a.state.stride[0] + h * a.state.stride[1];
  float* so = static_cast<float*>(a.out_state.data) + b * a.out_state.stride[0] + h * a.out_state.stride[1];
  const int64_t ss = a.state.stride[2], os = a.out_state.stride[2];
  // state fragments of all 8 column blocks: [block][tile c * 2 + row half]
  float2 sv[8][4];
#pragma unroll
  for (int nb = 0; nb < 8; ++nb)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int n = 16 * nb + 8 * c + 2 * t;
      sv[nb][2 * c] = __ldcs(reinterpret_cast<const float2*>(st + pr0 * ss + n));
      sv[nb][2 * c + 1] = __ldcs(reinterpret_cast<const float2*>(st + pr1 * ss + n));
    }
  // per-row inputs of rows pr0 / pr1 (independent of the prep pass)
  const int64_t vb = b * a.value.stride[0] + h * a.value.stride[1];
  const int64_t pb = b * a.prev_value.stride[0] + h * a.prev_value.stride[1];
  const int64_t zb = b * a.gate.stride[0] + h * a.gate.stride[1];
  float x[2], xp[2], z[2], mx[2][2], mz[2][2], mo[2][2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int p = hr ? pr1 : pr0;
    x[hr] = ld_t(a.value, vb + p * a.value.stride[2]);
    xp[hr] = ld_t(a.prev_value, pb + p * a.prev_value.stride[2]);
    z[hr] = ld_t(a.gate, zb + p * a.gate.stride[2]);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int r = 2 * t + e;
      mx[hr][e] = mz[hr][e] = mo[hr][e] = 0.0f;
      if (r < R) {
        mx[hr][e] = rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2]));
        mz[hr][e] = rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] + p * a.mimo_z.stride[2]));
        mo[hr][e] = ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
      }
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // q, k (workspace, activation type) and the previous k into shared memory; ranks >= R are zero
  const float* ws = static_cast<const float*>(a.workspace.data) + ((int64_t)b * a.heads + h) * (2 * R * N + 4);
  const uint16_t* wsq = reinterpret_cast<const uint16_t*>(ws);
  const m3_tensor& pk = a.prev_k;
  const int64_t kb = b * pk.stride[0] + h * pk.stride[1];
  for (int i = tid; i < KR * N; i += kStepThreads) {
    const int r = i / N, n = i % N;
    uint16_t qv = 0, kv = 0, kpv = 0;
    if (r < R) {
      qv = wsq[r * N + n];
      kv = wsq[R * N + r * N + n];
      const T e = from_f<T>(ld_t(pk, kb + r * pk.stride[2] + n * pk.stride[3]));
      kpv = *reinterpret_cast<const uint16_t*>(&e);
    }
    qs[r][n] = qv;
    kT[n][r] = kv;
    kpT[n][r] = kpv;
  }
  const float4 sc = *reinterpret_cast<const float4*>(ws + 2 * R * N);  // alpha, beta, gamma, D
  // A fragments of the rank values: rows g / g + 8, rank columns 2t, 2t + 1 (upper 8 columns zero)
  float xr[2][2], zr[2][2];
  uint32_t ax[4] = {0u, 0u, 0u, 0u}, axp[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float xv[2], xpv[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      xv[e] = rnd<T>(x[hr] * mx[hr][e]);
      xpv[e] = rnd<T>(xp[hr] * mx[hr][e]);
      xr[hr][e] = xv[e];
      zr[hr][e] = rnd<T>(z[hr] * mz[hr][e]);
    }
    ax[hr] = pack_t2<T>(xv[0], xv[1]);
    axp[hr] = pack_t2<T>(xpv[0], xpv[1]);
  }
  __syncthreads();
  float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) {
    float ns[2][4];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int nc = 16 * nb + 8 * c + g;  // B column of this lane (ranks 2t, 2t + 1)
      const uint32_t bk = *reinterpret_cast<const uint32_t*>(&kT[nc][2 * t]);
      const uint32_t bkp = *reinterpret_cast<const uint32_t*>(&kpT[nc][2 * t]);
      float u1[4] = {0.f, 0.f, 0.f, 0.f}, u2[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816<T>(u1, axp, bkp, 0u);
      mma16816<T>(u2, ax, bk, 0u);
      const float2 s0 = sv[nb][2 * c], s1 = sv[nb][2 * c + 1];
      ns[c][0] = sc.x * s0.x + sc.y * u1[0] + sc.z * u2[0];
      ns[c][1] = sc.x * s0.y + sc.y * u1[1] + sc.z * u2[1];
      ns[c][2] = sc.x * s1.x + sc.y * u1[2] + sc.z * u2[2];
      ns[c][3] = sc.x * s1.y + sc.y * u1[3] + sc.z * u2[3];
      const int n = 16 * nb + 8 * c + 2 * t;
      __stcs(reinterpret_cast<float2*>(so + pr0 * os + n), make_float2(ns[c][0], ns[c][1]));
      __stcs(reinterpret_cast<float2*>(so + pr1 * os + n), make_float2(ns[c][2], ns[c][3]));
    }
    // Y += bf16(S') Q over these 16 columns: A = the two S' tiles, B = q_g[n] (rank g)
    const uint32_t a2[4] = {pack_t2<T>(ns[0][0], ns[0][1]), pack_t2<T>(ns[0][2], ns[0][3]),
                            pack_t2<T>(ns[1][0], ns[1][1]), pack_t2<T>(ns[1][2], ns[1][3])};
    const uint32_t bq0 = *reinterpret_cast<const uint32_t*>(&qs[g][16 * nb + 2 * t]);
    const uint32_t bq1 = *reinterpret_cast<const uint32_t*>(&qs[g][16 * nb + 8 + 2 * t]);
    mma16816<T>(y, a2, bq0, bq1);
  }
  // y fragment: (row g, ranks 2t, 2t + 1), (row g + 8, ranks 2t, 2t + 1);
  // out_p = sum_r mo_r silu(z mz_r) (S' q_r + D x mx_r), ranks summed across the four lanes t
  float o[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float acc = 0.0f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float zz = zr[hr][e];
      acc += (y[2 * hr + e] + sc.w * xr[hr][e]) * __fdividef(zz, 1.0f + __expf(-zz)) * mo[hr][e];
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    o[hr] = acc;
  }
  if (t == 0) {
    T* yp = static_cast<T*>(a.y.data) + b * a.y.stride[0] + h * a.y.stride[1];
    yp[pr0 * a.y.stride[2]] = from_f<T>(o[0]);
    yp[pr1 * a.y.stride[2]] = from_f<T>(o[1]);
  }
}

// Name of the step kernel variant the last launch_step on this host thread chose.
thread_local const char* g_last_step_kernel = "none";

template <typename T, int R, int NV, int RPW>
static cudaError_t launch_step_two_pass(const m3_step_args& a, cudaStream_t stream) {
  const int64_t pairs = (int64_t)a.batch * a.heads;
  const int per_cta = kStepThreads / 32;
  const unsigned grid = (unsigned)((pairs + per_cta - 1) / per_cta);
  // Rank 1 keeps the per-pair kernel: its 8 units would leave 24 lanes of each warp idle.
  if (R > 1 && sizeof(T) == 2 && a.d_state == 128 && rows16(a.q) && rows16(a.k) && rows16(a.out_k)) {
    g_last_step_kernel = "two_pass_vec";
    step_prep_vec_kernel<T, R><<<grid, kStepThreads, 0, stream>>>(a);
  } else if (a.d_state == 128) {
    g_last_step_kernel = "two_pass";
    step_prep_kernel<T, R, 128><<<grid, kStepThreads, 0, stream>>>(a);
  } else {
    g_last_step_kernel = "two_pass";
    step_prep_kernel<T, R, 0><<<grid, kStepThreads, 0, stream>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int rows = RPW * (kStepThreads / 32);
  const m3_tensor& pk = a.prev_k;
  const int vec_prev_k = sizeof(T) == 2 && pk.stride[3] == 1 && (reinterpret_cast<uintptr_t>(pk.data) & 7u) == 0 &&
                         pk.stride[0] % 4 == 0 && pk.stride[1] % 4 == 0 && pk.stride[2] % 4 == 0;
  // Programmatic dependent launch: the stream pass starts while the prep pass runs and waits for it
  // (griddepcontrol.wait) only after issuing its state loads.
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  if constexpr (R > 1 && sizeof(T) == 2) {
    if (a.d_state == 128 && a.head_dim == 64) {
      g_last_step_kernel = "two_pass_mma";
      cudaLaunchConfig_t mc = {};
      mc.gridDim = dim3(a.heads, a.batch);
      mc.blockDim = dim3(kStepThreads);
      mc.stream = stream;
      mc.attrs = pdl;
      mc.numAttrs = 1;
      return cudaLaunchKernelEx(&mc, step_stream_mma_kernel<T, R>, a);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.head_dim + rows - 1) / rows, a.heads, a.batch);
  cfg.blockDim = dim3(kStepThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_stream_kernel<T, R, NV, RPW>, a, vec_prev_k);
}

bool step_vec_ok(const m3_step_args& a) {
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const m3_tensor& s = a.state;
  const m3_tensor& o = a.out_state;
  return a.d_state % 4 == 0 && a.d_state <= 256 && s.stride[3] == 1 && o.stride[3] == 1 && al16(s.data) &&
         al16(o.data) && s.stride[0] % 4 == 0 && s.stride[1] % 4 == 0 && s.stride[2] % 4 == 0 &&
         o.stride[0] % 4 == 0 && o.stride[1] % 4 == 0 && o.stride[2] % 4 == 0;
}

template <typename T, int R>
static cudaError_t launch_step_r(const m3_step_args& a, cudaStream_t stream) {
  const int N = a.d_state, P = a.head_dim;
  // Fewer (batch, head) pairs than two per SM: one launch (the single-pass kernel, each CTA repeating
  // its head's prologue) is shorter than the prep + stream pair, whose cost there is launch latency.
  const bool few = (long long)a.batch * a.heads < 2 * 148;
  if (a.workspace.data != nullptr && !few) {  // set exactly when step_vec_ok (m3_step_workspace_bytes)
    // kStepBigRows rows per warp once there are enough (batch, head) pairs to fill
    // the GPU several times; otherwise 2 rows per warp so that even batch 1 spreads over all SMs.
    const bool big = (long long)a.batch * a.heads >= 4 * 148;
    if (N <= 128)
      return big ? launch_step_two_pass<T, R, 1, kStepBigRows>(a, stream) : launch_step_two_pass<T, R, 1, 2>(a, stream);
    return big ? launch_step_two_pass<T, R, 2, 8>(a, stream) : launch_step_two_pass<T, R, 2, 2>(a, stream);
  }
  // Split rows across CTAs until the grid covers every SM a few times.
  int rows = P;
  const long long pairs = (long long)a.batch * a.heads;
  while (rows > 4 && pairs * ((P + rows - 1) / rows) < 4 * 148) rows >>= 1;
  dim3 grid((P + rows - 1) / rows, a.heads, a.batch);
  g_last_step_kernel = "single";
  const size_t smem = (128 + 3 * (size_t)R * N + 2 * R) * sizeof(float);
  auto go = [&](auto kern) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a, rows);
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

int64_t step_workspace_bytes(const m3_step_args& a) {
  if (!step_vec_ok(a)) return 0;
  return (int64_t)a.batch * a.heads * (2 * a.rank * a.d_state + 4) * (int64_t)sizeof(float);
}

const char* last_step_kernel() { return g_last_step_kernel; }

cudaError_t launch_step(const m3_step_args& a, cudaStream_t stream) {
  switch (a.value.dtype) {
    case M3_F32: return launch_step_t<float>(a, stream);
    case M3_F16: return launch_step_t<__half>(a, stream);
    default: return launch_step_t<__nv_bfloat16>(a, stream);
  }
}

}  // namespace m3
