// Chunked Mamba-3 SSD forward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Shapes served: bf16/fp16 activations, d_state N = 128, head_dim P = 64, any rank R in
// {1, 2, 4, 8}, up to 32 rotation angles. One CTA (256 threads) owns one (batch, head) pair and
// walks the sequence in tiles of 128 flattened (token, rank) rows (128 / R tokens), keeping the
// FP32 state S^T [N=128, P=64] resident in tensor memory for the whole sequence.
//
// Per tile (mamba3/ops.py:716-816 math; mamba3/_triton.py:74-413 is the reference's fused form):
//   stage   Q  = rot(norm(C) + C_bias)            [128 rows, 128]  bf16, K-major   (smem)
//           K  = rot(norm(B) + B_bias) * scale    [128 rows, 128]  bf16            (smem)
//           V  = x * mimo_x                       [128 rows, 64]   bf16            (smem)
//           V2 = V * e^{cum_last - cum}           [128 rows, 64]   bf16            (smem)
//           St = bf16(S^T) (state before tile)    [128 n, 64 p]    bf16            (smem)
//           TMEM S^T <- e^{cum_last} S^T
//   MMA 1   scores = Q K^T          -> TMEM [128 x 128] f32
//   MMA 2   Y_inter = Q St          -> TMEM [128 x 64]  f32    (B operand MN-major)
//   MMA 3   S^T += K^T V2           -> TMEM [128 x 64]  f32    (A and B operands MN-major)
//   W       = scores o decay (exp of cum differences below the diagonal, gamma/scale on same-token
//             pairs, 0 above), rounded to bf16 -> smem, K-major
//   MMA 4   Y_intra = W V           -> TMEM [128 x 64]  f32
//   epilogue y = e^{cum} Y_inter + Y_intra + D v, SiLU(z mz) gate, MIMO rank sum -> global
//
// All operand tiles use the 128-byte swizzled canonical layout: a tile of `rows` x `cols`
// 16-bit elements is stored as cols/64 column blocks of rows x 128 B; inside a block, row r,
// 16-byte chunk c lives at r*128 + ((c ^ (r & 7)) * 16). The same bytes serve as a K-major
// operand ([MN rows][K cols]) or as an MN-major one ([K rows][MN cols]).
//
// Synchronisation: one mbarrier tracks tcgen05.commit of each MMA group; every wait on it is
// bounded by %globaltimer (2 s) and sets the library's device error word instead of hanging.
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

namespace umma {

constexpr int kRows = 128;      // flattened (token, rank) rows per tile = MMA M
constexpr int kN = 128;         // d_state
constexpr int kP = 64;          // head_dim
constexpr int kThreads = 256;
constexpr int kMaxAngles = 32;

// Shared-memory map (bytes from the 1024-aligned base).
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kRows * kN * 2;    // 32 KB each
constexpr uint32_t kOffW = kOffK + kRows * kN * 2;
constexpr uint32_t kOffV = kOffW + kRows * kRows * 2;
constexpr uint32_t kOffV2 = kOffV + kRows * kP * 2;  // 16 KB each
constexpr uint32_t kOffST = kOffV2 + kRows * kP * 2;
constexpr uint32_t kOffF = kOffST + kN * kP * 2;      // float region
// float region (in floats)
constexpr int kFScal = 0;                      // 7 * 128 + 8 (cum, ecum, edec, scale, diag, dt, cumL2) + wsum
constexpr int kFPh = kFScal + 7 * 128 + 8;     // phase [128 tokens][33]
constexpr int kFSeg = kFPh + 128 * 33;         // 768
constexpr int kFCarry = kFSeg + 768;           // 2 * 128
constexpr int kFEnd = kFCarry + 256;
constexpr uint32_t kOffBar = kOffF + kFEnd * 4;        // mbarrier (8 B) + tmem slot (4 B) + abort flag
constexpr uint32_t kSmemBytes = kOffBar + 64 + 1024;   // + alignment slack

// TMEM column map (fp32 accumulators; lane = tile row / state row n).
constexpr uint32_t kColScores = 0;    // 128 columns
constexpr uint32_t kColIntra = 128;   // 64
constexpr uint32_t kColInter = 192;   // 64
constexpr uint32_t kColState = 256;   // 64
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of element (row, col) of a swizzled tile with `rows` rows (16-bit elements).
__device__ __forceinline__ uint32_t swz(int row, int col, int rows) {
  return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}

// Shared-memory matrix descriptor: SWIZZLE_128B, sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16 with FP32 accumulation.
__host__ __device__ constexpr uint32_t idesc(int m, int n, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for mbarrier phase `parity`; false (and the device error word set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t start = global_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 255u && global_ns() - start > 2000000000ull) {
      atomicExch(&g_device_error, kErrMbarTimeout);
      return false;
    }
  }
}

#define M3_TMEM_LD32(taddr, r)                                                                               \
  asm volatile(                                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"  \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),      \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),           \
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),           \
        "=r"(r[30]), "=r"(r[31])                                                                             \
      : "r"(taddr))

#define M3_TMEM_ST32(taddr, r)                                                                                \
  asm volatile(                                                                                               \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16," \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                      \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),       \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),           \
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),          \
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <typename T> __device__ __forceinline__ uint16_t bits16(float x) {
  T v = from_f<T>(x);
  return *reinterpret_cast<uint16_t*>(&v);
}
template <typename T> __device__ __forceinline__ float from_bits16(uint16_t b) {
  T v = *reinterpret_cast<T*>(&b);
  return to_f(v);
}

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 1) scan_umma_kernel(const m3_scan_args a) {
  constexpr int TOK = kRows / R;
  constexpr bool kBf16 = DType<T>::id == M3_BF16;
  const int h = blockIdx.x, b = blockIdx.y;
  const int S = a.num_angles, L = a.length;
  const int g = h / (a.heads / a.groups);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, half = warp >> 2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* fsm = reinterpret_cast<float*>(smem + kOffF);
  float* scal = fsm + kFScal;
  TileScalars ts{scal, scal + 128, scal + 256, scal + 384, scal + 512, scal + 640, scal + 7 * 128};
  float* cum_l2 = scal + 768;  // cum * log2(e), 128 floats (overlaps nothing: scal has 7*128+8)
  float* sPh = fsm + kFPh;
  float* seg = fsm + kFSeg;
  float* carry_off = fsm + kFCarry;
  float* carry_loc = carry_off + 128;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + kOffBar + 16);
  const uint32_t bar_addr = smem_u32(bar);
  const uint32_t sbase = smem_u32(smem);
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;

  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const T* vp = static_cast<const T*>(a.value.data);
  const T* zp = static_cast<const T*>(a.gate.data);
  T* yp = static_cast<T*>(a.y.data);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);

  // ---- set-up: TMEM allocation (warp 0), mbarrier, phase carry ----
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_addr));
    asm volatile("fence.mbarrier_init.release.cluster;");
    *abort_flag = 0;
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
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;

  // ---- initial state into TMEM: S^T[n][p] = S0[p][n] + c0 * sum_r v_r[p] k_r[n] ----
  {
    float c0 = 0.0f;
    if (a.initial_k.data) {
      float dt0, adt0;
      const int t_first = scan_token(a, 0);
      load_dt_adt(a, b, t_first, h, dt0, adt0);
      c0 = dt0 * (1.0f - sigmoidf_(load_trap(a, b, t_first, h)));
    }
    const int n = quad * 32 + lane;
    uint32_t r[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int p = half * 32 + j;
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
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          float vr = v;
          if (R > 1)
            vr = rnd<T>(v * rnd<T>(ld_t(a.mimo_x, h * a.mimo_x.stride[0] + rr * a.mimo_x.stride[1] +
                                                    p * a.mimo_x.stride[2])));
          acc += vr * ld_t(ik, b * ik.stride[0] + h * ik.stride[1] + rr * ik.stride[2] + n * ik.stride[3]);
        }
        s += c0 * acc;
      }
      r[j] = __float_as_uint(s);
    }
    M3_TMEM_ST32(tmem + lane_base + kColState + half * 32, r);
    tmem_wait_st();
  }

  const uint32_t id_scores = idesc(128, 128, kBf16, false, false);
  const uint32_t id_inter = idesc(128, 64, kBf16, false, true);
  const uint32_t id_state = idesc(128, 64, kBf16, true, true);
  const uint32_t id_intra = idesc(128, 64, kBf16, false, true);
  uint32_t phase_bit = 0;

  for (int t0 = 0; t0 < L; t0 += TOK) {
    const int nt = min(TOK, L - t0);
    float last_decay;
    tile_scalars(a, b, h, t0, nt, TOK, ts, last_decay);
    if (tid < TOK) cum_l2[tid] = ts.cum[tid] * kLog2e;
    if (has_phase) tile_phase(a, b, h, t0, nt, TOK, ts.dt, sPh, 33, carry_off, carry_loc, seg);
    else __syncthreads();

    // ---- stage Q, K (16 rows per warp) ----
    for (int row = warp * 16; row < warp * 16 + 16; ++row) {
      const int j = row / R, r = row % R;
      float qv[4], kv[4];
      const bool valid = j < nt;
      const int t = valid ? scan_token(a, t0 + j) : 0;
      if (valid) {
        const int64_t qb = b * a.q.stride[0] + (int64_t)t * a.q.stride[1] + g * a.q.stride[2] + r * a.q.stride[3];
        const int64_t kb = b * a.k.stride[0] + (int64_t)t * a.k.stride[1] + g * a.k.stride[2] + r * a.k.stride[3];
        float sq = 0.0f, sk = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = lane + 32 * e;
          qv[e] = to_f(qp[qb + n * a.q.stride[4]]);
          kv[e] = to_f(kp[kb + n * a.k.stride[4]]);
          sq += qv[e] * qv[e];
          sk += kv[e] * kv[e];
        }
        if (a.q_norm_w.data) {
          const float rq = rsqrtf(warp_sum(sq) * (1.0f / kN) + a.norm_eps);
          const float rk = rsqrtf(warp_sum(sk) * (1.0f / kN) + a.norm_eps);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = lane + 32 * e;
            qv[e] = rnd<T>(qv[e] * rq * rnd<T>(ld_t(a.q_norm_w, n * a.q_norm_w.stride[0])));
            kv[e] = rnd<T>(kv[e] * rk * rnd<T>(ld_t(a.k_norm_w, n * a.k_norm_w.stride[0])));
          }
        }
        if (a.q_bias.data) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = lane + 32 * e;
            qv[e] = rnd<T>(qv[e] + rnd<T>(ld_t(a.q_bias, h * a.q_bias.stride[0] + r * a.q_bias.stride[1] +
                                                           n * a.q_bias.stride[2])));
            kv[e] = rnd<T>(kv[e] + rnd<T>(ld_t(a.k_bias, h * a.k_bias.stride[0] + r * a.k_bias.stride[1] +
                                                           n * a.k_bias.stride[2])));
          }
        }
        if (has_phase) {
          const float* ph = sPh + j * 33;
          if (a.mimo_rotation) {
            // pairs (m, m + 2S) with 2S == 64: slot e = 0 (n = lane) with slot e = 2 (n = lane + 64).
            if (lane < S) {
              float sn, cs;
              __sincosf(ph[lane], &sn, &cs);
              cs = rnd<T>(cs);
              sn = rnd<T>(sn);
              const float q0 = qv[0], q1 = qv[2], k0 = kv[0], k1 = kv[2];
              qv[0] = rnd<T>(rnd<T>(q0 * cs) - rnd<T>(q1 * sn));
              qv[2] = rnd<T>(rnd<T>(q0 * sn) + rnd<T>(q1 * cs));
              kv[0] = rnd<T>(rnd<T>(k0 * cs) - rnd<T>(k1 * sn));
              kv[2] = rnd<T>(rnd<T>(k0 * sn) + rnd<T>(k1 * cs));
            }
          } else {
            // adjacent pairs (2m, 2m+1): partner is the neighbouring lane in the same slot.
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float qo = __shfl_xor_sync(0xffffffffu, qv[e], 1);
              const float ko = __shfl_xor_sync(0xffffffffu, kv[e], 1);
              const int n = lane + 32 * e;
              const int m = n >> 1;
              if (m < S) {
                float sn, cs;
                __sincosf(ph[m], &sn, &cs);
                cs = rnd<T>(cs);
                sn = rnd<T>(sn);
                if ((n & 1) == 0) {
                  qv[e] = rnd<T>(rnd<T>(qv[e] * cs) - rnd<T>(qo * sn));
                  kv[e] = rnd<T>(rnd<T>(kv[e] * cs) - rnd<T>(ko * sn));
                } else {
                  qv[e] = rnd<T>(rnd<T>(qo * sn) + rnd<T>(qv[e] * cs));
                  kv[e] = rnd<T>(rnd<T>(ko * sn) + rnd<T>(kv[e] * cs));
                }
              }
            }
          }
        }
        if (a.final_k.data && t0 + j == L - 1) {
          const m3_tensor& fk = a.final_k;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            static_cast<T*>(fk.data)[b * fk.stride[0] + h * fk.stride[1] + r * fk.stride[2] +
                                     (lane + 32 * e) * fk.stride[3]] = from_f<T>(kv[e]);
        }
        const float sc = ts.scale[j];
#pragma unroll
        for (int e = 0; e < 4; ++e) kv[e] = kv[e] * sc;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) { qv[e] = 0.0f; kv[e] = 0.0f; }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = lane + 32 * e;
        *reinterpret_cast<uint16_t*>(smem + kOffQ + swz(row, n, kRows)) = bits16<T>(qv[e]);
        *reinterpret_cast<uint16_t*>(smem + kOffK + swz(row, n, kRows)) = bits16<T>(kv[e]);
      }
      // V and V2 rows (p = 2 lane, 2 lane + 1)
      float v0 = 0.0f, v1 = 0.0f;
      if (valid) {
        const int64_t vb = b * a.value.stride[0] + (int64_t)t * a.value.stride[1] + h * a.value.stride[2];
        v0 = to_f(vp[vb + (2 * lane) * a.value.stride[3]]);
        v1 = to_f(vp[vb + (2 * lane + 1) * a.value.stride[3]]);
        if (R > 1) {
          const int64_t mb = h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1];
          v0 = rnd<T>(v0 * rnd<T>(ld_t(a.mimo_x, mb + (2 * lane) * a.mimo_x.stride[2])));
          v1 = rnd<T>(v1 * rnd<T>(ld_t(a.mimo_x, mb + (2 * lane + 1) * a.mimo_x.stride[2])));
        }
      }
      const float ed = valid ? ts.edec[j] : 0.0f;
      const uint32_t pv = (uint32_t)bits16<T>(v0) | ((uint32_t)bits16<T>(v1) << 16);
      const uint32_t pv2 = (uint32_t)bits16<T>(v0 * ed) | ((uint32_t)bits16<T>(v1 * ed) << 16);
      *reinterpret_cast<uint32_t*>(smem + kOffV + swz(row, 2 * lane, kRows)) = pv;
      *reinterpret_cast<uint32_t*>(smem + kOffV2 + swz(row, 2 * lane, kRows)) = pv2;
    }

    // ---- state: TMEM S^T -> bf16 St tile (state before this tile), then S^T *= e^{cum_last} ----
    {
      uint32_t r[32];
      fence_after();
      M3_TMEM_LD32(tmem + lane_base + kColState + half * 32, r);
      tmem_wait_ld();
      const int n = quad * 32 + lane;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float x0 = __uint_as_float(r[c * 8 + 2 * i]);
          const float x1 = __uint_as_float(r[c * 8 + 2 * i + 1]);
          w[i] = (uint32_t)bits16<T>(x0) | ((uint32_t)bits16<T>(x1) << 16);
        }
        *reinterpret_cast<uint4*>(smem + kOffST + swz(n, half * 32 + c * 8, kN)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * last_decay);
      M3_TMEM_ST32(tmem + lane_base + kColState + half * 32, r);
      tmem_wait_st();
    }
    fence_async_smem();
    fence_before();
    __syncthreads();

    // ---- MMA group 1: scores, inter, state update ----
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColScores, sdesc(sbase + kOffQ + koff, 16, 1024), sdesc(sbase + kOffK + koff, 16, 1024),
                id_scores, kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColInter, sdesc(sbase + kOffQ + koff, 16, 1024),
                sdesc(sbase + kOffST + kk * 2048, kN * 128, 1024), id_inter, kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        mma_f16(tmem + kColState, sdesc(sbase + kOffK + kk * 2048, kRows * 128, 1024),
                sdesc(sbase + kOffV2 + kk * 2048, kRows * 128, 1024), id_state, 1);
      }
      mma_commit(bar_addr);
    }
    if (!mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    fence_after();

    // ---- W = scores o decay -> smem (bf16, K-major), 64 columns per thread ----
    {
      const int i = quad * 32 + lane;
      const int ti = i / R;
      const int col0 = half * 64;
      const bool all_masked = (col0 / R) > ((quad * 32 + 31) / R);  // warp-uniform
      if (all_masked) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + c * 8, kRows)) = make_uint4(0, 0, 0, 0);
      } else {
        const float ci = cum_l2[min(ti, TOK - 1)];
        const float di = ts.diag[min(ti, TOK - 1)];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r[32];
          M3_TMEM_LD32(tmem + lane_base + kColScores + col0 + hh * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float vals[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int jcol = col0 + hh * 32 + c * 8 + e * 2 + u;
                const int tj = jcol / R;
                const float s = __uint_as_float(r[c * 8 + e * 2 + u]);
                float wv = 0.0f;
                if (tj < ti) wv = s * ex2_approx(ci - cum_l2[tj]);
                else if (tj == ti) wv = s * di;
                vals[u] = wv;
              }
              w[e] = (uint32_t)bits16<T>(vals[0]) | ((uint32_t)bits16<T>(vals[1]) << 16);
            }
            *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + hh * 32 + c * 8, kRows)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();

    // ---- MMA group 2: intra = W V ----
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColIntra, sdesc(sbase + kOffW + koff, 16, 1024),
                sdesc(sbase + kOffV + kk * 2048, kRows * 128, 1024), id_intra, kk > 0);
      }
      mma_commit(bar_addr);
    }
    if (!mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    fence_after();

    // ---- epilogue: 32 output columns per thread ----
    {
      const int i = quad * 32 + lane;
      const int ti = i / R, r = i % R;
      uint32_t ra[32], ri[32];
      M3_TMEM_LD32(tmem + lane_base + kColIntra + half * 32, ra);
      M3_TMEM_LD32(tmem + lane_base + kColInter + half * 32, ri);
      tmem_wait_ld();
      const bool valid = ti < nt;
      const int t = valid ? scan_token(a, t0 + ti) : 0;
      const float ec = valid ? ts.ecum[ti] : 0.0f;
      float out[32];
      const int64_t zb = b * a.gate.stride[0] + (int64_t)t * a.gate.stride[1] + h * a.gate.stride[2];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 vv = *reinterpret_cast<const uint4*>(smem + kOffV + swz(i, half * 32 + c * 8, kRows));
        const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = c * 8 + e;
          const int p = half * 32 + j;
          const float v = from_bits16<T>((uint16_t)(vw[e >> 1] >> ((e & 1) * 16)));
          float y = ec * __uint_as_float(ri[j]) + __uint_as_float(ra[j]) + Dh * v;
          float z = valid ? to_f(zp[zb + p * a.gate.stride[3]]) : 0.0f;
          if (R > 1) {
            z = rnd<T>(z * rnd<T>(ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] +
                                                 p * a.mimo_z.stride[2])));
            y *= siluf_(z);
            y *= ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
          } else {
            y *= siluf_(z);
          }
          out[j] = y;
        }
      }
      if (R > 1) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
#pragma unroll
          for (int o = 1; o < R; o <<= 1) out[j] += __shfl_xor_sync(0xffffffffu, out[j], o);
        }
      }
      if (valid && r == 0) {
        const int64_t ob = b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2];
#pragma unroll
        for (int j = 0; j < 32; ++j) yp[ob + (half * 32 + j) * a.y.stride[3]] = from_f<T>(out[j]);
      }
    }
    if (t0 + TOK >= L && a.final_phase.data && has_phase && tid < S) {
      const m3_tensor& fp = a.final_phase;
      static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + tid * fp.stride[2]] = sPh[(nt - 1) * 33 + tid];
    }
    fence_before();
    __syncthreads();
    if (*abort_flag) break;
  }

  // ---- final state: S[p][n] from TMEM S^T ----
  fence_after();
  if (!*abort_flag) {
    uint32_t r[32];
    M3_TMEM_LD32(tmem + lane_base + kColState + half * 32, r);
    tmem_wait_ld();
    const int n = quad * 32 + lane;
    const m3_tensor& fs = a.final_state;
    float* fsp = static_cast<float*>(fs.data) + b * fs.stride[0] + h * fs.stride[1] + n * fs.stride[3];
#pragma unroll
    for (int j = 0; j < 32; ++j) fsp[(half * 32 + j) * fs.stride[2]] = __uint_as_float(r[j]);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T, int R>
static cudaError_t launch_r(const m3_scan_args& a, cudaStream_t stream) {
  auto kern = scan_umma_kernel<T, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<dim3(a.heads, a.batch), kThreads, kSmemBytes, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_t(const m3_scan_args& a, cudaStream_t stream) {
  switch (a.rank) {
    case 1: return launch_r<T, 1>(a, stream);
    case 2: return launch_r<T, 2>(a, stream);
    case 4: return launch_r<T, 4>(a, stream);
    default: return launch_r<T, 8>(a, stream);
  }
}

}  // namespace umma

bool scan_umma_supported(const m3_scan_args& a) {
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;
  return (a.value.dtype == M3_BF16 || a.value.dtype == M3_F16) && a.d_state == umma::kN &&
         a.head_dim == umma::kP && (a.rank == 1 || a.rank == 2 || a.rank == 4 || a.rank == 8) &&
         (!has_phase || (a.mimo_rotation ? a.num_angles == umma::kMaxAngles : a.num_angles <= umma::kMaxAngles));
}

cudaError_t launch_scan_umma(const m3_scan_args& a, cudaStream_t stream) {
  return a.value.dtype == M3_BF16 ? umma::launch_t<__nv_bfloat16>(a, stream) : umma::launch_t<__half>(a, stream);
}

}  // namespace m3
