// Chunked Mamba-3 SSD forward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Shapes served: bf16/fp16 activations, d_state N = 128, head_dim P = 64, any rank R in
// {1, 2, 4, 8}, up to 32 rotation angles. A pre-pass (token_prep_kernel) computes the per-token
// values every head shares — RMS factors of the q/k rows and pi*tanh(angle) — once into the
// caller's workspace. Then one CTA (512 threads) owns one (batch, head) pair and
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

// Optional per-section cycle counters of CTA (0, 0), thread 0 (probe builds only).
#ifdef M3_SECTION_TIMING
__device__ unsigned long long g_section_cycles[16];
#define M3_MARK(k)                                                                    \
  do {                                                                                \
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) {                     \
      const long long now_ = clock64();                                               \
      g_section_cycles[k] += (unsigned long long)(now_ - mark_prev_);                 \
      mark_prev_ = now_;                                                              \
    }                                                                                 \
  } while (0)
#else
#define M3_MARK(k) \
  do {             \
  } while (0)
#endif

constexpr int kRows = 128;      // flattened (token, rank) rows per tile = MMA M
constexpr int kN = 128;         // d_state
constexpr int kP = 64;          // head_dim
constexpr int kThreads = 512;   // 16 warps: warp w owns TMEM lane quadrant (w % 4), column part (w / 4)
constexpr int kMaxAngles = 32;
constexpr int kMaxRank = 8;

// Shared-memory map (bytes from the 1024-aligned base).
constexpr uint32_t kOffQ = 0;                          // Q' [128 rows][128]   32 KB
constexpr uint32_t kOffK = kOffQ + kRows * kN * 2;     // K' [128 rows][128]   32 KB
constexpr uint32_t kOffW = kOffK + kRows * kN * 2;     // W  [128][128]        32 KB (holds V2 while staging)
constexpr uint32_t kOffV = kOffW + kRows * kRows * 2;  // V  [128 rows][64]    16 KB
constexpr uint32_t kOffZ = kOffV + kRows * kP * 2;     // z  [128 tokens][64]  16 KB
constexpr uint32_t kOffST = kOffZ + kRows * kP * 2;    // St [128 n][64 p]     16 KB
constexpr uint32_t kOffF = kOffST + kN * kP * 2;       // float region
// float region (in floats)
constexpr int kFScal = 0;                          // per-token scalars, 11 x 128 + 16
constexpr int kFConst = kFScal + 11 * 128 + 16;    // per-CTA constants
constexpr int kCWq = 0, kCWk = 128, kCBq = 256, kCBk = kCBq + kMaxRank * kN, kCMx = kCBk + kMaxRank * kN,
              kCMz = kCMx + kMaxRank * kP, kCMo = kCMz + kMaxRank * kP, kCEnd = kCMo + kMaxRank * kP;
constexpr int kFPh = kFConst + kCEnd;              // (cos, sin) [128 tokens][32] float2
constexpr int kFSeg = kFPh + 128 * 32 * 2;         // 1024
constexpr int kFCarry = kFSeg + 1024;              // 2 * 128
constexpr int kFEnd = kFCarry + 256;
constexpr uint32_t kOffBar = kOffF + kFEnd * 4;         // mbarrier (8 B) + tmem slot (4 B) + abort flag
constexpr uint32_t kSmemBytes = kOffBar + 64 + 1024;    // + alignment slack

// TMEM column map (fp32 accumulators; lane = tile row, or state row n).
constexpr uint32_t kColScores = 0;    // 128 columns; the intra accumulator reuses columns 0..63
constexpr uint32_t kColIntra = 0;
constexpr uint32_t kColInter = 128;   // 64
constexpr uint32_t kColState = 192;   // 64
constexpr uint32_t kTmemCols = 256;

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

#define M3_TMEM_LD16(taddr, r)                                                                             \
  asm volatile(                                                                                            \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15},"  \
      " [%16];"                                                                                            \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),    \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]) \
      : "r"(taddr))

#define M3_TMEM_ST16(taddr, r)                                                                                \
  asm volatile(                                                                                               \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" \
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),    \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t w);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t w) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <typename T> __device__ __forceinline__ float lo16(uint32_t w) {
  uint16_t b = (uint16_t)(w & 0xFFFFu);
  return to_f(*reinterpret_cast<T*>(&b));
}
template <typename T> __device__ __forceinline__ float hi16(uint32_t w) {
  uint16_t b = (uint16_t)(w >> 16);
  return to_f(*reinterpret_cast<T*>(&b));
}

// 4 consecutive 16-bit elements at element index `idx` (stride 1) or with a generic stride.
template <typename T>
__device__ __forceinline__ uint2 load4(const T* base, int64_t idx, int64_t stride, bool vec) {
  if (vec) return *reinterpret_cast<const uint2*>(base + idx);
  const uint16_t* b = reinterpret_cast<const uint16_t*>(base);
  const uint32_t e0 = b[idx], e1 = b[idx + stride], e2 = b[idx + 2 * stride], e3 = b[idx + 3 * stride];
  return make_uint2(e0 | (e1 << 16), e2 | (e3 << 16));
}
template <typename T>
__device__ __forceinline__ uint32_t load2(const T* base, int64_t idx, int64_t stride, bool vec) {
  if (vec) return *reinterpret_cast<const uint32_t*>(base + idx);
  const uint16_t* b = reinterpret_cast<const uint16_t*>(base);
  return (uint32_t)b[idx] | ((uint32_t)b[idx + stride] << 16);
}

// Per-token pre-pass: ws[(b*L + t) * W + ...] with W = 2R + S holds the RMS factor of each q row
// (r), of each k row (R + r) and pi*tanh(angle) (2R + s). Token index in original order.
// One warp per token.
template <typename T>
__global__ void __launch_bounds__(256) token_prep_kernel(const m3_scan_args a, float* ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * 8 + warp;
  const int64_t total = (int64_t)a.batch * a.length;
  if (tok >= total) return;
  const int b = (int)(tok / a.length), t = (int)(tok % a.length);
  const int R = a.rank, S = a.num_angles, W = 2 * R + S;
  float* o = ws + tok * W;
  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const bool has_norm = a.q_norm_w.data != nullptr;
  for (int r = 0; r < R; ++r) {
    float rq = 1.0f, rk = 1.0f;
    if (has_norm) {
      // groups: the kernel reads group g = h / (H / G); every group's rows are normalised.
      float sq = 0.0f, sk = 0.0f;
      const int64_t qb = b * a.q.stride[0] + (int64_t)t * a.q.stride[1] + r * a.q.stride[3];
      const int64_t kb = b * a.k.stride[0] + (int64_t)t * a.k.stride[1] + r * a.k.stride[3];
      for (int n = lane; n < a.d_state; n += 32) {
        const float x = to_f(qp[qb + n * a.q.stride[4]]);
        const float y = to_f(kp[kb + n * a.k.stride[4]]);
        sq += x * x;
        sk += y * y;
      }
      rq = rsqrtf(warp_sum(sq) / a.d_state + a.norm_eps);
      rk = rsqrtf(warp_sum(sk) / a.d_state + a.norm_eps);
    }
    if (lane == 0) {
      o[r] = rq;
      o[R + r] = rk;
    }
  }
  if (a.angles.data) {
    for (int sidx = lane; sidx < S; sidx += 32)
      o[2 * R + sidx] = kPi * tanhf(ld_t(a.angles, b * a.angles.stride[0] + (int64_t)t * a.angles.stride[1] +
                                                 sidx * a.angles.stride[2]));
  }
}

// x - 2pi * trunc(x / 2pi): the remainder of fmod (exact for |x| < 2pi, a few ulp beyond).
__device__ __forceinline__ float fmod_2pi(float x) { return x - kTwoPi * truncf(x * (1.0f / kTwoPi)); }

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, 1) scan_umma_kernel(const m3_scan_args a, int vec_qk, int vec_vz,
                                                                 int vec_y) {
  constexpr int TOK = kRows / R;
  constexpr int kWarps = kThreads / 32;
  constexpr int kSL = TOK / kWarps > 0 ? TOK / kWarps : 1;   // phase tokens per warp segment
  constexpr int kSegs = TOK / kSL;                           // phase segments per tile (<= 16)
  constexpr int kRowsPerWarp = kRows / kWarps;               // staging rows per warp (8)
  constexpr bool kBf16 = DType<T>::id == M3_BF16;
  // Largest |cum - cmid| for which the decay can be split into per-row operand factors
  // e^{cum_i - cmid} (Q rows) and e^{cmid - cum_j} (K rows) without leaving the 16-bit range.
  constexpr float kLim = kBf16 ? 80.0f : 8.0f;
  const int h = blockIdx.x, b = blockIdx.y;
  const int S = a.num_angles, L = a.length;
  const int g = h / (a.heads / a.groups);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, part = warp >> 2;
  const int WS = 2 * R + S;  // workspace floats per token

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* fsm = reinterpret_cast<float*>(smem + kOffF);
  float* scal = fsm + kFScal;
  TileScalars ts{scal, scal + 128, scal + 256, scal + 384, scal + 512, scal + 640, scal + 7 * 128};
  float* cum_l2 = scal + 768;    // cum * log2(e)
  float* fq = scal + 1024;       // Q row factor
  float* fk = scal + 1152;       // K row factor (includes scale)
  float* mode = scal + 1280;     // [0] cmid, [1] cl, [2] factorized
  float* cst = fsm + kFConst;
  float2* scs = reinterpret_cast<float2*>(fsm + kFPh);  // (cos, sin) [TOK][32]
  float* seg = fsm + kFSeg;                             // [16][32] segment sums, then bases / offsets
  float* carry = fsm + kFCarry;                         // [0..31] block offset, [32..63] within-block sum
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + kOffBar + 16);
  const uint32_t bar_addr = smem_u32(bar);
  const uint32_t sbase = smem_u32(smem);
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;
  const bool has_ws = a.workspace.data != nullptr;
  const float* ws = static_cast<const float*>(a.workspace.data);

  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const T* vp = static_cast<const T*>(a.value.data);
  const T* zp = static_cast<const T*>(a.gate.data);
  T* yp = static_cast<T*>(a.y.data);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  const int64_t q_b = b * a.q.stride[0] + g * a.q.stride[2] + 4 * lane * a.q.stride[4];
  const int64_t k_b = b * a.k.stride[0] + g * a.k.stride[2] + 4 * lane * a.k.stride[4];
  const int64_t v_b = b * a.value.stride[0] + h * a.value.stride[2] + 2 * lane * a.value.stride[3];
  const int64_t z_b = b * a.gate.stride[0] + h * a.gate.stride[2] + 2 * lane * a.gate.stride[3];
  const int64_t ws_b = (int64_t)b * L * WS;

  // ---- set-up: TMEM allocation (warp 0), mbarrier, per-CTA constants, phase carry ----
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
  for (int i = tid; i < R * kN; i += kThreads) {
    const int r = i / kN, n = i % kN;
    float bq = 0.0f, bk = 0.0f;
    if (a.q_bias.data) {
      bq = ld_t(a.q_bias, h * a.q_bias.stride[0] + r * a.q_bias.stride[1] + n * a.q_bias.stride[2]);
      bk = ld_t(a.k_bias, h * a.k_bias.stride[0] + r * a.k_bias.stride[1] + n * a.k_bias.stride[2]);
    }
    cst[kCBq + i] = bq;
    cst[kCBk + i] = bk;
  }
  if (R > 1) {
    for (int i = tid; i < R * kP; i += kThreads) {
      const int r = i / kP, p = i % kP;
      cst[kCMx + i] = ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2]);
      cst[kCMz + i] = ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] + p * a.mimo_z.stride[2]);
      cst[kCMo + i] = ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
    }
  }
  if (tid < 32) {
    float off = 0.0f;
    if (a.initial_phase.data && tid < S) {
      const m3_tensor& t = a.initial_phase;
      off = ld_t(t, b * t.stride[0] + h * t.stride[1] + tid * t.stride[2]);
    }
    carry[tid] = off;
    carry[32 + tid] = 0.0f;
  }
  // Per-lane norm weights for the 4 state elements this lane stages.
  float wq[4], wk[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const bool nw = a.q_norm_w.data != nullptr;
    wq[e] = nw ? ld_t(a.q_norm_w, (4 * lane + e) * a.q_norm_w.stride[0]) : 1.0f;
    wk[e] = nw ? ld_t(a.k_norm_w, (4 * lane + e) * a.k_norm_w.stride[0]) : 1.0f;
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;

  // ---- initial state into TMEM: S^T[n][p] = S0[p][n] + c0 sum_r (v mx_r)[p] k_r[n] ----
  {
    float c0 = 0.0f;
    if (a.initial_k.data) {
      float dt0, adt0;
      const int t_first = scan_token(a, 0);
      load_dt_adt(a, b, t_first, h, dt0, adt0);
      c0 = dt0 * (1.0f - sigmoidf_(load_trap(a, b, t_first, h)));
    }
    const int n = quad * 32 + lane;
    uint32_t r16[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int p = part * 16 + j;
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
          const float vr = R > 1 ? v * cst[kCMx + rr * kP + p] : v;
          acc += vr * ld_t(ik, b * ik.stride[0] + h * ik.stride[1] + rr * ik.stride[2] + n * ik.stride[3]);
        }
        s += c0 * acc;
      }
      r16[j] = __float_as_uint(s);
    }
    M3_TMEM_ST16(tmem + lane_base + kColState + part * 16, r16);
    tmem_wait_st();
  }

  const uint32_t id_scores = idesc(128, 128, kBf16, false, false);
  const uint32_t id_nmn = idesc(128, 64, kBf16, false, true);   // K-major A, MN-major B, N = 64
  const uint32_t id_state = idesc(128, 64, kBf16, true, true);  // MN-major A and B
  uint32_t phase_bit = 0;
  float phi = 1.0f;  // TMEM holds S / phi
#ifdef M3_SECTION_TIMING
  long long mark_prev_ = clock64();
#endif

  for (int t0 = 0; t0 < L; t0 += TOK) {
    const int nt = min(TOK, L - t0);
    M3_MARK(0);

    // ---- issue this tile's row loads first (q, k, value, gate, norm factors) ----
    uint2 qraw[kRowsPerWarp], kraw[kRowsPerWarp];
    uint32_t vraw[kRowsPerWarp], zraw[kRowsPerWarp];
    float rqf[kRowsPerWarp], rkf[kRowsPerWarp];
#pragma unroll
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      const int row = warp * kRowsPerWarp + rr;
      const int j = row / R, r = row % R;
      qraw[rr] = kraw[rr] = make_uint2(0, 0);
      vraw[rr] = zraw[rr] = 0;
      rqf[rr] = rkf[rr] = 1.0f;
      if (j < nt) {
        const int t = scan_token(a, t0 + j);
        qraw[rr] = load4(qp, q_b + (int64_t)t * a.q.stride[1] + r * a.q.stride[3], a.q.stride[4], vec_qk);
        kraw[rr] = load4(kp, k_b + (int64_t)t * a.k.stride[1] + r * a.k.stride[3], a.k.stride[4], vec_qk);
        vraw[rr] = load2(vp, v_b + (int64_t)t * a.value.stride[1], a.value.stride[3], vec_vz);
        if (r == 0) zraw[rr] = load2(zp, z_b + (int64_t)t * a.gate.stride[1], a.gate.stride[3], vec_vz);
        if (has_ws) {
          rqf[rr] = ws[ws_b + (int64_t)t * WS + r];
          rkf[rr] = ws[ws_b + (int64_t)t * WS + R + r];
        }
      }
    }

    M3_MARK(1);
    float last_decay;
    tile_scalars(a, b, h, t0, nt, TOK, ts, last_decay);
    M3_MARK(2);
    // Decay factorisation for this tile (warp 0): cmid = cum of the middle token.
    if (warp == 0) {
      const float cmid = ts.cum[(nt - 1) >> 1];
      float dev = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = lane + 32 * k;
        if (j < nt) dev = fmaxf(dev, fabsf(ts.cum[j] - cmid));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dev = fmaxf(dev, __shfl_xor_sync(0xffffffffu, dev, o));
      const bool fact = dev <= kLim;
      const float ecm = expf(cmid);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = lane + 32 * k;
        if (j < TOK) {
          const float c = ts.cum[j];
          cum_l2[j] = c * kLog2e;
          if (j < nt) {
            fq[j] = fact ? __expf(c - cmid) : 1.0f;
            fk[j] = fact ? ts.scale[j] * __expf(cmid - c) : ts.scale[j];
            ts.ecum[j] = fact ? ecm : ts.ecum[j];
          } else {
            fq[j] = 0.0f;
            fk[j] = 0.0f;
          }
        }
      }
      if (lane == 0) {
        mode[0] = cmid;
        mode[1] = ts.cum[nt - 1];
        mode[2] = fact ? 1.0f : 0.0f;
      }
    }
    M3_MARK(3);
    // ---- phase -> (cos, sin) per (token, angle); warp w owns tokens [w*kSL, (w+1)*kSL) ----
    if (has_phase) {
      const int j0 = warp * kSL;
      float ph[kSL];
      if (warp < kSegs) {
        if (a.phase.data) {
#pragma unroll
          for (int u = 0; u < kSL; ++u) {
            const int j = j0 + u;
            ph[u] = 0.0f;
            if (j < nt && lane < S) {
              const int t = scan_token(a, t0 + j);
              ph[u] = ld_t(a.phase, b * a.phase.stride[0] + (int64_t)t * a.phase.stride[1] + h * a.phase.stride[2] +
                                        lane * a.phase.stride[3]);
            }
          }
        } else {
          float loc = 0.0f;
#pragma unroll
          for (int u = 0; u < kSL; ++u) {
            const int j = j0 + u;
            float inc = 0.0f;
            if (j < nt && lane < S) {
              const int t = scan_token(a, t0 + j);
              inc = fmod_2pi(ws[ws_b + (int64_t)t * WS + 2 * R + lane] * ts.dt[j]);
            }
            loc += inc;
            ph[u] = loc;  // segment-local inclusive sum
          }
          seg[warp * 32 + lane] = loc;
        }
      }
      __syncthreads();
      if (!a.phase.data) {
        if (warp == 0) {
          // Carry the 64-token blocked accumulation across the segments (mamba3/model.py:246-251).
          float off = carry[lane], loc = carry[32 + lane];
          for (int sg = 0; sg < kSegs; ++sg) {
            const int gi = t0 + sg * kSL;
            if (gi > 0 && (gi % kPhaseBlock) == 0) {
              off = fmodf(off + loc, kTwoPi);
              loc = 0.0f;
            }
            const float tot = seg[sg * 32 + lane];
            seg[sg * 32 + lane] = loc;        // within-block sum before this segment
            seg[512 + sg * 32 + lane] = off;  // block offset of this segment
            loc += tot;
          }
          carry[lane] = off;
          carry[32 + lane] = loc;
        }
        __syncthreads();
        if (warp < kSegs) {
          const float base = seg[warp * 32 + lane], off = seg[512 + warp * 32 + lane];
#pragma unroll
          for (int u = 0; u < kSL; ++u) ph[u] = fmod_2pi((base + ph[u]) + off);
        }
      }
      if (warp < kSegs && lane < 32) {
#pragma unroll
        for (int u = 0; u < kSL; ++u) {
          float sn, cs;
          __sincosf(ph[u], &sn, &cs);
          scs[(j0 + u) * 32 + lane] = make_float2(cs, sn);
          if (t0 + j0 + u == L - 1 && a.final_phase.data && lane < S) {
            const m3_tensor& fp = a.final_phase;
            static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + lane * fp.stride[2]] = ph[u];
          }
        }
      }
    }
    __syncthreads();
    const bool fact = mode[2] != 0.0f;
    M3_MARK(4);

    // ---- stage Q', K', V (8 rows per warp; lane holds elements 4*lane .. 4*lane+3) ----
#pragma unroll
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      const int row = warp * kRowsPerWarp + rr;
      const int j = row / R, r = row % R;
      const bool valid = j < nt;
      const float2 q01 = unpack2<T>(qraw[rr].x), q23 = unpack2<T>(qraw[rr].y);
      const float2 k01 = unpack2<T>(kraw[rr].x), k23 = unpack2<T>(kraw[rr].y);
      const float4 bq = *reinterpret_cast<const float4*>(cst + kCBq + r * kN + 4 * lane);
      const float4 bk = *reinterpret_cast<const float4*>(cst + kCBk + r * kN + 4 * lane);
      const float rq = rqf[rr], rk = rkf[rr];
      float qv[4] = {fmaf(q01.x * rq, wq[0], bq.x), fmaf(q01.y * rq, wq[1], bq.y), fmaf(q23.x * rq, wq[2], bq.z),
                     fmaf(q23.y * rq, wq[3], bq.w)};
      float kv[4] = {fmaf(k01.x * rk, wk[0], bk.x), fmaf(k01.y * rk, wk[1], bk.y), fmaf(k23.x * rk, wk[2], bk.z),
                     fmaf(k23.y * rk, wk[3], bk.w)};
      if (has_phase) {
        const float2* cs_row = scs + min(j, TOK - 1) * 32;
        if (a.mimo_rotation) {
          // pairs (n, n + 64) for n < S (2S == 64): the partner lives in lane ^ 16.
          float qo[4], ko[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            qo[e] = __shfl_xor_sync(0xffffffffu, qv[e], 16);
            ko[e] = __shfl_xor_sync(0xffffffffu, kv[e], 16);
          }
          const int m0 = 4 * (lane & 15);
          if (m0 < S) {
            const float4 c01 = *reinterpret_cast<const float4*>(cs_row + m0);
            const float4 c23 = *reinterpret_cast<const float4*>(cs_row + m0 + 2);
            const float cs[4] = {c01.x, c01.z, c23.x, c23.z};
            const float sn[4] = {c01.y, c01.w, c23.y, c23.w};
            if (lane < 16) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                qv[e] = qv[e] * cs[e] - qo[e] * sn[e];
                kv[e] = kv[e] * cs[e] - ko[e] * sn[e];
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                qv[e] = qo[e] * sn[e] + qv[e] * cs[e];
                kv[e] = ko[e] * sn[e] + kv[e] * cs[e];
              }
            }
          }
        } else if (2 * lane < S) {
          // adjacent pairs (2m, 2m+1) with m = 2 lane, 2 lane + 1 (S is even here or the tail is masked)
          const float4 c = *reinterpret_cast<const float4*>(cs_row + 2 * lane);
          float q0 = qv[0], q1 = qv[1], k0 = kv[0], k1 = kv[1];
          qv[0] = q0 * c.x - q1 * c.y;
          qv[1] = q0 * c.y + q1 * c.x;
          kv[0] = k0 * c.x - k1 * c.y;
          kv[1] = k0 * c.y + k1 * c.x;
          if (2 * lane + 1 < S) {
            q0 = qv[2]; q1 = qv[3]; k0 = kv[2]; k1 = kv[3];
            qv[2] = q0 * c.z - q1 * c.w;
            qv[3] = q0 * c.w + q1 * c.z;
            kv[2] = k0 * c.z - k1 * c.w;
            kv[3] = k0 * c.w + k1 * c.z;
          }
        }
      }
      if (valid && a.final_k.data && t0 + j == L - 1) {
        const m3_tensor& fkt = a.final_k;
        T* fkp = static_cast<T*>(fkt.data) + b * fkt.stride[0] + h * fkt.stride[1] + r * fkt.stride[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) fkp[(4 * lane + e) * fkt.stride[3]] = from_f<T>(kv[e]);
      }
      const float fqj = valid ? fq[j] : 0.0f, fkj = valid ? fk[j] : 0.0f;
      *reinterpret_cast<uint2*>(smem + kOffQ + swz(row, 4 * lane, kRows)) =
          make_uint2(pack2<T>(qv[0] * fqj, qv[1] * fqj), pack2<T>(qv[2] * fqj, qv[3] * fqj));
      *reinterpret_cast<uint2*>(smem + kOffK + swz(row, 4 * lane, kRows)) =
          make_uint2(pack2<T>(kv[0] * fkj, kv[1] * fkj), pack2<T>(kv[2] * fkj, kv[3] * fkj));
      // V row (p = 2 lane, 2 lane + 1); V2 = V e^{cum_last - cum} in the W buffer when not factorised.
      uint32_t vw = vraw[rr];
      float2 v = unpack2<T>(vw);
      if (R > 1) {
        const float2 mx = *reinterpret_cast<const float2*>(cst + kCMx + r * kP + 2 * lane);
        v.x *= mx.x;
        v.y *= mx.y;
        vw = pack2<T>(v.x, v.y);
      }
      *reinterpret_cast<uint32_t*>(smem + kOffV + swz(row, 2 * lane, kRows)) = vw;
      if (!fact) {
        const float ed = valid ? ts.edec[j] : 0.0f;
        *reinterpret_cast<uint32_t*>(smem + kOffW + swz(row, 2 * lane, kRows)) = pack2<T>(v.x * ed, v.y * ed);
      }
      if (r == 0) *reinterpret_cast<uint32_t*>(smem + kOffZ + swz(j, 2 * lane, kRows)) = zraw[rr];
    }

    M3_MARK(5);
    // ---- state: TMEM X (S = phi X) -> St = S in 16 bits (state before this tile); X *= new factor ----
    const float cmid = mode[0], cl = mode[1];
    const float state_mult = (fact ? expf(cmid) : last_decay) * phi;
    const float phi_new = fact ? expf(cl - cmid) : 1.0f;
    {
      uint32_t r16[16];
      fence_after();
      M3_TMEM_LD16(tmem + lane_base + kColState + part * 16, r16);
      tmem_wait_ld();
      const int n = quad * 32 + lane;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = pack2<T>(__uint_as_float(r16[c * 8 + 2 * i]) * phi, __uint_as_float(r16[c * 8 + 2 * i + 1]) * phi);
        *reinterpret_cast<uint4*>(smem + kOffST + swz(n, part * 16 + c * 8, kN)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) r16[j] = __float_as_uint(__uint_as_float(r16[j]) * state_mult);
      M3_TMEM_ST16(tmem + lane_base + kColState + part * 16, r16);
      tmem_wait_st();
    }
    phi = phi_new;
    fence_async_smem();
    fence_before();
    __syncthreads();

    M3_MARK(6);
    // ---- MMA group 1: scores = Q' K'^T, inter = Q' St, X += K'^T V (or V2) ----
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
                sdesc(sbase + kOffST + kk * 2048, kN * 128, 1024), id_nmn, kk > 0);
      }
      const uint32_t vsrc = fact ? kOffV : kOffW;
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        mma_f16(tmem + kColState, sdesc(sbase + kOffK + kk * 2048, kRows * 128, 1024),
                sdesc(sbase + vsrc + kk * 2048, kRows * 128, 1024), id_state, 1);
      }
      mma_commit(bar_addr);
    }
    if (!mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    fence_after();

    M3_MARK(7);
    // ---- W = scores o decay -> smem (16-bit, K-major); 32 columns per thread ----
    {
      const int i = quad * 32 + lane;
      const int ti = min(i / R, TOK - 1);
      const int col0 = part * 32;
      const bool all_masked = (col0 / R) > ((quad * 32 + 31) / R);  // warp-uniform
      if (all_masked) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + c * 8, kRows)) = make_uint4(0, 0, 0, 0);
      } else {
        uint32_t r32[32];
        M3_TMEM_LD32(tmem + lane_base + kColScores + col0, r32);
        tmem_wait_ld();
        const float di = ts.diag[ti];
        const int lo = ti * R - col0;  // columns [lo, lo + R) are this row's token; below lo: earlier tokens
        if (fact) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int k0 = c * 8 + e * 2;
              const float s0 = __uint_as_float(r32[k0]), s1 = __uint_as_float(r32[k0 + 1]);
              const float w0 = k0 < lo ? s0 : (k0 < lo + R ? s0 * di : 0.0f);
              const float w1 = k0 + 1 < lo ? s1 : (k0 + 1 < lo + R ? s1 * di : 0.0f);
              w[e] = pack2<T>(w0, w1);
            }
            *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + c * 8, kRows)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else {
          const float ci = cum_l2[ti];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float vals[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int k0 = c * 8 + e * 2 + u;
                const float sv = __uint_as_float(r32[k0]);
                vals[u] = k0 < lo ? sv * ex2_approx(ci - cum_l2[(col0 + k0) / R]) : (k0 < lo + R ? sv * di : 0.0f);
              }
              w[e] = pack2<T>(vals[0], vals[1]);
            }
            *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + c * 8, kRows)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    }
    fence_async_smem();
    fence_before();
    __syncthreads();

    M3_MARK(8);
    // ---- MMA group 2: intra = W V (into the scores columns 0..63) ----
    if (tid == 0) {
      fence_after();
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColIntra, sdesc(sbase + kOffW + koff, 16, 1024),
                sdesc(sbase + kOffV + kk * 2048, kRows * 128, 1024), id_nmn, kk > 0);
      }
      mma_commit(bar_addr);
    }
    if (!mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    fence_after();

    M3_MARK(9);
    // ---- epilogue: 16 output columns per thread ----
    {
      const int i = quad * 32 + lane;
      const int ti = i / R, r = i % R;
      const int tc = min(ti, TOK - 1);
      uint32_t ra[16], ri[16];
      M3_TMEM_LD16(tmem + lane_base + kColIntra + part * 16, ra);
      M3_TMEM_LD16(tmem + lane_base + kColInter + part * 16, ri);
      tmem_wait_ld();
      const bool valid = ti < nt;
      const float gi = ts.ecum[tc];
      float out[16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 vv = *reinterpret_cast<const uint4*>(smem + kOffV + swz(i, part * 16 + c * 8, kRows));
        const uint4 zz = *reinterpret_cast<const uint4*>(smem + kOffZ + swz(tc, part * 16 + c * 8, kRows));
        const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
        const uint32_t zw[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 v = unpack2<T>(vw[e]);
          const float2 z = unpack2<T>(zw[e]);
          const float vz[2] = {v.x, v.y};
          float zz2[2] = {z.x, z.y};
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int jj = c * 8 + e * 2 + u;
            const int p = part * 16 + jj;
            float y = gi * __uint_as_float(ri[jj]) + __uint_as_float(ra[jj]) + Dh * vz[u];
            float zv = zz2[u];
            if (R > 1) zv *= cst[kCMz + r * kP + p];
            y *= __fdividef(zv, 1.0f + __expf(-zv));
            if (R > 1) y *= cst[kCMo + r * kP + p];
            out[jj] = y;
          }
        }
      }
      if (R > 1) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
          for (int o = 1; o < R; o <<= 1) out[jj] += __shfl_xor_sync(0xffffffffu, out[jj], o);
        }
      }
      if (valid && r == 0) {
        const int t = scan_token(a, t0 + ti);
        const int64_t ob = b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2] +
                           (int64_t)(part * 16) * a.y.stride[3];
        if (vec_y) {
          uint4* dst = reinterpret_cast<uint4*>(yp + ob);
          dst[0] = make_uint4(pack2<T>(out[0], out[1]), pack2<T>(out[2], out[3]), pack2<T>(out[4], out[5]),
                              pack2<T>(out[6], out[7]));
          dst[1] = make_uint4(pack2<T>(out[8], out[9]), pack2<T>(out[10], out[11]), pack2<T>(out[12], out[13]),
                              pack2<T>(out[14], out[15]));
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) yp[ob + jj * a.y.stride[3]] = from_f<T>(out[jj]);
        }
      }
    }
    M3_MARK(10);
    fence_before();
    __syncthreads();
    M3_MARK(11);
    if (*abort_flag) break;
  }

  // ---- final state: S[p][n] = phi X^T ----
  fence_after();
  if (!*abort_flag) {
    uint32_t r16[16];
    M3_TMEM_LD16(tmem + lane_base + kColState + part * 16, r16);
    tmem_wait_ld();
    const int n = quad * 32 + lane;
    const m3_tensor& fs = a.final_state;
    float* fsp = static_cast<float*>(fs.data) + b * fs.stride[0] + h * fs.stride[1] + n * fs.stride[3];
#pragma unroll
    for (int j = 0; j < 16; ++j) fsp[(part * 16 + j) * fs.stride[2]] = __uint_as_float(r16[j]) * phi;
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

static bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

template <typename T, int R>
static cudaError_t launch_r(const m3_scan_args& a, cudaStream_t stream) {
  // 8-byte vector loads of q/k rows and 4-byte loads of value/gate pairs need unit element stride and
  // aligned row starts; otherwise the kernel uses element loads.
  auto even = [](int64_t s, int m) { return s % m == 0; };
  const int vec_qk = a.q.stride[4] == 1 && a.k.stride[4] == 1 && aligned(a.q.data, 8) && aligned(a.k.data, 8) &&
                     even(a.q.stride[0], 4) && even(a.q.stride[1], 4) && even(a.q.stride[2], 4) &&
                     even(a.q.stride[3], 4) && even(a.k.stride[0], 4) && even(a.k.stride[1], 4) &&
                     even(a.k.stride[2], 4) && even(a.k.stride[3], 4);
  const int vec_vz = a.value.stride[3] == 1 && a.gate.stride[3] == 1 && aligned(a.value.data, 4) &&
                     aligned(a.gate.data, 4) && even(a.value.stride[0], 2) && even(a.value.stride[1], 2) &&
                     even(a.value.stride[2], 2) && even(a.gate.stride[0], 2) && even(a.gate.stride[1], 2) &&
                     even(a.gate.stride[2], 2);
  const int vec_y = a.y.stride[3] == 1 && aligned(a.y.data, 16) && even(a.y.stride[0], 8) &&
                    even(a.y.stride[1], 8) && even(a.y.stride[2], 8);
  if (a.workspace.data) {
    const int64_t tokens = (int64_t)a.batch * a.length;
    token_prep_kernel<T><<<(unsigned)((tokens + 7) / 8), 256, 0, stream>>>(a, static_cast<float*>(a.workspace.data));
    cudaError_t pe = cudaGetLastError();
    if (pe != cudaSuccess) return pe;
  }
  auto kern = scan_umma_kernel<T, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<dim3(a.heads, a.batch), kThreads, kSmemBytes, stream>>>(a, vec_qk, vec_vz, vec_y);
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

int64_t scan_umma_workspace_bytes(const m3_scan_args& a) {
  const bool need = a.q_norm_w.data != nullptr || a.angles.data != nullptr;
  if (!need) return 0;
  return (int64_t)a.batch * a.length * (2 * a.rank + a.num_angles) * (int64_t)sizeof(float);
}

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
