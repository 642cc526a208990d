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

constexpr int kRows = 64;       // flattened (token, rank) rows per tile = MMA M of the row GEMMs
constexpr int kN = 128;         // d_state
constexpr int kP = 64;          // head_dim
constexpr int kThreads = 256;   // 8 warps; two CTAs share an SM
constexpr int kWarps = kThreads / 32;
constexpr int kMaxAngles = 32;

// Shared-memory map (bytes from the 1024-aligned base).
constexpr uint32_t kOffQ = 0;                          // Q' [64 rows][128]    16 KB
constexpr uint32_t kOffK = kOffQ + kRows * kN * 2;     // K' [64 rows][128]    16 KB
constexpr uint32_t kOffW = kOffK + kRows * kN * 2;     // W  [64][64]           8 KB
constexpr uint32_t kOffV = kOffW + kRows * kRows * 2;  // V  [64 rows][64]      8 KB
constexpr uint32_t kOffV2 = kOffV + kRows * kP * 2;    // V2 [64 rows][64]      8 KB (unfactorised tiles)
constexpr uint32_t kOffST = kOffV2 + kRows * kP * 2;   // St [128 n][64 p]     16 KB
constexpr uint32_t kOffZ = kOffST + kN * kP * 2;       // z  [tokens][64] x 2 buffers (tile parity)
constexpr uint32_t kOffF = kOffZ + 2 * kRows * kP * 2; // float region
// float region (in floats): per-token scalars, then constants / workspace rows sized by the rank.
constexpr int kSCum = 0, kSEcum = 64, kSEdec = 128, kSScale = 192, kSDiag = 256, kSDt = 320, kSWsum = 384,
              kSCumL2 = 448, kSFq = 512, kSFk = 576, kSMode = 640, kSRaw = 656, kSEnd = 656 + 3 * 68;
// Workspace floats per token: RMS factors of the q rows (R), of the k rows (R), pi*tanh(angle) (S),
// padded to a multiple of 4 so each token's row is a run of 16-byte chunks.
__host__ __device__ constexpr int ws_stride(int R, int S) { return ((2 * R + S + 3) / 4) * 4; }
template <int R> struct Layout {
  static constexpr int TOK = kRows / R;
  static constexpr int WSP = ws_stride(R, kMaxAngles);
  static constexpr int CBq = kSEnd, CBk = CBq + R * kN, CMx = CBk + R * kN, CMz = CMx + R * kP, CMo = CMz + R * kP;
  static constexpr int Ws = ((CMo + R * kP + 3) / 4) * 4;  // tile's workspace rows [TOK][WSP] (phase in place)
  static constexpr int Seg = Ws + TOK * WSP;            // [kWarps][32] sums, then [kWarps][32] offsets
  static constexpr int Carry = Seg + 2 * kWarps * 32;   // [0..31] block offset, [32..63] within-block sum
  static constexpr int FEnd = Carry + 64;
  static constexpr uint32_t OffBar = kOffF + ((FEnd * 4 + 15) / 16) * 16;  // mbarrier, tmem slot, abort flag
  static constexpr uint32_t SmemBytes = OffBar + 64 + 1024;                // + alignment slack
};

// TMEM columns (fp32). The M = 64 accumulators hold row m in lane (m % 16) + 32 (m / 16); the
// state (an M = 128 accumulator) holds row n in lane n.
constexpr uint32_t kColScores = 0;    // [64 x 64]
constexpr uint32_t kColInter = 64;    // [64 x 64]
constexpr uint32_t kColIntra = 128;   // [64 x 64]
constexpr uint32_t kColState = 192;   // S^T [128 x 64]
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

#define M3_TMEM_ST32(taddr, r)                                                                                \
  asm volatile(                                                                                               \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16," \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                      \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),       \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),           \
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),          \
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]))

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

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

// Per-token pre-pass: ws[(b*L + t) * W + ...] with W = ws_stride(R, S) holds the RMS factor of each
// q row (r), of each k row (R + r) and pi*tanh(angle) (2R + s). Token index in original order.
// One warp per token.
template <typename T>
__global__ void __launch_bounds__(256) token_prep_kernel(const m3_scan_args a, float* ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok = (int64_t)blockIdx.x * 8 + warp;
  const int64_t total = (int64_t)a.batch * a.length;
  if (tok >= total) return;
  const int b = (int)(tok / a.length), t = (int)(tok % a.length);
  const int R = a.rank, S = a.num_angles, W = ws_stride(R, S);
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
__global__ void __launch_bounds__(kThreads, 2) scan_umma_kernel(const m3_scan_args a, int vec_y) {
  using Lay = Layout<R>;
  constexpr int TOK = Lay::TOK;
  constexpr int kSL = TOK / kWarps > 0 ? TOK / kWarps : 1;   // phase tokens per warp segment
  constexpr int kSegs = TOK / kSL;                           // phase segments per tile (<= 8)
  constexpr int kRowsPerWarp = kRows / kWarps;               // staging rows per warp (8)
  constexpr bool kBf16 = DType<T>::id == M3_BF16;
  // Largest |cum - cmid| for which the decay can be split into per-row operand factors
  // e^{cum_i - cmid} (Q rows) and e^{cmid - cum_j} (K rows) without leaving the 16-bit range.
  constexpr float kLim = kBf16 ? 80.0f : 8.0f;
  const int h = blockIdx.x, b = blockIdx.y;
  const int S = a.num_angles, L = a.length;
  const int g = h / (a.heads / a.groups);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, part = warp >> 2;  // TMEM lane quadrant, column half
  const int WS = ws_stride(R, S);               // workspace floats per token

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* fsm = reinterpret_cast<float*>(smem + kOffF);
  float* cum = fsm + kSCum;
  float* ecum = fsm + kSEcum;
  float* edec = fsm + kSEdec;
  float* scale = fsm + kSScale;
  float* diag = fsm + kSDiag;
  float* sdt = fsm + kSDt;
  float* wsum = fsm + kSWsum;
  float* cum_l2 = fsm + kSCumL2;
  float* fq = fsm + kSFq;
  float* fk = fsm + kSFk;
  float* mode = fsm + kSMode;  // [0] cmid, [1] cum_last, [2] factorised, [3] e^{cum_last}
  float* sraw = fsm + kSRaw;   // raw per-token dt, adt, sigma of the next tile [3][68]
  float* cst = fsm;
  float* wsb = fsm + Lay::Ws;  // the tile's workspace rows; the phase replaces pi*tanh in place
  float* seg = fsm + Lay::Seg;
  float* carry = fsm + Lay::Carry;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::OffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + Lay::OffBar + 16);
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
  // Row bases (the rows themselves are contiguous and 16-byte aligned: scan_umma_supported).
  const int64_t q_b0 = b * a.q.stride[0] + g * a.q.stride[2];
  const int64_t k_b0 = b * a.k.stride[0] + g * a.k.stride[2];
  const int64_t v_b0 = b * a.value.stride[0] + h * a.value.stride[2];
  const int64_t z_b0 = b * a.gate.stride[0] + h * a.gate.stride[2];
  const int64_t ws_b = (int64_t)b * L * WS;

  // ---- loads of a tile, issued one tile ahead (cp.async for rows; see the tile loop) ----
  // q/k rows go straight into the Q'/K' tiles (processed in place), raw x into the W tile, z into the
  // z tile of the tile's parity, workspace rows into wsb.
  auto issue_qk = [&](int t0n, int ntn) {
    constexpr int kQChunks = kRows * (kN / 8);
    for (int c = tid; c < kQChunks; c += kThreads) {
      const int row = c >> 4, c8 = c & 15;
      const int j = row / R, r = row % R;
      if (j < ntn) {
        const int t = scan_token(a, t0n + j);
        const uint32_t off = swz(row, c8 * 8, kRows);
        cp_async16(sbase + kOffQ + off, qp + q_b0 + (int64_t)t * a.q.stride[1] + r * a.q.stride[3] + c8 * 8);
        cp_async16(sbase + kOffK + off, kp + k_b0 + (int64_t)t * a.k.stride[1] + r * a.k.stride[3] + c8 * 8);
      }
    }
  };
  auto issue_x = [&](int t0n, int ntn) {
    for (int c = tid; c < TOK * (kP / 8); c += kThreads) {
      const int j = c >> 3, c8 = c & 7;
      if (j < ntn) {
        const int t = scan_token(a, t0n + j);
        cp_async16(sbase + kOffW + swz(j, c8 * 8, kRows), vp + v_b0 + (int64_t)t * a.value.stride[1] + c8 * 8);
      }
    }
  };
  auto issue_z = [&](int t0n, int ntn, int par) {
    const uint32_t zoff = kOffZ + par * (kRows * kP * 2);
    for (int c = tid; c < TOK * (kP / 8); c += kThreads) {
      const int j = c >> 3, c8 = c & 7;
      if (j < ntn) {
        const int t = scan_token(a, t0n + j);
        cp_async16(sbase + zoff + swz(j, c8 * 8, kRows), zp + z_b0 + (int64_t)t * a.gate.stride[1] + c8 * 8);
      }
    }
  };
  // Per-token scalars of a tile: thread j <= TOK fetches the raw words of token j (j == TOK: the
  // first token after the tile) into registers without using them, so the loads stay in flight;
  // finish_scalars() converts them (softplus / heavy-tail / sigmoid) into sraw later.
  uint32_t raw_dt = 0, raw_adt = 0, raw_trap = 0;
  bool raw_ok = false;
  auto raw_word = [](const m3_tensor& t, int64_t idx) -> uint32_t {
    if (t.dtype == M3_F32) return __float_as_uint(static_cast<const float*>(t.data)[idx]);
    return (uint32_t)static_cast<const uint16_t*>(t.data)[idx];
  };
  auto word_to_f = [](uint32_t w, int dtype) -> float {
    if (dtype == M3_F32) return __uint_as_float(w);
    if (dtype == M3_BF16) return __uint_as_float(w << 16);
    return __half2float(__ushort_as_half((unsigned short)w));
  };
  auto fetch_scalars = [&](int t0n, int ntn) {
    raw_ok = false;
    if (tid <= TOK && t0n + tid < L && (tid < ntn || tid == TOK)) {
      const int t = scan_token(a, t0n + tid);
      raw_dt = raw_word(a.dt, b * a.dt.stride[0] + (int64_t)t * a.dt.stride[1] + h * a.dt.stride[2]);
      raw_adt = raw_word(a.adt, b * a.adt.stride[0] + (int64_t)t * a.adt.stride[1] + h * a.adt.stride[2]);
      raw_trap = raw_word(a.trap, b * a.trap.stride[0] + (int64_t)t * a.trap.stride[1] + h * a.trap.stride[2]);
      raw_ok = true;
    }
  };
  const float dt_bias_h = a.dt_bias.data ? ld_t(a.dt_bias, h * a.dt_bias.stride[0]) : 0.0f;
  auto finish_scalars = [&]() {
    if (tid <= TOK) {
      float dtv = 0.0f, adtv = 0.0f, sg = 0.0f;
      if (raw_ok) {
        if (a.dt_bias.data) {
          // mamba3/model.py:195-198: dt = softplus(delta + dt_bias); A = -heavytail(a) clamped <= -1e-4.
          dtv = softplusf_(word_to_f(raw_dt, a.dt.dtype) + dt_bias_h);
          adtv = fminf(-heavy_tailf(word_to_f(raw_adt, a.adt.dtype)), -kAFloor) * dtv;
        } else {
          dtv = word_to_f(raw_dt, a.dt.dtype);
          adtv = word_to_f(raw_adt, a.adt.dtype);
        }
        sg = sigmoidf_(word_to_f(raw_trap, a.trap.dtype));
      }
      sraw[tid] = dtv;
      sraw[68 + tid] = adtv;
      sraw[136 + tid] = sg;
    }
  };
  // Workspace rows (cp.async) or their stand-ins, and the phase tensor of the op-level API.
  auto fetch_small = [&](int t0n, int ntn) {
    if (has_ws) {
      const int chunks = WS / 4;  // <= 12: one 16-slot row per token, no division
      for (int c = tid; c < TOK * 16; c += kThreads) {
        const int j = c >> 4, c4 = c & 15;
        if (j < ntn && c4 < chunks) {
          const int t = scan_token(a, t0n + j);
          cp_async16(smem_u32(wsb + j * WS + 4 * c4), ws + ws_b + (int64_t)t * WS + 4 * c4);
        }
      }
    } else {
      for (int i = tid; i < TOK * 2 * R; i += kThreads) wsb[(i / (2 * R)) * WS + i % (2 * R)] = 1.0f;
    }
    if (a.phase.data) {
      for (int i = tid; i < TOK * S; i += kThreads) {
        const int j = i / S, sidx = i % S;
        float v = 0.0f;
        if (j < ntn) {
          const int t = scan_token(a, t0n + j);
          v = ld_t(a.phase, b * a.phase.stride[0] + (int64_t)t * a.phase.stride[1] + h * a.phase.stride[2] +
                                sidx * a.phase.stride[3]);
        }
        wsb[j * WS + 2 * R + sidx] = v;
      }
    }
  };

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
    cst[Lay::CBq + i] = bq;
    cst[Lay::CBk + i] = bk;
  }
  if (R > 1) {
    for (int i = tid; i < R * kP; i += kThreads) {
      const int r = i / kP, p = i % kP;
      cst[Lay::CMx + i] = ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2]);
      cst[Lay::CMz + i] = ld_t(a.mimo_z, h * a.mimo_z.stride[0] + r * a.mimo_z.stride[1] + p * a.mimo_z.stride[2]);
      cst[Lay::CMo + i] =
          ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
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
  // Loads of the first tile.
  {
    const int nt0 = min(TOK, L);
    issue_qk(0, nt0);
    issue_x(0, nt0);
    issue_z(0, nt0, 0);
    fetch_small(0, nt0);
    fetch_scalars(0, nt0);
    finish_scalars();
    cp_async_commit();
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
    uint32_t r32[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int p = part * 32 + j;
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
          const float vr = R > 1 ? v * cst[Lay::CMx + rr * kP + p] : v;
          acc += vr * ld_t(ik, b * ik.stride[0] + h * ik.stride[1] + rr * ik.stride[2] + n * ik.stride[3]);
        }
        s += c0 * acc;
      }
      r32[j] = __float_as_uint(s);
    }
    M3_TMEM_ST32(tmem + lane_base + kColState + part * 32, r32);
    tmem_wait_st();
  }

  const uint32_t id_scores = idesc(64, 64, kBf16, false, false);  // K-major A and B
  const uint32_t id_nmn = idesc(64, 64, kBf16, false, true);      // K-major A, MN-major B
  const uint32_t id_state = idesc(128, 64, kBf16, true, true);    // MN-major A and B
  uint32_t phase_bit = 0;
  float phi = 1.0f;  // TMEM holds S / phi
#ifdef M3_SECTION_TIMING
  long long mark_prev_ = clock64();
#endif

  int tile = 0;
  for (int t0 = 0; t0 < L; t0 += TOK, ++tile) {
    const int nt = min(TOK, L - t0);
    const int t0n = t0 + TOK, ntn = min(TOK, L - t0n);  // next tile (ntn <= 0: none)
    M3_MARK(0);
    cp_async_wait_all();  // this tile's rows, workspace rows (issued during the previous tile)
    __syncthreads();
    M3_MARK(1);

    // ---- per-token scalars (mamba3/ops.py:659-671) and the cumulative decay ----
    if (tid < TOK) {
      sdt[tid] = tid < nt ? sraw[tid] : 0.0f;
      cum[tid] = tid < nt ? sraw[68 + tid] : 0.0f;
      edec[tid] = sraw[136 + tid];
    } else if (tid == TOK) {
      wsum[4] = sraw[TOK];
      wsum[5] = sraw[136 + TOK];
    }
    __syncthreads();
    float cv = 0.0f;
    if (tid < 64) {
      cv = warp_incl_scan(tid < TOK ? cum[tid] : 0.0f, lane);
      if (lane == 31) wsum[tid >> 5] = cv;
      if (tid < TOK) {
        float sc = 0.0f, dg = 0.0f;
        if (tid < nt) {
          const float gamma = sdt[tid] * edec[tid];
          float nxt = 0.0f;
          if (tid + 1 < nt) nxt = sdt[tid + 1] * (1.0f - edec[tid + 1]);
          else if (t0 + tid + 1 < L) nxt = wsum[4] * (1.0f - wsum[5]);
          sc = gamma + nxt;
          dg = gamma / sc;
        }
        scale[tid] = sc;
        diag[tid] = dg;
      }
    }
    __syncthreads();
    if (tid < TOK) {
      if (tid >= 32) cv += wsum[0];
      cum[tid] = cv;
    }
    __syncthreads();
    // Decay factorisation for this tile (warp 0): cmid = cum of the middle token.
    if (warp == 0) {
      const float cmid = cum[(nt - 1) >> 1];
      const float cl = cum[nt - 1];
      float dev = 0.0f;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j < nt) dev = fmaxf(dev, fabsf(cum[j] - cmid));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dev = fmaxf(dev, __shfl_xor_sync(0xffffffffu, dev, o));
      const bool fact = dev <= kLim;
      const float ecm = expf(cmid);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int j = lane + 32 * k;
        if (j < TOK) {
          const float c = cum[j];
          cum_l2[j] = c * kLog2e;
          const bool v = j < nt;
          fq[j] = v ? (fact ? __expf(c - cmid) : 1.0f) : 0.0f;
          fk[j] = v ? (fact ? scale[j] * __expf(cmid - c) : scale[j]) : 0.0f;
          ecum[j] = v ? (fact ? ecm : expf(c)) : 0.0f;
          edec[j] = v ? expf(cl - c) : 0.0f;
        }
      }
      if (lane == 0) {
        mode[0] = cmid;
        mode[1] = cl;
        mode[2] = fact ? 1.0f : 0.0f;
        mode[3] = expf(cl);
      }
    }
    M3_MARK(2);
    // ---- phase of every (token, angle), written over pi*tanh(angle) in wsb ----
    if (a.angles.data) {
      const int j0 = warp * kSL;
      float ph[kSL];
      if (warp < kSegs) {
        float loc = 0.0f;
#pragma unroll
        for (int u = 0; u < kSL; ++u) {
          const int j = j0 + u;
          loc += (lane < S && j < nt) ? fmod_2pi(wsb[j * WS + 2 * R + lane] * sdt[j]) : 0.0f;
          ph[u] = loc;  // segment-local inclusive sum
        }
        seg[warp * 32 + lane] = loc;
      }
      __syncthreads();
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
          seg[sg * 32 + lane] = loc;                 // within-block sum before this segment
          seg[kWarps * 32 + sg * 32 + lane] = off;   // block offset of this segment
          loc += tot;
        }
        carry[lane] = off;
        carry[32 + lane] = loc;
      }
      __syncthreads();
      if (warp < kSegs && lane < S) {
        const float base = seg[warp * 32 + lane], off = seg[kWarps * 32 + warp * 32 + lane];
#pragma unroll
        for (int u = 0; u < kSL; ++u) {
          const int j = j0 + u;
          const float phv = fmod_2pi((base + ph[u]) + off);
          wsb[j * WS + 2 * R + lane] = phv;
          if (t0 + j == L - 1 && a.final_phase.data) {
            const m3_tensor& fp = a.final_phase;
            static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + lane * fp.stride[2]] = phv;
          }
        }
      }
    } else if (a.phase.data && a.final_phase.data && t0 + TOK >= L && tid < S) {
      const m3_tensor& fp = a.final_phase;
      static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + tid * fp.stride[2]] =
          wsb[(nt - 1) * WS + 2 * R + tid];
    }
    __syncthreads();
    const bool fact = mode[2] != 0.0f;
    M3_MARK(3);

    // ---- stage Q', K', V (8 rows per warp; lane holds elements 4*lane .. 4*lane+3) ----
#pragma unroll
    for (int rr = 0; rr < kRowsPerWarp; ++rr) {
      const int row = warp * kRowsPerWarp + rr;
      const int j = row / R, r = row % R;
      const bool valid = j < nt;
      const int jc = min(j, TOK - 1);
      const float* wrow = wsb + jc * WS;
      const uint32_t qk_off = swz(row, 4 * lane, kRows);
      const uint2 qraw = *reinterpret_cast<const uint2*>(smem + kOffQ + qk_off);
      const uint2 kraw = *reinterpret_cast<const uint2*>(smem + kOffK + qk_off);
      const float2 q01 = unpack2<T>(qraw.x), q23 = unpack2<T>(qraw.y);
      const float2 k01 = unpack2<T>(kraw.x), k23 = unpack2<T>(kraw.y);
      const float4 bq = *reinterpret_cast<const float4*>(cst + Lay::CBq + r * kN + 4 * lane);
      const float4 bk = *reinterpret_cast<const float4*>(cst + Lay::CBk + r * kN + 4 * lane);
      const float rq = wrow[r], rk = wrow[R + r];
      float qv[4] = {fmaf(q01.x * rq, wq[0], bq.x), fmaf(q01.y * rq, wq[1], bq.y), fmaf(q23.x * rq, wq[2], bq.z),
                     fmaf(q23.y * rq, wq[3], bq.w)};
      float kv[4] = {fmaf(k01.x * rk, wk[0], bk.x), fmaf(k01.y * rk, wk[1], bk.y), fmaf(k23.x * rk, wk[2], bk.z),
                     fmaf(k23.y * rk, wk[3], bk.w)};
      if (has_phase) {
        const float* phr = wrow + 2 * R;
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
            const float4 pv = *reinterpret_cast<const float4*>(phr + m0);
            const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float sn, cs;
              __sincosf(pa[e], &sn, &cs);
              if (lane < 16) {
                qv[e] = qv[e] * cs - qo[e] * sn;
                kv[e] = kv[e] * cs - ko[e] * sn;
              } else {
                qv[e] = qo[e] * sn + qv[e] * cs;
                kv[e] = ko[e] * sn + kv[e] * cs;
              }
            }
          }
        } else if (2 * lane < S) {
          // adjacent pairs (2m, 2m+1) with m = 2 lane, 2 lane + 1
          const float2 pv = *reinterpret_cast<const float2*>(phr + 2 * lane);
          float sn, cs;
          __sincosf(pv.x, &sn, &cs);
          float q0 = qv[0], q1 = qv[1], k0 = kv[0], k1 = kv[1];
          qv[0] = q0 * cs - q1 * sn;
          qv[1] = q0 * sn + q1 * cs;
          kv[0] = k0 * cs - k1 * sn;
          kv[1] = k0 * sn + k1 * cs;
          if (2 * lane + 1 < S) {
            __sincosf(pv.y, &sn, &cs);
            q0 = qv[2]; q1 = qv[3]; k0 = kv[2]; k1 = kv[3];
            qv[2] = q0 * cs - q1 * sn;
            qv[3] = q0 * sn + q1 * cs;
            kv[2] = k0 * cs - k1 * sn;
            kv[3] = k0 * sn + k1 * cs;
          }
        }
      }
      if (valid && a.final_k.data && t0 + j == L - 1) {
        const m3_tensor& fkt = a.final_k;
        T* fkp = static_cast<T*>(fkt.data) + b * fkt.stride[0] + h * fkt.stride[1] + r * fkt.stride[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) fkp[(4 * lane + e) * fkt.stride[3]] = from_f<T>(kv[e]);
      }
      // Rows past the end are zeroed by selection: their shared memory holds stale bytes.
      const float fqj = fq[jc], fkj = fk[jc];
      *reinterpret_cast<uint2*>(smem + kOffQ + qk_off) =
          valid ? make_uint2(pack2<T>(qv[0] * fqj, qv[1] * fqj), pack2<T>(qv[2] * fqj, qv[3] * fqj)) : make_uint2(0, 0);
      *reinterpret_cast<uint2*>(smem + kOffK + qk_off) =
          valid ? make_uint2(pack2<T>(kv[0] * fkj, kv[1] * fkj), pack2<T>(kv[2] * fkj, kv[3] * fkj)) : make_uint2(0, 0);
      // V row (p = 2 lane, 2 lane + 1) from the raw x row parked in the W tile; V2 = V e^{cum_last - cum}
      // when the tile is not factorised.
      uint32_t vw = valid ? *reinterpret_cast<const uint32_t*>(smem + kOffW + swz(j, 2 * lane, kRows)) : 0u;
      float2 v = unpack2<T>(vw);
      if (R > 1) {
        const float2 mx = *reinterpret_cast<const float2*>(cst + Lay::CMx + r * kP + 2 * lane);
        v.x *= mx.x;
        v.y *= mx.y;
        vw = pack2<T>(v.x, v.y);
      }
      *reinterpret_cast<uint32_t*>(smem + kOffV + swz(row, 2 * lane, kRows)) = vw;
      if (!fact) {
        const float ed = edec[jc];
        *reinterpret_cast<uint32_t*>(smem + kOffV2 + swz(row, 2 * lane, kRows)) = pack2<T>(v.x * ed, v.y * ed);
      }
    }
    M3_MARK(4);

    // ---- state: TMEM X (S = phi X) -> St = S in 16 bits (state before this tile); X *= factor ----
    const float cmid = mode[0], cl = mode[1];
    const float state_mult = (fact ? expf(cmid) : mode[3]) * phi;
    const float phi_new = fact ? expf(cl - cmid) : 1.0f;
    {
      uint32_t r32[32];
      fence_after();
      M3_TMEM_LD32(tmem + lane_base + kColState + part * 32, r32);
      tmem_wait_ld();
      const int n = quad * 32 + lane;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w[i] = pack2<T>(__uint_as_float(r32[c * 8 + 2 * i]) * phi, __uint_as_float(r32[c * 8 + 2 * i + 1]) * phi);
        *reinterpret_cast<uint4*>(smem + kOffST + swz(n, part * 32 + c * 8, kN)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) r32[j] = __float_as_uint(__uint_as_float(r32[j]) * state_mult);
      M3_TMEM_ST32(tmem + lane_base + kColState + part * 32, r32);
      tmem_wait_st();
    }
    phi = phi_new;
    fence_async_smem();
    fence_before();
    __syncthreads();
    M3_MARK(5);

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
      const uint32_t vsrc = fact ? kOffV : kOffV2;
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        mma_f16(tmem + kColState, sdesc(sbase + kOffK + kk * 2048, kRows * 128, 1024),
                sdesc(sbase + vsrc + kk * 2048, kRows * 128, 1024), id_state, 1);
      }
      mma_commit(bar_addr);
    }
    // While the tensor cores run: the next tile's scalars, workspace rows and z rows (other buffer).
    if (ntn > 0) {
      fetch_scalars(t0n, ntn);
      fetch_small(t0n, ntn);
      issue_z(t0n, ntn, (tile + 1) & 1);
    }
    // One thread polls the barrier; the others wait at __syncthreads without taking issue slots.
    if (tid == 0 && !mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    __syncthreads();
    fence_after();
    // Q'/K' are free now: the next tile's raw q/k rows.
    if (ntn > 0) issue_qk(t0n, ntn);
    M3_MARK(6);

    // ---- W = scores o decay -> smem (16-bit, K-major); lanes 0-15 hold rows, 32 columns each ----
    {
      const int i = quad * 16 + (lane & 15);
      const int ti = min(i / R, TOK - 1);
      const int col0 = part * 32;
      const bool all_masked = (col0 / R) > ((quad * 16 + 15) / R);  // warp-uniform
      if (all_masked) {
        if (lane < 16) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(smem + kOffW + swz(i, col0 + c * 8, kRows)) = make_uint4(0, 0, 0, 0);
        }
      } else {
        uint32_t r32[32];
        M3_TMEM_LD32(tmem + lane_base + kColScores + col0, r32);
        tmem_wait_ld();
        if (lane < 16) {
          const float di = diag[ti];
          const float ci = cum_l2[ti];
          const int lo = ti * R - col0;  // columns [lo, lo + R) are this row's token; below lo: earlier tokens
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
                float wv;
                if (k0 < lo) wv = fact ? sv : sv * ex2_approx(ci - cum_l2[(col0 + k0) / R]);
                else wv = k0 < lo + R ? sv * di : 0.0f;
                vals[u] = wv;
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
    M3_MARK(7);

    // ---- MMA group 2: intra = W V ----
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
    if (tid == 0 && !mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    __syncthreads();
    fence_after();
    // W is free now: the next tile's raw x rows.
    if (ntn > 0) issue_x(t0n, ntn);
    cp_async_commit();
    M3_MARK(8);

    // ---- epilogue: lanes 0-15 own rows, 32 output columns each ----
    {
      const int i = quad * 16 + (lane & 15);
      const int ti = i / R, r = i % R;
      const int tc = min(ti, TOK - 1);
      const uint32_t zoff = kOffZ + (tile & 1) * (kRows * kP * 2);
      uint32_t ra[32], ri[32];
      M3_TMEM_LD32(tmem + lane_base + kColIntra + part * 32, ra);
      M3_TMEM_LD32(tmem + lane_base + kColInter + part * 32, ri);
      tmem_wait_ld();
      const bool valid = lane < 16 && ti < nt;
      const float gi = ecum[tc];
      float out[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 vv = *reinterpret_cast<const uint4*>(smem + kOffV + swz(i, part * 32 + c * 8, kRows));
        const uint4 zz = *reinterpret_cast<const uint4*>(smem + zoff + swz(tc, part * 32 + c * 8, kRows));
        const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
        const uint32_t zw[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 v = unpack2<T>(vw[e]);
          const float2 z = unpack2<T>(zw[e]);
          const float vz[2] = {v.x, v.y};
          const float zz2[2] = {z.x, z.y};
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int jj = c * 8 + e * 2 + u;
            const int p = part * 32 + jj;
            float y = gi * __uint_as_float(ri[jj]) + __uint_as_float(ra[jj]) + Dh * vz[u];
            float zv = zz2[u];
            if (R > 1) zv *= cst[Lay::CMz + r * kP + p];
            y *= __fdividef(zv, 1.0f + __expf(-zv));
            if (R > 1) y *= cst[Lay::CMo + r * kP + p];
            out[jj] = y;
          }
        }
      }
      if (R > 1) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
#pragma unroll
          for (int o = 1; o < R; o <<= 1) out[jj] += __shfl_xor_sync(0xffffffffu, out[jj], o);
        }
      }
      if (valid && r == 0) {
        const int t = scan_token(a, t0 + ti);
        const int64_t ob = b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2] +
                           (int64_t)(part * 32) * a.y.stride[3];
        if (vec_y) {
          uint4* dst = reinterpret_cast<uint4*>(yp + ob);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            dst[c] = make_uint4(pack2<T>(out[8 * c], out[8 * c + 1]), pack2<T>(out[8 * c + 2], out[8 * c + 3]),
                                pack2<T>(out[8 * c + 4], out[8 * c + 5]), pack2<T>(out[8 * c + 6], out[8 * c + 7]));
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) yp[ob + jj * a.y.stride[3]] = from_f<T>(out[jj]);
        }
      }
    }
    M3_MARK(9);
    if (ntn > 0) finish_scalars();  // the next tile's scalars, loaded during the first MMA group
    fence_before();
    __syncthreads();
    M3_MARK(10);
    if (*abort_flag) break;
  }
  cp_async_wait_all();

  // ---- final state: S[p][n] = phi X^T ----
  fence_after();
  if (!*abort_flag) {
    uint32_t r32[32];
    M3_TMEM_LD32(tmem + lane_base + kColState + part * 32, r32);
    tmem_wait_ld();
    const int n = quad * 32 + lane;
    const m3_tensor& fs = a.final_state;
    float* fsp = static_cast<float*>(fs.data) + b * fs.stride[0] + h * fs.stride[1] + n * fs.stride[3];
#pragma unroll
    for (int j = 0; j < 32; ++j) fsp[(part * 32 + j) * fs.stride[2]] = __uint_as_float(r32[j]) * phi;
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
  // 16-byte vector stores of y need unit element stride and aligned row starts.
  auto even = [](int64_t s, int m) { return s % m == 0; };
  const int vec_y = a.y.stride[3] == 1 && aligned(a.y.data, 16) && even(a.y.stride[0], 8) &&
                    even(a.y.stride[1], 8) && even(a.y.stride[2], 8);
  if (a.workspace.data) {
    const int64_t tokens = (int64_t)a.batch * a.length;
    token_prep_kernel<T><<<(unsigned)((tokens + 7) / 8), 256, 0, stream>>>(a, static_cast<float*>(a.workspace.data));
    cudaError_t pe = cudaGetLastError();
    if (pe != cudaSuccess) return pe;
  }
  auto kern = scan_umma_kernel<T, R>;
  constexpr uint32_t smem = Layout<R>::SmemBytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(a.heads, a.batch), kThreads, smem, stream>>>(a, vec_y);
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
  return (int64_t)a.batch * a.length * umma::ws_stride(a.rank, a.num_angles) * (int64_t)sizeof(float);
}

// Rows of q/k (N elements), value and gate (P elements) that start on 16-byte boundaries and are
// contiguous, so the kernel can move them with 16-byte asynchronous copies.
static bool rows16(const m3_tensor& t, int nd) {
  if ((reinterpret_cast<uintptr_t>(t.data) & 15u) != 0 || t.stride[nd - 1] != 1) return false;
  for (int i = 0; i < nd - 1; ++i)
    if (t.stride[i] % 8 != 0) return false;
  return true;
}

bool scan_umma_supported(const m3_scan_args& a) {
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;
  return (a.value.dtype == M3_BF16 || a.value.dtype == M3_F16) && a.d_state == umma::kN &&
         rows16(a.q, 5) && rows16(a.k, 5) && rows16(a.value, 4) && rows16(a.gate, 4) &&
         !(a.q_norm_w.data != nullptr && a.phase.data != nullptr) &&
         a.head_dim == umma::kP && (a.rank == 1 || a.rank == 2 || a.rank == 4 || a.rank == 8) &&
         (!has_phase || (a.mimo_rotation ? a.num_angles == umma::kMaxAngles : a.num_angles <= umma::kMaxAngles));
}

cudaError_t launch_scan_umma(const m3_scan_args& a, cudaStream_t stream) {
  return a.value.dtype == M3_BF16 ? umma::launch_t<__nv_bfloat16>(a, stream) : umma::launch_t<__half>(a, stream);
}

}  // namespace m3
