// Chunked Mamba-3 SSD forward on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Shapes served: bf16/fp16 activations, d_state N = 128, head_dim P = 64, any rank R in
// {1, 2, 4, 8}, up to 32 rotation angles. A pre-pass (token_prep_kernel) computes the per-token
// values every head shares — RMS factors of the q/k rows and pi*tanh(angle) — once into the
// caller's workspace. Then one CTA (256 threads, 8 warps; two CTAs per SM) owns one
// (batch, head[, segment]) and walks its tokens in tiles of 64 flattened (token, rank) rows
// (64 / R tokens), keeping the FP32 state S^T [N=128, P=64] resident in tensor memory.
//
// Per tile (mamba3/ops.py:716-816 math; mamba3/_triton.py:74-413 is the reference's fused form):
//   stage   Q' = rot(norm(C) + C_bias) e^{cum - cmid}           [64 rows, 128] 16-bit, K-major
//           K' = rot(norm(B) + B_bias) scale e^{cmid - cum}     [64 rows, 128] 16-bit
//           V  = x mimo_x                                        [64 rows, 64]
//           V2 = V e^{cum_last - cum}  (only tiles whose decay range is too wide to factorise)
//           St = 16-bit copy of the state before the tile        [128 n, 64 p]
//           TMEM state rescaled by the tile's decay
//   MMA g1  scores = Q' K'^T   -> TMEM [64 x 64]  f32   (M = 64)
//           S^T   += K'^T V    -> TMEM [128 x 64] f32   (M = 128, A and B MN-major)
//           inter  = Q' St     -> TMEM [64 x 64]  f32   (B operand MN-major)
//   W       = causal mask of the scores (gamma/scale on same-token pairs, D on the diagonal,
//             exact per-element decay on unfactorised tiles), 16-bit -> smem, K-major
//   MMA g2  intra = W V        -> TMEM [64 x 64]  f32
//   epilogue y = e^{cmid} inter + intra, SiLU(z mz) gate, mimo_out rank sum -> global
//
// Long sequences with few (batch, head) pairs are split into segments: a state-only pass per
// segment, an FP32 scan over the segment records (seg_combine_kernel), then the main pass with
// every segment started from its true initial state.
//
// All operand tiles use the 128-byte swizzled canonical layout: a tile of `rows` x `cols`
// 16-bit elements is stored as cols/64 column blocks of rows x 128 B; inside a block, row r,
// 16-byte chunk c lives at r*128 + ((c ^ (r & 7)) * 16). The same bytes serve as a K-major
// operand ([MN rows][K cols]) or as an MN-major one ([K rows][MN cols]).
//
// Synchronisation: mbarriers track the TMA loads and tcgen05.commit of each MMA group; every wait
// is bounded by %globaltimer (2 s) and sets the library's device error word instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <initializer_list>
#include <mutex>

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
// cycles accumulate in registers and are added to g_section_cycles once, at the end
#define M3_MARK(k)                                            \
  do {                                                        \
    const long long now_ = clock64();                         \
    mark_acc_[k] += (unsigned int)(now_ - mark_prev_);        \
    mark_prev_ = now_;                                        \
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
constexpr int kSEcum = 0, kSEdec = 64, kSDiag = 128, kSCumL2 = 192, kSFq = 256, kSFk = 320, kSMode = 384,
              kSRaw = 400, kSEnd = 400 + 3 * 68;
// Workspace floats per token: RMS factors of the q rows (R), of the k rows (R), then, from the next
// 16-byte boundary, pi*tanh(angle) (S); padded to a multiple of 4 so each token's row is a run of
// 16-byte chunks. Inside the kernel the angle slots are overwritten by the packed (cos, sin) words
// of the tile's phases.
__host__ __device__ constexpr int ws_ang(int R) { return ((2 * R + 3) / 4) * 4; }
__host__ __device__ constexpr int ws_stride(int R, int S) { return ws_ang(R) + ((S + 3) / 4) * 4; }
template <int R> struct Layout {
  static constexpr int TOK = kRows / R;
  static constexpr int WSP = ws_stride(R, kMaxAngles);
  // CBq/CBk: packed bias words [R][64]; CMx/CMo: MIMO projections (float) [R][64]; CMz: mz packed
  // [R][32] (in the first half of its slot); CMxp: CMx packed [R][32]
  static constexpr int CBq = kSEnd, CBk = CBq + R * kN, CMx = CBk + R * kN, CMz = CMx + R * kP, CMo = CMz + R * kP;
  static constexpr int CMxp = CMo + R * kP;
  static_assert(CMz % 4 == 0 && CMo % 4 == 0, "16-byte aligned MIMO parameter rows");
  static constexpr int CWq = CMxp + R * kP / 2, CWk = CWq + kN / 2;   // packed norm weights [64]
  static constexpr int Ws = ((CWk + kN / 2 + 31) / 32) * 32;  // tile's workspace rows [TOK][WSP] (128 B)
  static constexpr int FEnd = Ws + TOK * WSP;
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

// Descriptor of the same tile `bytes` further on: the start-address field holds address / 16 in its
// low 14 bits, and shared-memory addresses stay below 256 KB, so the field never carries over.
__device__ __forceinline__ uint64_t sdesc_at(uint64_t d, uint32_t bytes) { return d + (uint64_t)(bytes >> 4); }

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

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Tiled TMA loads (no multicast) completing on an mbarrier; coordinates innermost first.
__device__ __forceinline__ void tma_load5(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load4(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load3(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Tensor maps of the row tiles: q/k [N, R, G, L, B] and x/z [P, H, L, B] (16-bit, 128-byte swizzle,
// boxes of 64 columns x one tile of rows), workspace rows [WS, L, B] (float, no swizzle).
struct alignas(64) TileMaps {
  CUtensorMap q, k, x, z, ws;
};

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

// Packed two-element arithmetic on 32-bit words holding two 16-bit values of type T.
template <typename T> struct Pk;
template <> struct Pk<__nv_bfloat16> { using v2 = __nv_bfloat162; };
template <> struct Pk<__half> { using v2 = __half2; };
template <typename T> __device__ __forceinline__ typename Pk<T>::v2 as2(uint32_t w) {
  return *reinterpret_cast<const typename Pk<T>::v2*>(&w);
}
template <typename T> __device__ __forceinline__ uint32_t asw(typename Pk<T>::v2 v) {
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <typename T> __device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
  return asw<T>(__hmul2(as2<T>(a), as2<T>(b)));
}
template <typename T> __device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
  return asw<T>(__hadd2(as2<T>(a), as2<T>(b)));
}
template <typename T> __device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
  return asw<T>(__hfma2(as2<T>(a), as2<T>(b), as2<T>(c)));
}
template <typename T> __device__ __forceinline__ uint32_t bcast2(float f) { return pack2<T>(f, f); }
// silu of both halves: z sigmoid(z) = h + h tanh(h) with h = z / 2 (hardware tanh approximation).
template <typename T> __device__ __forceinline__ uint32_t silu2(uint32_t z);
template <> __device__ __forceinline__ uint32_t silu2<__nv_bfloat16>(uint32_t z) {
  const uint32_t h = mul2<__nv_bfloat16>(z, 0x3F003F00u);  // 0.5 in both bf16 halves
  uint32_t t;
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(t) : "r"(h));
  return fma2<__nv_bfloat16>(h, t, h);
}
template <> __device__ __forceinline__ uint32_t silu2<__half>(uint32_t z) {
  const uint32_t h = mul2<__half>(z, 0x38003800u);  // 0.5 in both fp16 halves
  uint32_t t;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(t) : "r"(h));
  return fma2<__half>(h, t, h);
}
// Rotation of the pair (a0, a1) held in one word by the angle whose (cos, sin) word is cs:
// (a0 c - a1 s, a0 s + a1 c) = a * (c, c) + swap(a) * (-s, s).
template <typename T> __device__ __forceinline__ uint32_t rot_pair(uint32_t a, uint32_t cc, uint32_t ms) {
  return fma2<T>(__byte_perm(a, 0, 0x1032), ms, mul2<T>(a, cc));
}

// 16 TMEM columns of 16 lanes, twice: threads 0-15 read lanes base + t at column c, threads 16-31
// the same lanes at column c + 16 (the row layout of an M = 64 accumulator, all 32 threads busy).
#define M3_TMEM_LD16X2(taddr, r)                                                                              \
  asm volatile(                                                                                               \
      "tcgen05.ld.sync.aligned.16x32bx2.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15},"    \
      " [%16], 16;"                                                                                           \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),       \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])    \
      : "r"(taddr))

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
      o[ws_ang(R) + sidx] = kPi * tanhf(ld_t(a.angles, b * a.angles.stride[0] + (int64_t)t * a.angles.stride[1] +
                                                 sidx * a.angles.stride[2]));
  }
}

// Sequence segments. A long sequence with few (batch, head) pairs is split into segments of
// seg_len tokens (a multiple of 64, so the 64-token phase blocks line up), each scanned by its own
// CTA as a continuation of the previous one (the exact prefill -> continue semantics: the segment
// end acts as a sequence end, and the next segment folds the endpoint term of the boundary token
// through its initial k / value). Three launches: the state pass (kStateOnly) runs every segment but
// the last from a zero state and zero phase and records its end state, last phase, last rotated k,
// total decay and first-token endpoint weight; seg_combine_kernel scans those records over the
// segments in FP32 (rotating each local state and k by the true starting phase) into each
// segment's initial cache; the main pass then runs every segment from its initial cache.
// Per (segment, batch, head) record of floats: state [P][N], phase [32], k [R][N], c0, total decay.
__host__ __device__ constexpr int seg_rec(int R) { return kP * kN + kMaxAngles + R * kN + 4; }
constexpr int kRecPhase = kP * kN, kRecK = kP * kN + kMaxAngles;
__host__ __device__ constexpr int rec_c0(int R) { return kRecK + R * kN; }
struct SegArgs {
  int seg_len;   // tokens per segment (the whole sequence when nseg == 1)
  int nseg;
  int nblk;      // 64-token phase blocks per segment (seg_len / 64)
  float* part;   // state-pass records [nseg][B][H][seg_rec(R)]
  float* init;   // initial caches of the main pass [nseg][B][H][seg_rec(R)] (slot 0 unused)
  float* blk;    // state pass: in-block phase totals [nseg][B][H][nblk][32]
};

// softplus (torch threshold 20) and sigmoid of the per-token scalars with the hardware exp2/log2
// approximations (relative error ~1e-6, far below the 16-bit rounding of every operand the kernel
// stages); log(1 + e) is taken as e (1 - e / 2) below e = 1e-3, where 1 + e would round away e.
__device__ __forceinline__ float softplus_fast(float x) {
  if (x > 20.0f) return x;
  const float e = __expf(x);
  return e < 1e-3f ? e * (1.0f - 0.5f * e) : __logf(1.0f + e);
}
__device__ __forceinline__ float sigmoid_fast(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// x - 2pi * trunc(x / 2pi): the remainder of fmod (exact for |x| < 2pi, a few ulp beyond).
__device__ __forceinline__ float fmod_2pi(float x) { return x - kTwoPi * truncf(x * (1.0f / kTwoPi)); }

template <typename T, int R, bool kStateOnly>
__global__ void __launch_bounds__(kThreads, 2)
    scan_umma_kernel(const m3_scan_args a, const __grid_constant__ TileMaps tm, int vec_y, const SegArgs sg) {
  using Lay = Layout<R>;
  constexpr int TOK = Lay::TOK;
  constexpr bool kBf16 = DType<T>::id == M3_BF16;
  // Largest |cum - cmid| for which the decay can be split into per-row operand factors
  // e^{cum_i - cmid} (Q rows) and e^{cmid - cum_j} (K rows) without leaving the 16-bit range.
  constexpr float kLim = kBf16 ? 80.0f : 8.0f;
  // a.reverse == 2: both directions of a (batch, head) are adjacent CTAs (blockIdx.x = 2 h + dir),
  // so they are resident together and the second reader of a projection row can hit L2.
  const int h = a.reverse == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x, b = blockIdx.y;
  const int seg = a.reverse == 2 ? 0 : blockIdx.z;
  // This CTA's segment [seg_begin, L) in scan order; its end acts as the sequence end.
  const int seg_begin = seg * sg.seg_len;
  const int L = min(a.length, seg_begin + sg.seg_len);
  const bool last_seg = L == a.length;
  const int S = a.num_angles;
  const int g = h / (a.heads / a.groups);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quad = warp & 3, part = warp >> 2;  // TMEM lane quadrant, column half
  const int WS = ws_stride(R, S);               // workspace floats per token
  constexpr int WA = ws_ang(R);                 // first angle slot of a workspace row

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* fsm = reinterpret_cast<float*>(smem + kOffF);
  float* ecum = fsm + kSEcum;
  float* edec = fsm + kSEdec;
  float* diag = fsm + kSDiag;
  float* cum_l2 = fsm + kSCumL2;
  float* fq = fsm + kSFq;
  float* fk = fsm + kSFk;
  float* mode = fsm + kSMode;  // [0] cmid, [1] cum_last, [2] factorised, [3] e^{cum_last}
  float* sraw = fsm + kSRaw;   // raw per-token dt, adt, sigma of the next tile [3][68]
  float* cst = fsm;
  float* wsb = fsm + Lay::Ws;  // the tile's workspace rows; the phase replaces pi*tanh in place
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Lay::OffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OffBar + 8);
  int* abort_flag = reinterpret_cast<int*>(smem + Lay::OffBar + 16);
  // Forward scans load their row tiles with TMA (three boxes groups per tile complete on tma_bar);
  // reverse scans, whose tiles run backwards through memory, use per-row asynchronous copies.
  const uint32_t tma_bar = smem_u32(smem + Lay::OffBar + 24);
  // MMA completion: bar_addr tracks the scores MMAs, bar_b the inter + state-update MMAs issued after
  // them, bar_c the intra MMAs; each completes one phase per tile.
  const uint32_t bar_b = smem_u32(smem + Lay::OffBar + 32);
  const uint32_t bar_c = smem_u32(smem + Lay::OffBar + 40);
  // Scan direction of this CTA: a.reverse = 1 scans tokens L-1 .. 0; a.reverse = 2 runs both
  // directions in one launch (blockIdx.x = 2 h + direction), so the two reads of a sequence's projections
  // fall close together in time and the second is served from L2.
  const bool rev = a.reverse == 1 || (a.reverse == 2 && (blockIdx.x & 1));
  auto tok = [&](int ts) { return rev ? a.length - 1 - ts : ts; };
  const bool use_tma = !rev;
  const uint32_t bar_addr = smem_u32(bar);
  const uint32_t sbase = smem_u32(smem);
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;
  // per-token workspace rows (RMS factors, pi tanh(angle)) exist exactly when the pre-pass runs
  const bool has_ws = a.q_norm_w.data != nullptr || a.angles.data != nullptr;
  const float* ws = static_cast<const float*>(a.workspace.data);

  const T* qp = static_cast<const T*>(a.q.data);
  const T* kp = static_cast<const T*>(a.k.data);
  const T* vp = static_cast<const T*>(a.value.data);
  const T* zp = static_cast<const T*>(a.gate.data);
  T* yp = static_cast<T*>(rev && a.reverse == 2 ? a.y_reverse.data : a.y.data);
  const float Dh = ld_t(a.D, h * a.D.stride[0]);
  // Row bases (the rows themselves are contiguous and 16-byte aligned: scan_umma_supported).
  const int64_t q_b0 = b * a.q.stride[0] + g * a.q.stride[2];
  const int64_t k_b0 = b * a.k.stride[0] + g * a.k.stride[2];
  const int64_t v_b0 = b * a.value.stride[0] + h * a.value.stride[2];
  const int64_t z_b0 = b * a.gate.stride[0] + h * a.gate.stride[2];
  const int64_t ws_b = (int64_t)b * a.length * WS;

  // ---- loads of a tile, issued one tile ahead (cp.async for rows; see the tile loop) ----
  // q/k rows go straight into the Q'/K' tiles (processed in place), raw x into the W tile, z into the
  // z tile of the tile's parity, workspace rows into wsb.
  auto issue_qk = [&](int t0n, int ntn) {
    if (use_tma) {
      if (tid == 0) {
        mbar_expect_tx(tma_bar, (kStateOnly ? 2u : 4u) * (kRows * 64 * 2));
        if (!kStateOnly) {  // the state pass needs only the k rows
          tma_load5(sbase + kOffQ, &tm.q, 0, 0, g, t0n, b, tma_bar);
          tma_load5(sbase + kOffQ + kRows * 128, &tm.q, 64, 0, g, t0n, b, tma_bar);
        }
        tma_load5(sbase + kOffK, &tm.k, 0, 0, g, t0n, b, tma_bar);
        tma_load5(sbase + kOffK + kRows * 128, &tm.k, 64, 0, g, t0n, b, tma_bar);
      }
      return;
    }
    constexpr int kQChunks = kRows * (kN / 8);
    for (int c = tid; c < kQChunks; c += kThreads) {
      const int row = c >> 4, c8 = c & 15;
      const int j = row / R, r = row % R;
      if (j < ntn) {
        const int t = tok(t0n + j);
        const uint32_t off = swz(row, c8 * 8, kRows);
        if (!kStateOnly)
          cp_async16(sbase + kOffQ + off, qp + q_b0 + (int64_t)t * a.q.stride[1] + r * a.q.stride[3] + c8 * 8);
        cp_async16(sbase + kOffK + off, kp + k_b0 + (int64_t)t * a.k.stride[1] + r * a.k.stride[3] + c8 * 8);
      }
    }
  };
  auto issue_x = [&](int t0n, int ntn) {
    if (use_tma) {
      if (tid == 0) {
        mbar_expect_tx(tma_bar, (uint32_t)(TOK * kP * 2));
        tma_load4(sbase + (R == 1 ? kOffV : kOffW), &tm.x, 0, h, t0n, b, tma_bar);
      }
      return;
    }
    for (int c = tid; c < TOK * (kP / 8); c += kThreads) {
      const int j = c >> 3, c8 = c & 7;
      if (j < ntn) {
        const int t = tok(t0n + j);
        cp_async16(sbase + (R == 1 ? kOffV : kOffW) + swz(j, c8 * 8, kRows),
                   vp + v_b0 + (int64_t)t * a.value.stride[1] + c8 * 8);
      }
    }
  };
  auto issue_z = [&](int t0n, int ntn, int par) {
    const uint32_t zoff = kOffZ + par * (kRows * kP * 2);
    if (use_tma) {  // the z rows and (with a workspace) the workspace rows of the tile
      if (tid == 0) {  // (the state pass needs no z rows)
        mbar_expect_tx(tma_bar, (kStateOnly ? 0u : (uint32_t)(TOK * kP * 2)) + (has_ws ? (uint32_t)(TOK * WS * 4) : 0u));
        if (!kStateOnly) tma_load4(sbase + zoff, &tm.z, 0, h, t0n, b, tma_bar);
        if (has_ws) tma_load3(smem_u32(wsb), &tm.ws, 0, t0n, b, tma_bar);
      }
      return;
    }
    if constexpr (!kStateOnly) {
      for (int c = tid; c < TOK * (kP / 8); c += kThreads) {
        const int j = c >> 3, c8 = c & 7;
        if (j < ntn) {
          const int t = tok(t0n + j);
          cp_async16(sbase + zoff + swz(j, c8 * 8, kRows), zp + z_b0 + (int64_t)t * a.gate.stride[1] + c8 * 8);
        }
      }
    }
  };
  // Per-token scalars of a tile: thread j <= TOK fetches the dt and decay words of token j (j == TOK:
  // the first token after the tile) and thread 128 + j its trapezoid logit, into registers without
  // using them, so the loads stay in flight; finish_scalars() converts them (softplus / heavy-tail on
  // threads 0 .., sigmoid on threads 128 ..) into sraw later.
  uint32_t raw_dt = 0, raw_adt = 0, raw_trap = 0;
  bool raw_ok = false;
  const int jt = tid >= 128 ? tid - 128 : tid;  // token of this thread's raw scalar
  const bool trap_thread = tid >= 128;
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
    if (jt <= TOK && t0n + jt < L && (jt < ntn || jt == TOK)) {
      const int t = tok(t0n + jt);
      if (trap_thread) {
        raw_trap = raw_word(a.trap, b * a.trap.stride[0] + (int64_t)t * a.trap.stride[1] + h * a.trap.stride[2]);
      } else {
        raw_dt = raw_word(a.dt, b * a.dt.stride[0] + (int64_t)t * a.dt.stride[1] + h * a.dt.stride[2]);
        raw_adt = raw_word(a.adt, b * a.adt.stride[0] + (int64_t)t * a.adt.stride[1] + h * a.adt.stride[2]);
      }
      raw_ok = true;
    }
  };
  const float dt_bias_h = a.dt_bias.data ? ld_t(a.dt_bias, h * a.dt_bias.stride[0]) : 0.0f;
  auto finish_scalars = [&]() {
    if (jt <= TOK && trap_thread) {
      sraw[136 + jt] = raw_ok ? sigmoid_fast(word_to_f(raw_trap, a.trap.dtype)) : 0.0f;
    } else if (jt <= TOK) {
      float dtv = 0.0f, adtv = 0.0f;
      if (raw_ok) {
        if (a.dt_bias.data) {
          // mamba3/model.py:195-198: dt = softplus(delta + dt_bias); A = -heavytail(a) clamped <= -1e-4.
          dtv = softplus_fast(word_to_f(raw_dt, a.dt.dtype) + dt_bias_h);
          adtv = fminf(-heavy_tailf(word_to_f(raw_adt, a.adt.dtype)), -kAFloor) * dtv;
        } else {
          dtv = word_to_f(raw_dt, a.dt.dtype);
          adtv = word_to_f(raw_adt, a.adt.dtype);
        }
      }
      sraw[jt] = dtv;
      sraw[68 + jt] = adtv;
    }
  };
  // Workspace rows (cp.async) or their stand-ins, and the phase tensor of the op-level API.
  auto fetch_small = [&](int t0n, int ntn) {
    if (has_ws && use_tma) {
      // the workspace rows travel with the z rows (issue_z)
    } else if (has_ws) {
      const int chunks = WS / 4;  // <= 12: one 16-slot row per token, no division
      for (int c = tid; c < TOK * 16; c += kThreads) {
        const int j = c >> 4, c4 = c & 15;
        if (j < ntn && c4 < chunks) {
          const int t = tok(t0n + j);
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
          const int t = tok(t0n + j);
          v = ld_t(a.phase, b * a.phase.stride[0] + (int64_t)t * a.phase.stride[1] + h * a.phase.stride[2] +
                                sidx * a.phase.stride[3]);
        }
        wsb[j * WS + WA + sidx] = v;
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
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_b));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_c));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 3;" ::"r"(tma_bar));  // q/k, x, z (+ workspace)
    asm volatile("fence.mbarrier_init.release.cluster;");
    *abort_flag = 0;
  }
  uint32_t* cbq = reinterpret_cast<uint32_t*>(cst + Lay::CBq);  // packed bias words [R][64]
  uint32_t* cbk = reinterpret_cast<uint32_t*>(cst + Lay::CBk);
  uint32_t* cwq = reinterpret_cast<uint32_t*>(cst + Lay::CWq);  // packed norm weights [64]
  uint32_t* cwk = reinterpret_cast<uint32_t*>(cst + Lay::CWk);
  for (int i = tid; i < kN / 2; i += kThreads) {
    const bool nw = a.q_norm_w.data != nullptr;
    cwq[i] = nw ? pack2<T>(ld_t(a.q_norm_w, 2 * i * a.q_norm_w.stride[0]), ld_t(a.q_norm_w, (2 * i + 1) * a.q_norm_w.stride[0]))
                : 0u;
    cwk[i] = nw ? pack2<T>(ld_t(a.k_norm_w, 2 * i * a.k_norm_w.stride[0]), ld_t(a.k_norm_w, (2 * i + 1) * a.k_norm_w.stride[0]))
                : 0u;
  }
  for (int i = tid; i < R * kN / 2; i += kThreads) {
    const int r = i / (kN / 2), n = 2 * (i % (kN / 2));
    float bq[2] = {0.0f, 0.0f}, bk[2] = {0.0f, 0.0f};
    if (a.q_bias.data) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        bq[u] = ld_t(a.q_bias, h * a.q_bias.stride[0] + r * a.q_bias.stride[1] + (n + u) * a.q_bias.stride[2]);
        bk[u] = ld_t(a.k_bias, h * a.k_bias.stride[0] + r * a.k_bias.stride[1] + (n + u) * a.k_bias.stride[2]);
      }
    }
    cbq[i] = pack2<T>(bq[0], bq[1]);
    cbk[i] = pack2<T>(bk[0], bk[1]);
  }
  if (R > 1) {
    for (int i = tid; i < R * kP; i += kThreads) {
      const int r = i / kP, p = i % kP;
      cst[Lay::CMx + i] = ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] + p * a.mimo_x.stride[2]);
      cst[Lay::CMo + i] =
          ld_t(a.mimo_out, h * a.mimo_out.stride[0] + r * a.mimo_out.stride[1] + p * a.mimo_out.stride[2]);
    }
    // mz packed [R][32]: the gate product z mz is rounded to the activation dtype, as the reference's
    // `gate * mimo_z.to(gate.dtype)` is.
    uint32_t* cmzp = reinterpret_cast<uint32_t*>(cst + Lay::CMz);
    for (int i = tid; i < R * kP / 2; i += kThreads) {
      const int r = i / (kP / 2), p = 2 * (i % (kP / 2));
      const m3_tensor& mz = a.mimo_z;
      cmzp[i] = pack2<T>(ld_t(mz, h * mz.stride[0] + r * mz.stride[1] + p * mz.stride[2]),
                         ld_t(mz, h * mz.stride[0] + r * mz.stride[1] + (p + 1) * mz.stride[2]));
    }
    uint32_t* cmxp = reinterpret_cast<uint32_t*>(cst + Lay::CMxp);
    for (int i = tid; i < R * kP / 2; i += kThreads) {
      const int r = i / (kP / 2), p = 2 * (i % (kP / 2));
      const m3_tensor& mx = a.mimo_x;
      cmxp[i] = pack2<T>(ld_t(mx, h * mx.stride[0] + r * mx.stride[1] + p * mx.stride[2]),
                         ld_t(mx, h * mx.stride[0] + r * mx.stride[1] + (p + 1) * mx.stride[2]));
    }
  }
  const bool has_norm = a.q_norm_w.data != nullptr;
  const bool has_bias = a.q_bias.data != nullptr;
  // Initial cache of this segment: the caller's for the first segment; for later segments of the
  // main pass the combined records (state, last phase, rotated k of the token before the segment)
  // and that token's value row; nothing (zero state, zero phase) for later segments of the state pass.
  m3_tensor ist = a.initial_state, ikt = a.initial_k, ivt = a.initial_value, iph = a.initial_phase;
  if (seg > 0) {
    ist = ikt = ivt = iph = m3_tensor{};
    if (!kStateOnly) {
      constexpr int REC = seg_rec(R);
      float* rec = sg.init + (int64_t)seg * a.batch * a.heads * REC;
      const int64_t sb = (int64_t)a.heads * REC;
      ist = m3_tensor{rec, M3_F32, 4, {sb, REC, kN, 1, 0, 0}};
      iph = m3_tensor{rec + kRecPhase, M3_F32, 3, {sb, REC, 1, 0, 0, 0}};
      ikt = m3_tensor{rec + kRecK, M3_F32, 4, {sb, REC, kN, 1, 0, 0}};
      const int tprev = tok(seg_begin - 1);
      ivt = m3_tensor{const_cast<T*>(vp) + (int64_t)tprev * a.value.stride[1], a.value.dtype, 3,
                      {a.value.stride[0], a.value.stride[2], a.value.stride[3], 0, 0, 0}};
    }
  }
  // Loads of the first tile.
  {
    const int nt0 = min(TOK, L - seg_begin);
    issue_qk(seg_begin, nt0);
    issue_x(seg_begin, nt0);
    issue_z(seg_begin, nt0, 0);
    fetch_small(seg_begin, nt0);
    fetch_scalars(seg_begin, nt0);
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
    if (ikt.data || kStateOnly) {
      float dt0, adt0;
      const int t_first = tok(seg_begin);
      load_dt_adt(a, b, t_first, h, dt0, adt0);
      c0 = dt0 * (1.0f - sigmoidf_(load_trap(a, b, t_first, h)));
      // the state pass records the endpoint weight of its first token for the combine
      if (kStateOnly && tid == 0)
        sg.part[((int64_t)(seg * a.batch + b) * a.heads + h) * seg_rec(R) + rec_c0(R)] = c0;
    }
    const int n = quad * 32 + lane;
    uint32_t r32[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int p = part * 32 + j;
      float s = 0.0f;
      if (ist.data) {
        const m3_tensor& t = ist;
        s = ld_t(t, b * t.stride[0] + h * t.stride[1] + p * t.stride[2] + n * t.stride[3]);
      }
      if (ikt.data) {
        const m3_tensor& ik = ikt;
        const m3_tensor& iv = ivt;
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
  unsigned int mark_acc_[16];
  for (int k_ = 0; k_ < 16; ++k_) mark_acc_[k_] = 0;
#endif

  // Phase carry of this warp's angles (block offset, in-block sum). Rank 1 (64 tokens per tile): every
  // warp owns kPhA = 4 angles, s0 = 4 warp. Rank > 1 (at most 32 tokens, so a warp's scans are short):
  // warps 1 .. 6 own 6 angles each, s0 = 6 (warp - 1) (36 slots >= kMaxAngles), and warp 0, which
  // computes the per-token scalars meanwhile, has none (nor has warp 7).
  constexpr int kPhA = R == 1 ? 4 : 6;
  static_assert((R == 1 ? kWarps : 6) * kPhA >= kMaxAngles && kPhA % 2 == 0,
                "phase warps must cover every angle in pairs");
  const int ph_s0 = R == 1 ? kPhA * warp : ((warp >= 1 && warp <= 6) ? kPhA * (warp - 1) : kMaxAngles);
  float ph_off[kPhA], ph_loc[kPhA];
#pragma unroll
  for (int k = 0; k < kPhA; ++k) {
    const int sidx = ph_s0 + k;
    ph_off[k] = (iph.data && sidx < S)
                    ? ld_t(iph, b * iph.stride[0] + h * iph.stride[1] + sidx * iph.stride[2])
                    : 0.0f;
    ph_loc[k] = 0.0f;
  }
  uint32_t tma_phase = 0;
  int tile = 0;
  float decay_sum = 0.0f;  // state pass: total log-decay of the segment
  // the state pass's record of this (segment, batch, head)
  float* const prec = kStateOnly ? sg.part + ((int64_t)(seg * a.batch + b) * a.heads + h) * seg_rec(R) : nullptr;
  for (int t0 = seg_begin; t0 < L; t0 += TOK, ++tile) {
    const int nt = min(TOK, L - t0);
    const int t0n = t0 + TOK, ntn = min(TOK, L - t0n);  // next tile (ntn <= 0: none)
    M3_MARK(0);
    cp_async_wait_all();  // this tile's rows, workspace rows (issued during the previous tile)
    if (use_tma) {
      if (tid == 0 && !mbar_wait(tma_bar, tma_phase)) *abort_flag = 1;
      tma_phase ^= 1;
    }
    __syncthreads();
    M3_MARK(1);

    // ---- warp 0: per-token scalars (mamba3/ops.py:659-671) of tokens 2 lane, 2 lane + 1: cumulative
    // decay, trapezoid scale, decay factorisation; all in registers and shuffles ----
    if (warp == 0) {
      const int j0 = 2 * lane;
      float dtv[2], adv[2], sgv[2];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const bool v = j0 + m < nt;
        dtv[m] = v ? sraw[j0 + m] : 0.0f;
        adv[m] = v ? sraw[68 + j0 + m] : 0.0f;
        sgv[m] = v ? sraw[136 + j0 + m] : 0.0f;
      }
      const float incl = warp_incl_scan(adv[0] + adv[1], lane);
      const float cum2[2] = {incl - adv[1], incl};
      const int jm = (nt - 1) >> 1, jl = nt - 1;
      const float cmid = __shfl_sync(0xffffffffu, (jm & 1) ? cum2[1] : cum2[0], jm >> 1);
      const float cl = __shfl_sync(0xffffffffu, (jl & 1) ? cum2[1] : cum2[0], jl >> 1);
      // scale_j = gamma_j + dt_{j+1} (1 - sigma_{j+1}); the last token looks at the first one after the tile
      const float beta_up = __shfl_down_sync(0xffffffffu, dtv[0] * (1.0f - sgv[0]), 1);
      const float beta_next = (nt == TOK && t0 + TOK < L) ? sraw[TOK] * (1.0f - sraw[136 + TOK]) : 0.0f;
      const float nx[2] = {j0 + 1 < nt ? dtv[1] * (1.0f - sgv[1]) : 0.0f,
                           j0 + 2 < nt ? beta_up : ((j0 + 2 == TOK && nt == TOK) ? beta_next : 0.0f)};
      float scv[2], dg[2], dev = 0.0f;
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const bool v = j0 + m < nt;
        const float gamma = dtv[m] * sgv[m];
        scv[m] = v ? gamma + nx[m] : 0.0f;
        dg[m] = v ? gamma / scv[m] : 0.0f;
        if (v) dev = fmaxf(dev, fabsf(cum2[m] - cmid));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dev = fmaxf(dev, __shfl_xor_sync(0xffffffffu, dev, o));
      const bool fct = dev <= kLim;
      if (j0 < TOK) {
        float o_fq[2], o_fk[2], o_ec[2], o_ed[2];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const bool v = j0 + m < nt;
          const float c = cum2[m];
          o_fq[m] = v ? (fct ? __expf(c - cmid) : 1.0f) : 0.0f;
          o_fk[m] = v ? (fct ? scv[m] * __expf(cmid - c) : scv[m]) : 0.0f;
          o_ec[m] = v ? (fct ? __expf(cmid) : __expf(c)) : 0.0f;
          o_ed[m] = (v && !fct) ? __expf(cl - c) : 0.0f;
        }
        *reinterpret_cast<float2*>(cum_l2 + j0) = make_float2(cum2[0] * kLog2e, cum2[1] * kLog2e);
        *reinterpret_cast<float2*>(diag + j0) = make_float2(dg[0], dg[1]);
        *reinterpret_cast<float2*>(fq + j0) = make_float2(o_fq[0], o_fq[1]);
        *reinterpret_cast<float2*>(fk + j0) = make_float2(o_fk[0], o_fk[1]);
        *reinterpret_cast<float2*>(ecum + j0) = make_float2(o_ec[0], o_ec[1]);
        *reinterpret_cast<float2*>(edec + j0) = make_float2(o_ed[0], o_ed[1]);
      }
      if (lane == 0) {
        mode[0] = cmid;
        mode[1] = cl;
        mode[2] = fct ? 1.0f : 0.0f;
        mode[3] = __expf(cl);
      }
    }
    // No barrier: the phase section below reads only sraw (dt) and the workspace rows, so warps 1-7
    // start on their angles while warp 0 finishes the scalars; the barrier after the phases covers both.
    M3_MARK(2);
    // ---- phases -> packed (cos, sin) words over pi*tanh(angle) in wsb. A warp's angles s0 .. s0 + kPhA - 1
    // (carried block offset and in-block sum in registers,
    // mamba3/model.py:246-251); lane: tokens 2 lane, 2 lane + 1. SISO: word m = (cos_m, sin_m); MIMO
    // (S == 32): word q < 16 = (cos_2q, cos_2q+1), word 16 + q = (sin_2q, sin_2q+1), the element
    // pairs a staging word holds. ----
    if (has_phase) {
      const int s0 = ph_s0, j0 = 2 * lane;
      float ph[2][kPhA];
      if (s0 < S) {
        if (a.angles.data) {
          if (t0 > 0 && (t0 % kPhaseBlock) == 0) {
#pragma unroll
            for (int k = 0; k < kPhA; ++k) {
              ph_off[k] = fmodf(ph_off[k] + ph_loc[k], kTwoPi);
              ph_loc[k] = 0.0f;
            }
          }
          float inc[2][kPhA];
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int j = j0 + m;
            float in[kPhA] = {};
            float dtj = 0.0f;
            if (j < nt) {
              if constexpr (kPhA == 4) {  // s0 = 4 warp: one 16-byte load
                const float4 av = *reinterpret_cast<const float4*>(wsb + j * WS + WA + s0);
                in[0] = av.x;
                in[1] = av.y;
                in[2] = av.z;
                in[3] = av.w;
              } else {
#pragma unroll
                for (int k2 = 0; k2 < kPhA / 2; ++k2) {
                  const float2 av = *reinterpret_cast<const float2*>(wsb + j * WS + WA + s0 + 2 * k2);
                  in[2 * k2] = av.x;
                  in[2 * k2 + 1] = av.y;
                }
              }
              dtj = sraw[j];  // dt of token j (finish_scalars), not waiting for the scalar section
            }
#pragma unroll
            for (int k = 0; k < kPhA; ++k) inc[m][k] = s0 + k < S ? fmod_2pi(in[k] * dtj) : 0.0f;
          }
#pragma unroll
          for (int k = 0; k < kPhA; ++k) {
            const float x = warp_incl_scan(inc[0][k] + inc[1][k], lane);
            const float tot = __shfl_sync(0xffffffffu, x, 31);
            ph[0][k] = fmod_2pi((ph_loc[k] + (x - inc[1][k])) + ph_off[k]);
            ph[1][k] = fmod_2pi((ph_loc[k] + x) + ph_off[k]);
            ph_loc[k] += tot;
          }
          // The state pass records every completed 64-token block's in-block phase total, so the
          // combine can replay the exact block-offset carry (fmod at every block end) across it.
          if (kStateOnly && ((t0 + TOK) % kPhaseBlock) == 0 && lane == 0) {
            float* bp = sg.blk + (((int64_t)(seg * a.batch + b) * a.heads + h) * sg.nblk +
                                  (t0 + TOK - seg_begin) / kPhaseBlock - 1) * kMaxAngles;
#pragma unroll
            for (int k = 0; k < kPhA; ++k)
              if (s0 + k < S) bp[s0 + k] = ph_loc[k];
          }
        } else {
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int j = j0 + m;
#pragma unroll
            for (int k2 = 0; k2 < kPhA / 2; ++k2) {
              float2 pv = make_float2(0.0f, 0.0f);
              if (j < TOK) pv = *reinterpret_cast<const float2*>(wsb + j * WS + WA + s0 + 2 * k2);
              ph[m][2 * k2] = pv.x;
              ph[m][2 * k2 + 1] = pv.y;
            }
          }
        }
      }
      if (a.mimo_rotation) __syncthreads();  // MIMO words land on other warps' angle slots
      if (s0 < S) {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const int j = j0 + m;
          if (j < TOK) {
            float cs[kPhA], sn[kPhA];
#pragma unroll
            for (int k = 0; k < kPhA; ++k) __sincosf(ph[m][k], &sn[k], &cs[k]);  // |phase| < 2 pi
            if (!kStateOnly && t0 + j == L - 1 && last_seg && a.final_phase.data) {
              const m3_tensor& fp = a.final_phase;
#pragma unroll
              for (int k = 0; k < kPhA; ++k)
                if (s0 + k < S)
                  static_cast<float*>(fp.data)[b * fp.stride[0] + h * fp.stride[1] + (s0 + k) * fp.stride[2]] =
                      ph[m][k];
            }
            uint32_t* w = reinterpret_cast<uint32_t*>(wsb + j * WS + WA);
            if (a.mimo_rotation) {
#pragma unroll
              for (int k2 = 0; k2 < kPhA / 2; ++k2) {
                if (s0 + 2 * k2 < S) {
                  w[s0 / 2 + k2] = pack2<T>(cs[2 * k2], cs[2 * k2 + 1]);
                  w[16 + s0 / 2 + k2] = pack2<T>(sn[2 * k2], sn[2 * k2 + 1]);
                }
              }
            } else if (kPhA == 4 && s0 + 4 <= S) {
              *reinterpret_cast<uint4*>(w + s0) = make_uint4(pack2<T>(cs[0], sn[0]), pack2<T>(cs[1], sn[1]),
                                                             pack2<T>(cs[2], sn[2]), pack2<T>(cs[3], sn[3]));
            } else {
#pragma unroll
              for (int k2 = 0; k2 < kPhA / 2; ++k2) {
                const int sa = s0 + 2 * k2;
                if (sa + 1 < S) {
                  *reinterpret_cast<uint2*>(w + sa) =
                      make_uint2(pack2<T>(cs[2 * k2], sn[2 * k2]), pack2<T>(cs[2 * k2 + 1], sn[2 * k2 + 1]));
                } else if (sa < S) {
                  w[sa] = pack2<T>(cs[2 * k2], sn[2 * k2]);
                }
              }
            }
          }
        }
      }
    }
    __syncthreads();
    const bool fact = mode[2] != 0.0f;
    if (kStateOnly) decay_sum += mode[1];
    M3_MARK(3);

    // ---- stage Q', K' in place (packed 16-bit math): q' = rot(q rq w + b) fq, k' = rot(k rk w + b) fk.
    // Lane: row warp * 8 + 4 it + (lane >> 3), 16-byte chunks c = lane & 7 and c + 8 (elements 8 c ..,
    // 64 + 8 c ..), so the rotated chunks (the first S pairs; MIMO: n < 32 with n + 64) spread over all
    // lanes and a MIMO pair never leaves its lane. ----
    const uint32_t qko = kOffQ;
    const int c = lane & 7;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int row = warp * 8 + 4 * it + (lane >> 3);
      const int ts_ = row / R, r = row % R;
      const int j = ts_;
      const bool valid = j < nt;
      const float* wrow = wsb + ts_ * WS;
      const uint32_t off0 = qko + swz(row, 8 * c, kRows), off1 = qko + swz(row, 64 + 8 * c, kRows);
      uint32_t qv[8], kv[8];
      {
        // (the state pass loads no q rows: its Q' words are never stored, so their math folds away)
        const uint4 q0 = kStateOnly ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(smem + off0);
        const uint4 q1 = kStateOnly ? make_uint4(0, 0, 0, 0) : *reinterpret_cast<const uint4*>(smem + off1);
        const uint4 k0 = *reinterpret_cast<const uint4*>(smem + off0 + kRows * kN * 2);
        const uint4 k1 = *reinterpret_cast<const uint4*>(smem + off1 + kRows * kN * 2);
        qv[0] = q0.x; qv[1] = q0.y; qv[2] = q0.z; qv[3] = q0.w;
        qv[4] = q1.x; qv[5] = q1.y; qv[6] = q1.z; qv[7] = q1.w;
        kv[0] = k0.x; kv[1] = k0.y; kv[2] = k0.z; kv[3] = k0.w;
        kv[4] = k1.x; kv[5] = k1.y; kv[6] = k1.z; kv[7] = k1.w;
      }
      if (has_norm || has_bias) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int wo = 4 * c + 32 * hf;  // first packed word of this chunk
          const uint4 bq = *reinterpret_cast<const uint4*>(cbq + r * (kN / 2) + wo);
          const uint4 bk = *reinterpret_cast<const uint4*>(cbk + r * (kN / 2) + wo);
          const uint32_t bqa[4] = {bq.x, bq.y, bq.z, bq.w}, bka[4] = {bk.x, bk.y, bk.z, bk.w};
          if (has_norm) {
            const uint32_t rq2 = bcast2<T>(wrow[r]), rk2 = bcast2<T>(wrow[R + r]);
            const uint4 wq = *reinterpret_cast<const uint4*>(cwq + wo);
            const uint4 wk = *reinterpret_cast<const uint4*>(cwk + wo);
            const uint32_t wqa[4] = {wq.x, wq.y, wq.z, wq.w}, wka[4] = {wk.x, wk.y, wk.z, wk.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              qv[4 * hf + e] = fma2<T>(mul2<T>(qv[4 * hf + e], rq2), wqa[e], bqa[e]);
              kv[4 * hf + e] = fma2<T>(mul2<T>(kv[4 * hf + e], rk2), wka[e], bka[e]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              qv[4 * hf + e] = add2<T>(qv[4 * hf + e], bqa[e]);
              kv[4 * hf + e] = add2<T>(kv[4 * hf + e], bka[e]);
            }
          }
        }
      }
      if (has_phase) {
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(wrow + WA);
        if (a.mimo_rotation) {
          // pairs (n, n + 64) for n < 32: chunk c < 4 and chunk c + 8 of the same lane
          if (c < 4) {
            const uint4 c4 = *reinterpret_cast<const uint4*>(rw + 4 * c);
            const uint4 s4 = *reinterpret_cast<const uint4*>(rw + 16 + 4 * c);
            const uint32_t ca[4] = {c4.x, c4.y, c4.z, c4.w}, sa[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t ns = sa[e] ^ 0x80008000u;
              const uint32_t qa_ = qv[e], qb_ = qv[4 + e], ka_ = kv[e], kb_ = kv[4 + e];
              qv[e] = fma2<T>(qb_, ns, mul2<T>(qa_, ca[e]));         // a c - b s
              qv[4 + e] = fma2<T>(qa_, sa[e], mul2<T>(qb_, ca[e]));  // a s + b c
              kv[e] = fma2<T>(kb_, ns, mul2<T>(ka_, ca[e]));
              kv[4 + e] = fma2<T>(ka_, sa[e], mul2<T>(kb_, ca[e]));
            }
          }
        } else if (4 * c < S) {
          // adjacent pairs (2m, 2m + 1), m = 4 c + e, all in the first chunk
          const uint4 c4 = *reinterpret_cast<const uint4*>(rw + 4 * c);
          const uint32_t csa[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (4 * c + e < S) {
              const uint32_t cc = __byte_perm(csa[e], 0, 0x1010);
              const uint32_t ms = __byte_perm(csa[e], 0, 0x3232) ^ 0x00008000u;
              qv[e] = rot_pair<T>(qv[e], cc, ms);
              kv[e] = rot_pair<T>(kv[e], cc, ms);
            }
          }
        }
      }
      if (kStateOnly && valid && t0 + j == L - 1) {
        float* fkp = prec + kRecK + r * kN;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = (e < 4 ? 8 * c : 64 + 8 * c) + 2 * (e & 3);
          fkp[n] = lo16<T>(kv[e]);
          fkp[n + 1] = hi16<T>(kv[e]);
        }
      } else if (valid && last_seg && a.final_k.data && t0 + j == L - 1) {
        const m3_tensor& fkt = a.final_k;
        T* fkp = static_cast<T*>(fkt.data) + b * fkt.stride[0] + h * fkt.stride[1] + r * fkt.stride[2];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = (e < 4 ? 8 * c : 64 + 8 * c) + 2 * (e & 3);
          fkp[n * fkt.stride[3]] = from_f<T>(lo16<T>(kv[e]));
          fkp[(n + 1) * fkt.stride[3]] = from_f<T>(hi16<T>(kv[e]));
        }
      }
      // Rows outside the sequence (zero-filled by the TMA) would still carry the bias: zero them.
      const uint32_t fq2 = valid ? bcast2<T>(fq[j]) : 0u, fk2 = valid ? bcast2<T>(fk[j]) : 0u;
      if (!kStateOnly) {
        *reinterpret_cast<uint4*>(smem + off0) =
            make_uint4(mul2<T>(qv[0], fq2), mul2<T>(qv[1], fq2), mul2<T>(qv[2], fq2), mul2<T>(qv[3], fq2));
        *reinterpret_cast<uint4*>(smem + off1) =
            make_uint4(mul2<T>(qv[4], fq2), mul2<T>(qv[5], fq2), mul2<T>(qv[6], fq2), mul2<T>(qv[7], fq2));
      }
      *reinterpret_cast<uint4*>(smem + off0 + kRows * kN * 2) =
          make_uint4(mul2<T>(kv[0], fk2), mul2<T>(kv[1], fk2), mul2<T>(kv[2], fk2), mul2<T>(kv[3], fk2));
      *reinterpret_cast<uint4*>(smem + off1 + kRows * kN * 2) =
          make_uint4(mul2<T>(kv[4], fk2), mul2<T>(kv[5], fk2), mul2<T>(kv[6], fk2), mul2<T>(kv[7], fk2));
    }
    // ---- V = x mx_r: R = 1 keeps the x rows loaded into the V tile (rows past the end zeroed when they
    // came by row copies), R > 1 expands the x rows parked in the W tile. V2 = V e^{cum_last - cum} when
    // the tile is not factorised. 16-byte chunks: 64 rows x 8 chunks over 256 threads. ----
#pragma unroll
    for (int c = tid; c < kRows * (kP / 8); c += kThreads) {
      const int row = c >> 3, ch = c & 7;
      const int j = row / R, r = row % R;
      const int jc = min(j, TOK - 1);
      uint4 v4 = make_uint4(0, 0, 0, 0);
      if (R > 1) {
        if (j < nt) v4 = *reinterpret_cast<const uint4*>(smem + kOffW + swz(j, 8 * ch, kRows));
        const uint4 m4 = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const uint32_t*>(cst + Lay::CMxp) + r * (kP / 2) + 4 * ch);
        v4 = make_uint4(mul2<T>(v4.x, m4.x), mul2<T>(v4.y, m4.y), mul2<T>(v4.z, m4.z), mul2<T>(v4.w, m4.w));
        *reinterpret_cast<uint4*>(smem + kOffV + swz(row, 8 * ch, kRows)) = v4;
      } else if (j < nt) {
        if (!fact) v4 = *reinterpret_cast<const uint4*>(smem + kOffV + swz(row, 8 * ch, kRows));
      } else if (!use_tma) {
        *reinterpret_cast<uint4*>(smem + kOffV + swz(row, 8 * ch, kRows)) = v4;
      }
      if (!fact) {
        const uint32_t e2 = bcast2<T>(edec[jc]);
        *reinterpret_cast<uint4*>(smem + kOffV2 + swz(row, 8 * ch, kRows)) =
            make_uint4(mul2<T>(v4.x, e2), mul2<T>(v4.y, e2), mul2<T>(v4.z, e2), mul2<T>(v4.w, e2));
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
      if constexpr (!kStateOnly) {  // (the state pass has no inter-tile output term)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = pack2<T>(__uint_as_float(r32[c * 8 + 2 * i]) * phi, __uint_as_float(r32[c * 8 + 2 * i + 1]) * phi);
          *reinterpret_cast<uint4*>(smem + kOffST + swz(n, part * 32 + c * 8, kN)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
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

    // ---- MMA group 1, issued by two threads at once (one thread issues a tcgen05.mma every ~60
    // cycles; a second issuing warp doubles the rate). Thread 0: scores = Q' K'^T, committed on its own
    // so the W section starts as soon as they land. Thread 32: the state update X += K'^T V (or V2),
    // then inter = Q' St; both finish behind the W section. ----
    if (tid == 0 && !kStateOnly) {
      fence_after();
      const uint64_t dq = sdesc(sbase + kOffQ, 16, 1024), dk = sdesc(sbase + kOffK, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < kN / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColScores, sdesc_at(dq, koff), sdesc_at(dk, koff), id_scores, kk > 0);
      }
      mma_commit(bar_addr);
    }
    if (tid == 32) {
      fence_after();
      const uint64_t dkm = sdesc(sbase + kOffK, kRows * 128, 1024);
      const uint64_t dv = sdesc(sbase + (fact ? kOffV : kOffV2), kRows * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk)
        mma_f16(tmem + kColState, sdesc_at(dkm, kk * 2048), sdesc_at(dv, kk * 2048), id_state, 1);
      if (!kStateOnly) {
        const uint64_t dq = sdesc(sbase + kOffQ, 16, 1024), dst = sdesc(sbase + kOffST, kN * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
          mma_f16(tmem + kColInter, sdesc_at(dq, koff), sdesc_at(dst, kk * 2048), id_nmn, kk > 0);
        }
      }
      mma_commit(bar_b);
    }
    // While the tensor cores run: the next tile's scalars, workspace rows and z rows (other buffer).
    if (ntn > 0) {
      fetch_scalars(t0n, ntn);
      fetch_small(t0n, ntn);
      issue_z(t0n, ntn, (tile + 1) & 1);
    }
    if constexpr (kStateOnly) {
      // The state update is the state pass's only MMA; once it has read K' and V the next tile's rows
      // can land.
      if (tid == 0 && !mbar_wait(bar_b, phase_bit)) *abort_flag = 1;
      phase_bit ^= 1;
      __syncthreads();
      fence_after();
      if (ntn > 0) {
        issue_qk(t0n, ntn);
        issue_x(t0n, ntn);
      }
      cp_async_commit();
      if (ntn > 0) finish_scalars();
      fence_before();
      __syncthreads();
      if (*abort_flag) break;
      continue;
    }
    // One thread polls the barrier; the others wait at __syncthreads without taking issue slots.
    if (tid == 0 && !mbar_wait(bar_addr, phase_bit)) *abort_flag = 1;
    __syncthreads();
    fence_after();
    M3_MARK(6);

    // ---- W = scores o decay -> smem (16-bit, K-major). Thread: row quad * 16 + (lane & 15), columns
    // c0 .. c0 + 15 with c0 = part * 32 + (lane >> 4) * 16. ----
    {
      const int i = quad * 16 + (lane & 15);
      const int ti = min(i / R, TOK - 1);
      const int c0 = part * 32 + (lane >> 4) * 16;
      const bool all_masked = (part * 32) / R > (quad * 16 + 15) / R;  // warp-uniform
      uint4 w0 = make_uint4(0, 0, 0, 0), w1 = make_uint4(0, 0, 0, 0);
      if (!all_masked) {
        uint32_t r16[16];
        M3_TMEM_LD16X2(tmem + lane_base + kColScores + part * 32, r16);
        tmem_wait_ld();
        const float di = diag[ti];
        const float ci = cum_l2[ti];
        // Branch-free: below the row token's block the score (times the exact decay when the tile is not
        // factorised), on it gamma / scale (plus D on the diagonal itself: the D v term), above it 0.
        float f[16];
        if (fact) {
#pragma unroll
          for (int k = 0; k < 16; ++k) f[k] = 1.0f;
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) f[k] = ex2_approx(ci - cum_l2[(c0 + k) / R]);
        }
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float vals[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = c0 + 2 * e + u, tk = col / R, ti_ = i / R;
            const float sv = __uint_as_float(r16[2 * e + u]);
            const float same = fmaf(sv, di, col == i ? Dh : 0.0f);
            vals[u] = tk < ti_ ? sv * f[2 * e + u] : (tk == ti_ ? same : 0.0f);
          }
          w[e] = pack2<T>(vals[0], vals[1]);
        }
        w0 = make_uint4(w[0], w[1], w[2], w[3]);
        w1 = make_uint4(w[4], w[5], w[6], w[7]);
      }
      *reinterpret_cast<uint4*>(smem + kOffW + swz(i, c0, kRows)) = w0;
      *reinterpret_cast<uint4*>(smem + kOffW + swz(i, c0 + 8, kRows)) = w1;
    }
    fence_async_smem();
    fence_before();
    __syncthreads();
    M3_MARK(7);

    // ---- MMA group 2: intra = W V ----
    if (tid == 0) {
      fence_after();
      const uint64_t dw = sdesc(sbase + kOffW, 16, 1024), dv = sdesc(sbase + kOffV, kRows * 128, 1024);
#pragma unroll
      for (int kk = 0; kk < kRows / 16; ++kk) {
        const uint32_t koff = (kk >> 2) * (kRows * 128) + (kk & 3) * 32;
        mma_f16(tmem + kColIntra, sdesc_at(dw, koff), sdesc_at(dv, kk * 2048), id_nmn, kk > 0);
      }
      mma_commit(bar_c);
    }
    // the state update and inter (bar_b) and scores (with bar_c) have finished: Q'/K' are free, so the
    // next tile's raw q/k rows can start.
    if (tid == 0 && !mbar_wait(bar_b, phase_bit)) *abort_flag = 1;
    if (use_tma) {
      if (ntn > 0) issue_qk(t0n, ntn);  // one thread issues the TMA boxes; the others skip
    }
    if (tid == 0 && !mbar_wait(bar_c, phase_bit)) *abort_flag = 1;
    phase_bit ^= 1;
    __syncthreads();
    fence_after();
    // Row copies of the next tile's q/k (reverse scans) need every thread, after the barrier.
    if (!use_tma && ntn > 0) issue_qk(t0n, ntn);
    // W and V are free now: the next tile's raw x rows.
    if (ntn > 0) issue_x(t0n, ntn);
    cp_async_commit();
    M3_MARK(8);

    // ---- epilogue: thread row quad * 16 + (lane & 15), output columns p0 .. p0 + 15 ----
    {
      const int i = quad * 16 + (lane & 15);
      const int ti = i / R, r = i % R;
      const int tc = min(ti, TOK - 1);
      const int p0 = part * 32 + (lane >> 4) * 16;
      const uint32_t zoff = kOffZ + (tile & 1) * (kRows * kP * 2);
      uint32_t ra[16], ri[16];
      M3_TMEM_LD16X2(tmem + lane_base + kColIntra + part * 32, ra);
      M3_TMEM_LD16X2(tmem + lane_base + kColInter + part * 32, ri);
      tmem_wait_ld();
      const bool valid = ti < nt;
      const float gi = ecum[tc];
      float out[16];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 zz = *reinterpret_cast<const uint4*>(smem + zoff + swz(tc, p0 + 8 * c, kRows));
        const uint32_t zw[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int jj = 8 * c + 2 * e;
          // D v arrives through the diagonal of W (intra)
          const float y0 = fmaf(gi, __uint_as_float(ri[jj]), __uint_as_float(ra[jj]));
          const float y1 = fmaf(gi, __uint_as_float(ri[jj + 1]), __uint_as_float(ra[jj + 1]));
          if (R == 1) {
            const float2 g = unpack2<T>(silu2<T>(zw[e]));
            out[jj] = y0 * g.x;
            out[jj + 1] = y1 * g.y;
          } else {
            const uint32_t mzw = reinterpret_cast<const uint32_t*>(cst + Lay::CMz)[r * (kP / 2) + (p0 + jj) / 2];
            const float2 g = unpack2<T>(silu2<T>(mul2<T>(zw[e], mzw)));
            out[jj] = y0 * g.x;
            out[jj + 1] = y1 * g.y;
          }
        }
      }
      if (R == 1) {
        if (valid) {
          const int t = tok(t0 + ti);
          const int64_t ob = b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2] +
                             (int64_t)p0 * a.y.stride[3];
          if (vec_y) {
            uint4* dst = reinterpret_cast<uint4*>(yp + ob);
#pragma unroll
            for (int c = 0; c < 2; ++c)
              dst[c] = make_uint4(pack2<T>(out[8 * c], out[8 * c + 1]), pack2<T>(out[8 * c + 2], out[8 * c + 3]),
                                  pack2<T>(out[8 * c + 4], out[8 * c + 5]), pack2<T>(out[8 * c + 6], out[8 * c + 7]));
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) yp[ob + jj * a.y.stride[3]] = from_f<T>(out[jj]);
          }
        }
      } else {
        // times mo_r, then the rank sum as a reduce-scatter over the R adjacent lanes of a token: each
        // exchange halves the columns a lane carries (the lane with bit `o` keeps the upper half), so
        // lane r ends with 16 / R finished columns starting at p0 + cb.
        const float4* mo4 = reinterpret_cast<const float4*>(cst + Lay::CMo + r * kP + p0);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 m = mo4[q4];
          out[4 * q4] *= m.x;
          out[4 * q4 + 1] *= m.y;
          out[4 * q4 + 2] *= m.z;
          out[4 * q4 + 3] *= m.w;
        }
        int cb = 0;
#pragma unroll
        for (int o = 1, cnt = 16; o < R; o <<= 1, cnt >>= 1) {
          const bool up = (lane & o) != 0;
#pragma unroll
          for (int i = 0; i < cnt / 2; ++i) {
            const float send = up ? out[i] : out[i + cnt / 2];
            const float keep = up ? out[i + cnt / 2] : out[i];
            out[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
          if (up) cb += cnt / 2;
        }
        constexpr int kCols = 16 / R;
        if (valid) {
          const int t = tok(t0 + ti);
          const int64_t ob = b * a.y.stride[0] + (int64_t)t * a.y.stride[1] + h * a.y.stride[2] +
                             (int64_t)(p0 + cb) * a.y.stride[3];
          if (vec_y && kCols >= 2) {
            uint32_t w[kCols / 2];
#pragma unroll
            for (int i = 0; i < kCols / 2; ++i) w[i] = pack2<T>(out[2 * i], out[2 * i + 1]);
            if constexpr (kCols == 8) {
              *reinterpret_cast<uint4*>(yp + ob) = make_uint4(w[0], w[1], w[2], w[3]);
            } else if constexpr (kCols == 4) {
              *reinterpret_cast<uint2*>(yp + ob) = make_uint2(w[0], w[1]);
            } else {
              *reinterpret_cast<uint32_t*>(yp + ob) = w[0];
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < kCols; ++jj) yp[ob + jj * a.y.stride[3]] = from_f<T>(out[jj]);
          }
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
#ifdef M3_SECTION_TIMING
  if (blockIdx.x == 0 && blockIdx.y == 0 && tid == 0)
    for (int k_ = 0; k_ < 16; ++k_) atomicAdd(&g_section_cycles[k_], (unsigned long long)mark_acc_[k_]);
#endif

  // ---- final state: S[p][n] = phi X^T ----
  fence_after();
  if (!*abort_flag && (kStateOnly || last_seg) && !(a.reverse == 2 && rev)) {
    uint32_t r32[32];
    M3_TMEM_LD32(tmem + lane_base + kColState + part * 32, r32);
    tmem_wait_ld();
    const int n = quad * 32 + lane;
    if (kStateOnly) {  // the segment's record: end state [P][N] and total log-decay
#pragma unroll
      for (int j = 0; j < 32; ++j) prec[(part * 32 + j) * kN + n] = __uint_as_float(r32[j]) * phi;
      if (tid == 0) prec[rec_c0(R) + 1] = decay_sum;
    } else {
      const m3_tensor& fs = a.final_state;
      float* fsp = static_cast<float*>(fs.data) + b * fs.stride[0] + h * fs.stride[1] + n * fs.stride[3];
#pragma unroll
      for (int j = 0; j < 32; ++j) fsp[(part * 32 + j) * fs.stride[2]] = __uint_as_float(r32[j]) * phi;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Scan over segments (one CTA per (head, batch), FP32): turns the state-pass records into the
// initial cache of every later segment. phi_s, the block offset at the start of segment s, follows
// from phi_{s-1} by replaying the blocked carry over segment s - 1's recorded block totals T_k,
// phi <- fmod(phi + T_k, 2 pi) (model.py:246-251, bit for bit what an unsplit scan carries). With the
// true end state S and last rotated k of segment s - 1, and segment s's record (local end state S_s,
// local last rotated k_s, endpoint weight c0_s of its first token, total log-decay D_s):
//   S <- e^{D_s} (S + c0_s sum_r (v mx_r) k_r^T) + S_s R(phi_s)^T     (v: value of the token before s)
//   k <- R(phi_s) k_s
// R(phi) rotates the rotation pairs of the N axis (SISO (2i, 2i+1), MIMO (i, 2S + i)): the state pass
// ran segment s from phase 0, and rotating every k of a segment by one extra angle rotates its whole
// state contribution by it (mamba3/ops.py:35-84 pair layout, ops.py:804-816 state carry). A
// precomputed phase tensor already holds absolute phases: then nothing is rotated.
// Thread t owns state row p = t / 4 and the columns [16 q, 16 q + 16) and [64 + 16 q, 64 + 16 q + 16),
// q = t % 4, so both members of every rotation pair stay in one thread.
template <int R>
__global__ void __launch_bounds__(256) seg_combine_kernel(const m3_scan_args a, const SegArgs sg) {
  constexpr int REC = seg_rec(R);
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int S = a.num_angles;
  const bool mimo = a.mimo_rotation != 0;
  const bool carry = a.angles.data != nullptr;  // in-kernel phase: segments ran from phase 0
  const int p = tid >> 2, q = tid & 3;
  __shared__ float ph[kMaxAngles], cs[kMaxAngles], sn[kMaxAngles];
  __shared__ float kt[R * kN];
  __shared__ float xv[R * kP];
  auto rec = [&](float* base, int s_) { return base + ((int64_t)(s_ * a.batch + b) * a.heads + h) * REC; };
  auto col = [&](int i) { return i < 16 ? 16 * q + i : 64 + 16 * q + (i - 16); };
  float st[32];
  {
    const float* r0 = rec(sg.part, 0);
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(r0 + p * kN + col(i));
      st[i] = v.x, st[i + 1] = v.y, st[i + 2] = v.z, st[i + 3] = v.w;
    }
    if (tid < kMaxAngles) {
      const m3_tensor& ip = a.initial_phase;
      ph[tid] = (carry && ip.data && tid < S) ? ld_t(ip, b * ip.stride[0] + h * ip.stride[1] + tid * ip.stride[2]) : 0.0f;
    }
    for (int i = tid; i < R * kN; i += blockDim.x) kt[i] = r0[kRecK + i];
  }
  __syncthreads();
  for (int s_ = 1; s_ < sg.nseg; ++s_) {
    float* ri = rec(sg.init, s_);
    if (carry && tid < S) {  // block offset at the start of segment s_
      const float* bt = sg.blk + ((int64_t)((s_ - 1) * a.batch + b) * a.heads + h) * sg.nblk * kMaxAngles + tid;
      float off = ph[tid];
      for (int k = 0; k < sg.nblk; ++k) off = fmodf(off + bt[k * kMaxAngles], kTwoPi);
      ph[tid] = off;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4*>(ri + p * kN + col(i)) = make_float4(st[i], st[i + 1], st[i + 2], st[i + 3]);
    if (tid < kMaxAngles) ri[kRecPhase + tid] = ph[tid];
    for (int i = tid; i < R * kN; i += blockDim.x) ri[kRecK + i] = kt[i];
    if (s_ == sg.nseg - 1) break;
    const float* rp = rec(sg.part, s_);
    const float c0 = rp[rec_c0(R)], decay = __expf(rp[rec_c0(R) + 1]);
    const int tprev = scan_token(a, s_ * sg.seg_len - 1);
    if (tid < kP) {
      const float v = ld_t(a.value, b * a.value.stride[0] + (int64_t)tprev * a.value.stride[1] + h * a.value.stride[2] +
                                        tid * a.value.stride[3]);
#pragma unroll
      for (int r = 0; r < R; ++r)
        xv[r * kP + tid] = R > 1 ? v * ld_t(a.mimo_x, h * a.mimo_x.stride[0] + r * a.mimo_x.stride[1] +
                                                           tid * a.mimo_x.stride[2])
                                 : v;
    }
    if (tid < kMaxAngles) sincosf(carry && tid < S ? ph[tid] : 0.0f, &sn[tid], &cs[tid]);
    __syncthreads();
    float loc[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(rp + p * kN + col(i));
      loc[i] = v.x, loc[i + 1] = v.y, loc[i + 2] = v.z, loc[i + 3] = v.w;
    }
    if (!carry) {
      // absolute phases: the local records are already true
    } else if (!mimo) {
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const int ang = (16 * q + i) >> 1;
        if (ang < S) {
          const float x0 = loc[i], x1 = loc[i + 1];
          loc[i] = x0 * cs[ang] - x1 * sn[ang];
          loc[i + 1] = x0 * sn[ang] + x1 * cs[ang];
        }
      }
    } else if (16 * q < S) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int ang = 16 * q + i;
        if (ang < S) {
          const float x0 = loc[i], x1 = loc[16 + i];
          loc[i] = x0 * cs[ang] - x1 * sn[ang];
          loc[16 + i] = x0 * sn[ang] + x1 * cs[ang];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = col(i);
      float u = 0.0f;
#pragma unroll
      for (int r = 0; r < R; ++r) u += xv[r * kP + p] * kt[r * kN + n];
      st[i] = decay * (st[i] + c0 * u) + loc[i];
    }
    __syncthreads();  // every thread has read kt and xv
    // k of the segment's last token: its local rotation composed with the starting phase.
    for (int t = tid; t < R * 64; t += blockDim.x) {
      const int r = t >> 6, i = t & 63;
      const int n0 = mimo ? i : 2 * i, n1 = mimo ? i + 64 : 2 * i + 1;
      const float x0 = rp[kRecK + r * kN + n0], x1 = rp[kRecK + r * kN + n1];
      const int ang = i;
      if (carry && ang < S) {
        kt[r * kN + n0] = x0 * cs[ang] - x1 * sn[ang];
        kt[r * kN + n1] = x0 * sn[ang] + x1 * cs[ang];
      } else {
        kt[r * kN + n0] = x0;
        kt[r * kN + n1] = x1;
      }
    }
    __syncthreads();
  }
}

static bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against the driver).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 16-bit row tiles: dims / element strides innermost first (strides of dims 1.. only).
static bool encode_rows(CUtensorMap* map, const m3_tensor& t, int rank, const uint64_t* dims, const int64_t* strides,
                        const uint32_t* box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t gdim[5], gstr[4];
  cuuint32_t bdim[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
  }
  // A dimension of extent 1 is only ever read at coordinate 0: give it a valid nonzero stride.
  for (int i = 0; i + 1 < rank; ++i) gstr[i] = (cuuint64_t)(dims[i + 1] == 1 ? 8 : strides[i]) * 2;
  const CUtensorMapDataType dt = t.dtype == M3_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return enc(map, dt, (cuuint32_t)rank, t.data, gdim, gstr, bdim, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Segment plan of a call: how many segments and how long. Automatic (a.segments == 0): one segment
// while the (batch, head) pairs fill every SM; otherwise as many segments as fill the two CTA slots
// of every SM, each at least kMinSegTokens long. a.segments == 1 forces one segment, n >= 2 asks for
// n (at least 64 tokens each). Segments hold a multiple of 64 tokens (the phase block).
constexpr int kMinSegTokens = 256;

static int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();  // clear the sticky-free error of the query
      return 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

struct SegPlan {
  int nseg, seg_len;
};

static SegPlan seg_plan(const m3_scan_args& a) {
  const int64_t L = a.length;
  if (a.reverse == 2) return {1, (int)L};  // both directions in one launch: no split
  int want = 1;
  if (a.segments >= 2) {
    want = (int)std::min<int64_t>(a.segments, (L + 63) / 64);
  } else if (a.segments == 0) {
    const int64_t pairs = (int64_t)a.batch * a.heads;
    const int sms = sm_count();
    if (pairs < sms) want = (int)std::min<int64_t>(2LL * sms / pairs, L / kMinSegTokens);
  }
  want = std::max(1, std::min(want, 64));
  if (want == 1) return {1, (int)L};
  const int64_t len = ((L + want - 1) / want + 63) / 64 * 64;
  return {(int)((L + len - 1) / len), (int)len};
}

// Floats of the per-token rows, rounded up to a 256-byte boundary; the segment records follow.
static int64_t token_row_floats(const m3_scan_args& a) {
  const bool rows = a.q_norm_w.data != nullptr || a.angles.data != nullptr;
  if (!rows) return 0;
  return ((int64_t)a.batch * a.length * ws_stride(a.rank, a.num_angles) + 63) / 64 * 64;
}

// Segment scratch: the state-pass records and the initial caches ([nseg][B][H][seg_rec] each),
// then the block phase totals ([nseg][B][H][seg_len / 64][32]).
static int64_t seg_floats(const m3_scan_args& a, const SegPlan& sp) {
  if (sp.nseg <= 1) return 0;
  const int64_t pairs = (int64_t)sp.nseg * a.batch * a.heads;
  return 2 * pairs * seg_rec(a.rank) + pairs * (sp.seg_len / kPhaseBlock) * kMaxAngles;
}

static int64_t workspace_floats(const m3_scan_args& a) { return token_row_floats(a) + seg_floats(a, seg_plan(a)); }

template <typename T, int R>
static cudaError_t launch_r(const m3_scan_args& a, cudaStream_t stream) {
  // 16-byte vector stores of y need unit element stride and aligned row starts.
  auto even = [](int64_t s, int m) { return s % m == 0; };
  const int vec_y = a.y.stride[3] == 1 && aligned(a.y.data, 16) && even(a.y.stride[0], 8) &&
                    even(a.y.stride[1], 8) && even(a.y.stride[2], 8) &&
                    (a.reverse != 2 || aligned(a.y_reverse.data, 16));
  const bool token_rows = a.q_norm_w.data != nullptr || a.angles.data != nullptr;
  const SegPlan sp = seg_plan(a);
  SegArgs sg{sp.seg_len, sp.nseg, sp.seg_len / kPhaseBlock, nullptr, nullptr, nullptr};
  if (sp.nseg > 1) {
    const int64_t pairs = (int64_t)sp.nseg * a.batch * a.heads;
    sg.part = static_cast<float*>(a.workspace.data) + token_row_floats(a);
    sg.init = sg.part + pairs * seg_rec(R);
    sg.blk = sg.init + pairs * seg_rec(R);
  }
  if (token_rows) {
    const int64_t tokens = (int64_t)a.batch * a.length;
    token_prep_kernel<T><<<(unsigned)((tokens + 7) / 8), 256, 0, stream>>>(a, static_cast<float*>(a.workspace.data));
    cudaError_t pe = cudaGetLastError();
    if (pe != cudaSuccess) return pe;
  }
  constexpr uint32_t TOK = Layout<R>::TOK;
  TileMaps tm;
  memset(&tm, 0, sizeof(tm));
  if (a.reverse != 1) {
    const uint64_t dq[5] = {(uint64_t)a.d_state, (uint64_t)R, (uint64_t)a.groups, (uint64_t)a.length,
                            (uint64_t)a.batch};
    const uint32_t bq[5] = {64, (uint32_t)R, 1, TOK, 1};
    const int64_t sq[4] = {a.q.stride[3], a.q.stride[2], a.q.stride[1], a.q.stride[0]};
    const int64_t sk[4] = {a.k.stride[3], a.k.stride[2], a.k.stride[1], a.k.stride[0]};
    const uint64_t dx[4] = {(uint64_t)a.head_dim, (uint64_t)a.heads, (uint64_t)a.length, (uint64_t)a.batch};
    const uint32_t bx[4] = {64, 1, TOK, 1};
    const int64_t sx[3] = {a.value.stride[2], a.value.stride[1], a.value.stride[0]};
    const int64_t sz[3] = {a.gate.stride[2], a.gate.stride[1], a.gate.stride[0]};
    if (!encode_rows(&tm.q, a.q, 5, dq, sq, bq) || !encode_rows(&tm.k, a.k, 5, dq, sk, bq) ||
        !encode_rows(&tm.x, a.value, 4, dx, sx, bx) || !encode_rows(&tm.z, a.gate, 4, dx, sz, bx))
      return cudaErrorInvalidValue;
    if (token_rows) {
      PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
      const int W = ws_stride(R, a.num_angles);
      const cuuint64_t gdim[3] = {(cuuint64_t)W, (cuuint64_t)a.length, (cuuint64_t)a.batch};
      const cuuint64_t gstr[2] = {(cuuint64_t)W * 4, (cuuint64_t)a.length * W * 4};
      const cuuint32_t bdim[3] = {(cuuint32_t)W, TOK, 1}, estr[3] = {1, 1, 1};
      if (enc == nullptr ||
          enc(&tm.ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.workspace.data, gdim, gstr, bdim, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    }
  }
  constexpr uint32_t smem = Layout<R>::SmemBytes;
  if (sp.nseg > 1) {
    auto pass1 = scan_umma_kernel<T, R, true>;
    cudaError_t e = cudaFuncSetAttribute(pass1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    pass1<<<dim3(a.heads, a.batch, sp.nseg - 1), kThreads, smem, stream>>>(a, tm, vec_y, sg);
    seg_combine_kernel<R><<<dim3(a.heads, a.batch), 256, 0, stream>>>(a, sg);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  auto kern = scan_umma_kernel<T, R, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(a.reverse == 2 ? 2 * a.heads : a.heads, a.batch, a.reverse == 2 ? 1 : sp.nseg), kThreads, smem, stream>>>(a, tm, vec_y, sg);
  return cudaGetLastError();
}

// Summary of a whole sequence for a context-parallel caller: the state pass alone, run as one
// segment from the caller's initial cache (or zeros), writing the segment record of every (batch,
// head) into `record` [B][H][seg_rec(R)] and the 64-token block phase totals into `blocks`
// [B][H][L / 64][32]. The workspace holds the per-token rows as for an unsplit scan.
template <typename T, int R>
static cudaError_t summary_r(const m3_scan_args& a, float* record, float* blocks, cudaStream_t stream) {
  if (a.reverse) return cudaErrorInvalidValue;  // forward scans only
  const bool token_rows = a.q_norm_w.data != nullptr || a.angles.data != nullptr;
  SegArgs sg{a.length, 1, a.length / kPhaseBlock, record, nullptr, blocks};
  if (token_rows) {
    const int64_t tokens = (int64_t)a.batch * a.length;
    token_prep_kernel<T><<<(unsigned)((tokens + 7) / 8), 256, 0, stream>>>(a, static_cast<float*>(a.workspace.data));
    cudaError_t pe = cudaGetLastError();
    if (pe != cudaSuccess) return pe;
  }
  TileMaps tm;
  memset(&tm, 0, sizeof(tm));
  {
    constexpr uint32_t TOK = Layout<R>::TOK;
    const uint64_t dq[5] = {(uint64_t)a.d_state, (uint64_t)R, (uint64_t)a.groups, (uint64_t)a.length,
                            (uint64_t)a.batch};
    const uint32_t bq[5] = {64, (uint32_t)R, 1, TOK, 1};
    const int64_t sq[4] = {a.q.stride[3], a.q.stride[2], a.q.stride[1], a.q.stride[0]};
    const int64_t sk[4] = {a.k.stride[3], a.k.stride[2], a.k.stride[1], a.k.stride[0]};
    const uint64_t dx[4] = {(uint64_t)a.head_dim, (uint64_t)a.heads, (uint64_t)a.length, (uint64_t)a.batch};
    const uint32_t bx[4] = {64, 1, TOK, 1};
    const int64_t sx[3] = {a.value.stride[2], a.value.stride[1], a.value.stride[0]};
    if (!encode_rows(&tm.q, a.q, 5, dq, sq, bq) || !encode_rows(&tm.k, a.k, 5, dq, sk, bq) ||
        !encode_rows(&tm.x, a.value, 4, dx, sx, bx))
      return cudaErrorInvalidValue;
    if (token_rows) {
      PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
      const int W = ws_stride(R, a.num_angles);
      const cuuint64_t gdim[3] = {(cuuint64_t)W, (cuuint64_t)a.length, (cuuint64_t)a.batch};
      const cuuint64_t gstr[2] = {(cuuint64_t)W * 4, (cuuint64_t)a.length * W * 4};
      const cuuint32_t bdim[3] = {(cuuint32_t)W, TOK, 1}, estr[3] = {1, 1, 1};
      if (enc == nullptr ||
          enc(&tm.ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.workspace.data, gdim, gstr, bdim, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    }
  }
  constexpr uint32_t smem = Layout<R>::SmemBytes;
  auto pass1 = scan_umma_kernel<T, R, true>;
  cudaError_t e = cudaFuncSetAttribute(pass1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  pass1<<<dim3(a.heads, a.batch, 1), kThreads, smem, stream>>>(a, tm, 0, sg);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t summary_t(const m3_scan_args& a, float* record, float* blocks, cudaStream_t stream) {
  switch (a.rank) {
    case 1: return summary_r<T, 1>(a, record, blocks, stream);
    case 2: return summary_r<T, 2>(a, record, blocks, stream);
    case 4: return summary_r<T, 4>(a, record, blocks, stream);
    default: return summary_r<T, 8>(a, record, blocks, stream);
  }
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
  return umma::workspace_floats(a) * (int64_t)sizeof(float);
}

int scan_umma_segments(const m3_scan_args& a) { return umma::seg_plan(a).nseg; }

// Rows of q/k (N elements), value and gate (P elements) that start on 16-byte boundaries and are
// contiguous, so the kernel can move them with 16-byte asynchronous copies.
static bool rows16(const m3_tensor& t, int nd) {
  if ((reinterpret_cast<uintptr_t>(t.data) & 15u) != 0 || t.stride[nd - 1] != 1) return false;
  for (int i = 0; i < nd - 1; ++i)
    if (t.stride[i] % 8 != 0 || t.stride[i] < 0) return false;
  return true;
}

// Tensor-map strides: every dimension of extent > 1 advances through memory.
static bool strided(const m3_tensor& t, std::initializer_list<int64_t> extents) {
  int i = 0;
  for (int64_t e : extents) {
    if (e > 1 && t.stride[i] == 0) return false;
    ++i;
  }
  return true;
}

bool scan_umma_supported(const m3_scan_args& a) {
  const bool has_phase = a.phase.data != nullptr || a.angles.data != nullptr;
  return (a.value.dtype == M3_BF16 || a.value.dtype == M3_F16) && a.d_state == umma::kN &&
         rows16(a.q, 5) && rows16(a.k, 5) && rows16(a.value, 4) && rows16(a.gate, 4) &&
         strided(a.q, {a.batch, a.length, a.groups, a.rank}) && strided(a.k, {a.batch, a.length, a.groups, a.rank}) &&
         strided(a.value, {a.batch, a.length, a.heads}) && strided(a.gate, {a.batch, a.length, a.heads}) &&
         !(a.q_norm_w.data != nullptr && a.phase.data != nullptr) &&
         a.head_dim == umma::kP && (a.rank == 1 || a.rank == 2 || a.rank == 4 || a.rank == 8) &&
         (!has_phase || (a.mimo_rotation ? a.num_angles == umma::kMaxAngles : a.num_angles <= umma::kMaxAngles));
}

#ifdef M3_SECTION_TIMING
// Probe builds only: per-section cycle totals of CTA (0, 0), thread 0, summed over launches.
extern "C" int m3_probe_read_sections(unsigned long long* host16, int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(host16, umma::g_section_cycles, 16 * sizeof(unsigned long long)) != cudaSuccess) return -1;
  if (clear) {
    unsigned long long zero[16] = {};
    if (cudaMemcpyToSymbol(umma::g_section_cycles, zero, sizeof(zero)) != cudaSuccess) return -1;
  }
  return 0;
}
#endif

cudaError_t launch_scan_summary(const m3_scan_args& a, float* record, float* blocks, cudaStream_t stream) {
  return a.value.dtype == M3_BF16 ? umma::summary_t<__nv_bfloat16>(a, record, blocks, stream)
                                  : umma::summary_t<__half>(a, record, blocks, stream);
}

int scan_summary_record_floats(int rank) { return umma::seg_rec(rank); }

cudaError_t launch_scan_umma(const m3_scan_args& a, cudaStream_t stream) {
  return a.value.dtype == M3_BF16 ? umma::launch_t<__nv_bfloat16>(a, stream) : umma::launch_t<__half>(a, stream);
}

}  // namespace m3
