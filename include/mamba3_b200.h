/*
 * mamba3_b200 — C ABI of the B200 (sm_100a) Mamba-3 chunked-SSD and decode-step kernels.
 *
 * These entry points replace the Triton dispatch of jreoka/mamba3:
 *   m3_scan_fwd  replaces  mamba3/ops.py:253-505   (_fused_chunk_scan / _fused_chunk_scan_impl,
 *                                                   i.e. the per-chunk _chunk_main_kernel +
 *                                                   _chunk_state_kernel launches of
 *                                                   mamba3/_triton.py:416-561)
 *   m3_step_fwd  replaces  mamba3/ops.py:87-190    (fused_step -> mamba3/_triton.py:950-1151)
 *
 * Conventions
 *   - Every tensor is passed as an m3_tensor: device pointer, element dtype and element strides
 *     (not bytes). Shapes are given once in the argument struct. A NULL data pointer marks an
 *     optional tensor as absent.
 *   - `stream` is a cudaStream_t (passed as void*). Kernels are enqueued on it; nothing
 *     synchronises, allocates or frees memory, so every call can be captured in a CUDA graph.
 *   - Return value: 0 on success, otherwise an M3_ERR_* code; m3_last_error() then returns a
 *     human-readable message (thread-local). Shape/dtype/stride checks happen before launch.
 *   - Device-side waits are bounded; a wait that gives up sets a device error word that
 *     m3_device_error() reads (synchronising the device).
 */
#ifndef MAMBA3_B200_H
#define MAMBA3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M3_ABI_VERSION 3

enum m3_dtype { M3_F32 = 0, M3_F16 = 1, M3_BF16 = 2 };

enum m3_status {
  M3_OK = 0,
  M3_ERR_SHAPE = 1,       /* a shape is inconsistent or unsupported */
  M3_ERR_DTYPE = 2,       /* an unsupported or inconsistent dtype */
  M3_ERR_LAYOUT = 3,      /* a stride/alignment requirement is not met */
  M3_ERR_ARGUMENT = 4,    /* missing required tensor / invalid flag */
  M3_ERR_CUDA = 5,        /* a CUDA runtime error at launch */
};

typedef struct m3_tensor {
  void* data;             /* device pointer, NULL = absent */
  int32_t dtype;          /* enum m3_dtype */
  int32_t ndim;           /* number of valid entries in stride[] */
  int64_t stride[6];      /* element strides, outermost first */
} m3_tensor;

/*
 * Chunked SSD forward over a whole sequence (prefill / forward).
 * Semantics: mamba3/ops.py:544-822 (mamba3_scan), including the endpoint-cache continuation
 * (ops.py:679-686), q/k head expansion + bias + rotation (ops.py:698-714) and the bidirectional
 * reverse direction of mamba3/model.py:330-362 when `reverse` is set.
 *
 * Inputs (B=batch, L=length, G=groups, H=heads, R=rank, N=d_state, P=head_dim, S=num_angles):
 *   q, k            [B,L,G,R,N]  activation dtype; rows are RMS-normalised in-kernel when
 *                                q_norm_w/k_norm_w are given ([N], any float dtype)
 *   q_bias, k_bias  [H,R,N]      optional, added after head expansion (model.py:211-212)
 *   value, gate     [B,L,H,P]    activation dtype
 *   adt, dt         [B,L,H]      float32 discretisation, or — when dt_bias is given — the raw
 *                                decay/delta logits of the in_proj split (model.py:195-198):
 *                                dt = softplus(delta + dt_bias), adt = min(-heavytail(a), -1e-4)*dt
 *   trap            [B,L,H]      trapezoid logits (any float dtype)
 *   phase           [B,L,H,S]    optional float32 precomputed phase, or
 *   angles          [B,L,S]      optional raw angle logits: the phase is accumulated in-kernel
 *                                with the 64-token blocked fmod scheme of model.py:215-256,
 *                                starting from initial_phase [B,H,S] (float32, optional)
 *   D               [H]
 *   mimo_x/z/out    [H,R,P]      required iff R > 1
 *   initial_state   [B,H,P,N]    float32, optional
 *   initial_k       [B,H,R,N]    optional endpoint cache (rotated previous k)
 *   initial_value   [B,H,P]      optional endpoint cache (previous value)
 *   workspace       float32 scratch of m3_scan_workspace_bytes(args) bytes (contiguous), required
 *                   when that size is non-zero: per-token values shared by all heads (RMS factors
 *                   of q/k rows, pi*tanh(angle)) computed once by a pre-pass instead of per head
 * Outputs:
 *   y               [B,L,H,P]    activation dtype
 *   final_state     [B,H,P,N]    float32
 *   final_phase     [B,H,S]      float32, optional (phase at the last token)
 *   final_k         [B,H,R,N]    activation dtype, optional (biased, rotated k of the last token)
 */
typedef struct m3_scan_args {
  int32_t batch, length, groups, heads, rank, d_state, head_dim, num_angles;
  int32_t reverse;        /* 1: scan tokens L-1..0 (bidirectional backward direction); 2: both
                             directions in one launch, forward into y, backward into y_reverse
                             (the second read of each projection row is served from L2; no caches) */
  int32_t mimo_rotation;  /* 1: rotate pairs (i, 2S+i) (MIMO layout); 0: adjacent pairs (2i, 2i+1) */
  int32_t chunk_hint;     /* caller's chunk size (validated > 0; the kernel tiles internally) */
  int32_t device;         /* CUDA device ordinal of every tensor and of `stream` (-1: current) */
  float norm_eps;         /* RMS-norm epsilon for q_norm_w / k_norm_w */
  int32_t segments;       /* sequence segments scanned in parallel: 0 = automatic (split only when
                             batch x heads leaves SMs idle), 1 = never split, n >= 2 = n segments */
  m3_tensor q, k, q_norm_w, k_norm_w, q_bias, k_bias;
  m3_tensor value, gate;
  m3_tensor adt, dt, trap, dt_bias;
  m3_tensor phase, angles, initial_phase;
  m3_tensor D, mimo_x, mimo_z, mimo_out;
  m3_tensor initial_state, initial_k, initial_value;
  m3_tensor y, final_state, final_phase, final_k;
  m3_tensor workspace;
  m3_tensor y_reverse;    /* [B,L,H,P] backward-direction output when reverse == 2 (same strides as y) */
} m3_scan_args;

/*
 * One decode step (mamba3/ops.py:87-190 contract; math of mamba3/model.py:460-484 +
 * mamba3/ops.py:825-879): advance the phase, rotate q/k, update the FP32 state with the
 * exp-trapezoidal rule, y = sum_r mo_r * silu(z mz_r) * (S' q_r + D v_r).
 *   q, k        [B,H,R,N]  activation dtype, unrotated (strides may be 0 along H)
 *   q_bias/k_bias [H,R,N]  optional, added before rotation
 *   value, gate [B,H,P]
 *   adt, dt     [B,H]      float32;  trap [B,H] any float dtype
 *   angle_rate  [B,S]      raw angle logits (shared across heads)
 *   D [H]; mimo_x/z/out [H,R,P] iff R > 1
 *   phase [B,H,S] f32, state [B,H,P,N] f32, prev_k [B,H,R,N], prev_value [B,H,P]  (the cache)
 * Outputs: y [B,H,P]; out_phase [B,H,S] f32; out_state [B,H,P,N] f32 (may alias `state`
 * exactly, for in-place decoding); out_k [B,H,R,N] (rotated k). out_phase/out_k must not
 * alias phase/prev_k.
 *   workspace   float32 scratch of m3_step_workspace_bytes(args) bytes (contiguous), required
 *               when that size is non-zero: the per-(batch, head) rotated q/k and decay scalars
 *               a pre-pass computes so that the state pass is a pure stream over HBM
 * Model mode (the projection post-processing of mamba3/model.py:189-199 done in the kernel):
 *   q_norm_w, k_norm_w [N]  optional, together: q/k are the raw C/B rows of the projection and
 *               are RMS-normalised (epsilon norm_eps) with these weights before the bias
 *   dt_bias [H] optional: dt holds the raw delta logits and adt the raw decay logits (any float
 *               dtype); the kernel forms dt = softplus(delta + dt_bias) and
 *               adt = min(-heavy_tail(decay), -1e-4) * dt
 */
typedef struct m3_step_args {
  int32_t batch, heads, rank, d_state, head_dim, num_angles;
  int32_t device;         /* CUDA device ordinal of every tensor and of `stream` (-1: current) */
  float norm_eps;         /* RMS-norm epsilon for q_norm_w / k_norm_w */
  m3_tensor q, k, q_bias, k_bias, value, gate;
  m3_tensor adt, dt, trap, angle_rate, D, mimo_x, mimo_z, mimo_out;
  m3_tensor phase, state, prev_k, prev_value;
  m3_tensor y, out_phase, out_state, out_k;
  m3_tensor workspace;
  m3_tensor q_norm_w, k_norm_w, dt_bias;
} m3_step_args;

/*
 * Residual add + RMSNorm between blocks, one pass (mamba3/model.py:487-520 block
 * `hidden + mixer(norm(hidden))` with norm = F.rms_norm(x, w.to(x.dtype), eps), and the cast of
 * the normalised rows to the next in_proj's input dtype under autocast):
 *   r = x (+ m);  out_x = r (optional, may alias x);  out_n = round(r * rsqrt(mean(r^2) + eps) * w)
 *   x, m, out_x, out_n  [rows, dim] (element strides);  w [dim];  out_n may not alias x or m.
 * The reference does this with separate PyTorch ops (add, rms_norm, dtype cast); no Triton kernel
 * of the reference corresponds to it.
 */
typedef struct m3_norm_args {
  int64_t rows;
  int32_t dim, device;  /* device: CUDA ordinal of the tensors and `stream` (-1: current) */
  float eps;
  int32_t reserved;
  m3_tensor x, m, w, out_x, out_n;
} m3_norm_args;

int m3_residual_rmsnorm(const m3_norm_args* args, void* stream);

/*
 * Few-row projection y = x W^T of a decode step (the in_proj / out_proj nn.Linear calls of
 * mamba3/model.py:422-484 at batch <= 4, a library GEMM in the reference): x [rows][in_dim],
 * W [out_dim][in_dim], y [rows][out_dim], one 16-bit dtype; FP32 accumulation, y rounded once.
 * rows 1..4, in_dim a multiple of 8 (<= 16384); x / W rows contiguous and 16-byte aligned.
 */
typedef struct m3_gemv_args {
  int64_t out_dim, in_dim;
  int32_t rows, device; /* device: CUDA ordinal of the tensors and `stream` (-1: current) */
  m3_tensor x, w, y;
} m3_gemv_args;

int m3_gemv(const m3_gemv_args* args, void* stream);

/* Chunked SSD forward. Returns M3_OK or an M3_ERR_* code. */
int m3_scan_fwd(const m3_scan_args* args, void* stream);

/* Bytes of float32 workspace m3_scan_fwd needs for these arguments (0 = none); a negative value
 * is minus an M3_ERR_* code (null arguments, non-positive sizes) with m3_last_error() set. */
int64_t m3_scan_workspace_bytes(const m3_scan_args* args);

/* Number of sequence segments the tensor-core scan kernel splits these sizes into (args->segments
 * and the GPU's SM count decide; 1 = no split). Negative: minus an M3_ERR_* code. */
int m3_scan_segments(const m3_scan_args* args);

/*
 * Context-parallel prefill: summary of one rank's slice of a sequence (forward scans on the
 * tensor-core layout). Runs the scan's state pass over the whole slice, starting from args' initial
 * cache (or zeros) and phase 0 when no initial_phase is given, and writes per (batch, head) a record
 * of m3_scan_summary_floats(rank) floats into `record` ([B][H][record]): the end state [P=64][N=128]
 * at offset 0, the biased last k rotated by the slice's own phases [R][N] at offset 64*128 + 32,
 * then the endpoint weight dt(1 - sigmoid(trap)) of the slice's first token and the slice's total
 * log-decay sum(adt). With in-kernel phases (angles) the slice length must be a multiple of 64 and
 * `blocks` ([B][H][L/64][32]) receives every 64-token block's in-block phase total, from which the
 * block-offset carry (mamba3/model.py:246-251) continues across slices. Uses the workspace of
 * m3_scan_workspace_bytes with args->segments = 1. No counterpart in the reference, which has no
 * multi-GPU path; the state algebra is that of mamba3/ops.py:804-816.
 */
int m3_scan_summary(const m3_scan_args* args, float* record, float* blocks, void* stream);

/* Floats per (batch, head) record written by m3_scan_summary for this MIMO rank. */
int m3_scan_summary_floats(int rank);

/*
 * Training kernels of the chunked SSD core (the gradients the reference's training path takes by
 * autograd through mamba3/ops.py:716-816, with the _BmmFloat GEMMs of ops.py:202-250). The core
 * op, per (batch, head), rows i = (token t, rank r), chunks of m3_ssd_chunk_rows() rows:
 *   y_i = e^{cum_t} (S_c q_i) + sum_{j in chunk, token(j) <= t} Wt_ij v_j,
 *   Wt_ij = e^{cum_t - cum_s} (q_i . k_j) for earlier tokens s, diag_t (q_i . k_j) on token t,
 *   S_{c+1} = e^{cum_last} S_c + sum_j e^{cum_last - cum_s} v_j k_j^T,
 * cum = inclusive cumsum of adt inside the chunk. All tensors float32 with element strides:
 *   q, k [B,L,H,R,N] (k already times the trapezoid scale), v [B,L,H,R,P] (rank values),
 *   adt, diag [B,L,H], initial_state / final_state / dfinal / dinitial [B,H,P,N],
 *   y / dy [B,L,H,R,P], chunk_states [B,H,ceil(L*R/rows),P,N] (written by the forward, read by
 *   the backward), dq, dk [B,L,H,R,N], dv [B,L,H,R,P], dadt, ddiag [B,L,H].
 * d_state <= 128 and head_dim <= 64, multiples of 8. initial_state, dfinal and dinitial may be
 * null (zeros / not written). Chunks run in parallel: the forward writes each chunk's state
 * contribution into chunk_states and scans them (in place) into the chunk-start states; the
 * backward scans the chunk gradients in reverse in its workspace. The bias, rotation, scale, D skip, gate and rank sum around the core are left to the
 * caller's autograd.
 */
typedef struct m3_ssd_args {
  int32_t batch, length, heads, rank, d_state, head_dim;
  int32_t device; /* CUDA device ordinal of every tensor and of `stream` (-1: current) */
  int32_t reserved;
  m3_tensor q, k, v, adt, diag, initial_state;
  m3_tensor y, final_state, chunk_states;
  m3_tensor dy, dfinal;
  m3_tensor dq, dk, dv, dadt, ddiag, dinitial;
  m3_tensor workspace; /* float32, 16-byte aligned, m3_ssd_workspace_bytes(args, backward) bytes */
} m3_ssd_args;

/*
 * Training prelude of the SSD core, fused: per (batch, token, head, rank) row, qb = q_g + q_bias,
 * kb = k_g + k_bias (g = the head's Q/K group), rotated by `phase` (SISO pairs (2m, 2m + 1), MIMO
 * pairs (m, 2S + m); mamba3/ops.py:35-84), k additionally times scale (the trapezoid scale,
 * ops.py:665-676), each step rounded to the activation dtype as the reference's tensor ops round;
 * written as float32 rows qf, kc [B,L,H,R,N]. The backward writes the gradients of the biased,
 * unrotated rows (dqb, dkb [B,L,H,R,N]), of the phase (dphase [B,L,H,S], may be null) and of the
 * scale (dscale [B,L,H]); the caller sums dqb over the heads of a group and over tokens for the
 * q / bias gradients. q, k [B,L,G,R,N] in the activation dtype; biases [H,R,N] or null; phase
 * [B,L,H,S] float32 or null; scale [B,L,H] float32. d_state <= 128, a multiple of 4 (MIMO angle
 * count a multiple of 4); float32 rows contiguous and 16-byte aligned.
 */
typedef struct m3_prelude_args {
  int32_t batch, length, groups, heads, rank, d_state, num_angles, mimo_rotation;
  int32_t device; /* CUDA device ordinal of every tensor and of `stream` (-1: current) */
  int32_t reserved;
  m3_tensor q, k, q_bias, k_bias, phase, scale;
  m3_tensor qf, kc;
  m3_tensor dqf, dkc, dqb, dkb, dphase, dscale;
} m3_prelude_args;

int m3_ssd_prelude_fwd(const m3_prelude_args* args, void* stream);
int m3_ssd_prelude_bwd(const m3_prelude_args* args, void* stream);

/* Rows (token, rank) per chunk of the training kernels. */
int m3_ssd_chunk_rows(void);

/* Bytes of float32 scratch the training forward (backward = 0) or backward (1) needs; negative:
 * minus an M3_ERR_* code. */
int64_t m3_ssd_workspace_bytes(const m3_ssd_args* args, int backward);

/* Forward of the SSD core for training: y, final_state and chunk_states. M3_OK or M3_ERR_*. */
int m3_ssd_train_fwd(const m3_ssd_args* args, void* stream);

/* Backward of the SSD core: dq, dk, dv, dadt, ddiag (and dinitial when given) from dy (and dfinal
 * when given), q, k, v, adt, diag and the forward's chunk_states. M3_OK or M3_ERR_*. */
int m3_ssd_train_bwd(const m3_ssd_args* args, void* stream);

/* Fixed scratch size of m3_scan_fwd_noalloc, per GPU that loads the library: 8 MiB. */
#define M3_NOALLOC_WORKSPACE_BYTES (8 * 1024 * 1024)

/*
 * Chunked SSD forward that allocates nothing, for callers that cannot call cudaMalloc where they
 * run the scan (a host runtime that owns all device memory through its own pool, a plugin that
 * must not touch its host process's allocator). Same arguments and results as m3_scan_fwd, but
 * args->workspace is ignored: the scratch is a fixed array inside the library's device image,
 * M3_NOALLOC_WORKSPACE_BYTES per GPU, held until process exit. Sizes whose scratch
 * (m3_scan_workspace_bytes) exceeds that limit are rejected with M3_ERR_SHAPE. The first call on
 * a device looks up the array's device address once; make that first call before any stream
 * capture. The address is cached for the life of the process, so the entry point must not be
 * used on a device after cudaDeviceReset() of that device. All calls share the one array, so calls
 * on one device that overlap on the GPU race on it; calls ordered on one stream are safe. Has no
 * counterpart in the reference.
 */
int m3_scan_fwd_noalloc(const m3_scan_args* args, void* stream);

/* Decode step. Returns M3_OK or an M3_ERR_* code. */
int m3_step_fwd(const m3_step_args* args, void* stream);

/* Bytes of float32 workspace m3_step_fwd needs for these arguments (0 = none). */
int64_t m3_step_workspace_bytes(const m3_step_args* args);

/* Message for the last non-zero status returned on this host thread. */
const char* m3_last_error(void);

/* ABI version (M3_ABI_VERSION). */
int m3_abi_version(void);

/* Synchronises the current device and returns the device error word (0 = no bounded wait
 * ever gave up); `clear` resets it. Never called on a hot path. */
int m3_device_error(int clear);

/* Name of the scan kernel variant the last m3_scan_fwd on this thread launched
 * ("umma" for the tcgen05 tensor-core kernel, "simt" for the FP32 CUDA-core kernel). */
const char* m3_last_scan_kernel(void);

/* Name of the decode-step kernel variant the last m3_step_fwd on this thread launched:
 * "single" (one launch per step, each CTA repeating its head's prologue), "two_pass" (per-(batch,
 * head) prep pass + state stream pass) or "two_pass_vec" (the 16-byte-row MIMO prep + stream pass). */
const char* m3_last_step_kernel(void);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA3_B200_H */
