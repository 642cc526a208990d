// Per-tile prologue shared by the chunked-SSD kernels: discretisation scalars and phase.
//
// A CTA owns one (batch, head) pair and walks the sequence in scan order, one tile of TOK
// tokens at a time. These helpers fill shared-memory arrays for the current tile:
//   s_cum[j]   inclusive cumsum of adt over the tile            (mamba3/ops.py:739)
//   s_ecum[j]  exp(cum_j)                 (inter-chunk decay, ops.py:740)
//   s_edec[j]  exp(cum_last - cum_j)      (state-carry decay, ops.py:806)
//   s_scale[j] gamma_j + dt_{j+1}(1 - sigma_{j+1})   (ops.py:659-665; 0 after the last token)
//   s_diag[j]  gamma_j / scale_j          (same-token diagonal, ops.py:671, 775-783)
//   s_ph[j][s] phase of token j           (precomputed, or accumulated with model.py:215-256)
#pragma once

#include "common.cuh"

namespace m3 {

// Original token index of scan-order position `ts` (bidirectional backward direction reads
// the sequence back to front, mamba3/model.py:333).
__device__ __forceinline__ int scan_token(const m3_scan_args& a, int ts) {
  return a.reverse ? (a.length - 1 - ts) : ts;
}

// dt and adt of token t for head h (fp32 tensors, or raw logits with dt_bias).
__device__ __forceinline__ void load_dt_adt(const m3_scan_args& a, int b, int t, int h, float& dtv, float& adtv) {
  const int64_t ia = b * a.adt.stride[0] + (int64_t)t * a.adt.stride[1] + h * a.adt.stride[2];
  const int64_t id = b * a.dt.stride[0] + (int64_t)t * a.dt.stride[1] + h * a.dt.stride[2];
  if (a.dt_bias.data) {
    // mamba3/model.py:195-198: dt = softplus(delta + dt_bias); A = -heavytail(a) clamped <= -1e-4.
    dtv = softplusf_(ld_t(a.dt, id) + ld_t(a.dt_bias, h));
    const float A = fminf(-heavy_tailf(ld_t(a.adt, ia)), -kAFloor);
    adtv = A * dtv;
  } else {
    dtv = ld_t(a.dt, id);
    adtv = ld_t(a.adt, ia);
  }
}

__device__ __forceinline__ float load_trap(const m3_scan_args& a, int b, int t, int h) {
  return ld_t(a.trap, b * a.trap.stride[0] + (int64_t)t * a.trap.stride[1] + h * a.trap.stride[2]);
}

struct TileScalars {
  float* cum;
  float* ecum;
  float* edec;
  float* scale;
  float* diag;
  float* dt;     // dt of each tile token (phase increments)
  float* wsum;   // >= 8 floats scratch (warp totals of the scan, look-ahead token)
};

// Fill the per-token scalars of tile [t0, t0 + nt) (scan order). All loads are issued in one
// parallel round (thread j loads token j; one extra thread loads the first token after the tile).
// Requires TOK <= 128 and blockDim.x >= 160. Ends with __syncthreads().
__device__ inline void tile_scalars(const m3_scan_args& a, int b, int h, int t0, int nt, int TOK,
                                    const TileScalars& s, float& last_decay) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  // Round 1: raw per-token values. adt is parked in `cum`, sigma in `edec`.
  if (tid <= TOK) {
    float dtv = 0.0f, adtv = 0.0f, sg = 0.0f;
    if (t0 + tid < a.length && (tid < nt || tid == TOK)) {
      const int t = scan_token(a, t0 + tid);
      load_dt_adt(a, b, t, h, dtv, adtv);
      sg = sigmoidf_(load_trap(a, b, t, h));
    }
    if (tid < TOK) {
      s.dt[tid] = tid < nt ? dtv : 0.0f;
      s.cum[tid] = tid < nt ? adtv : 0.0f;
      s.edec[tid] = sg;
    } else {
      s.wsum[4] = dtv;
      s.wsum[5] = sg;
    }
  }
  __syncthreads();
  // Round 2: trapezoid scalars and the inclusive scan of adt (4 warps x 32).
  float v = 0.0f;
  if (tid < 128) {
    const float adtv = tid < TOK ? s.cum[tid] : 0.0f;
    v = warp_incl_scan(adtv, lane);
    if (lane == 31) s.wsum[tid >> 5] = v;
    if (tid < TOK) {
      float scale = 0.0f, diag = 0.0f;
      if (tid < nt) {
        const float gamma = s.dt[tid] * s.edec[tid];
        float nxt = 0.0f;
        if (tid + 1 < nt) nxt = s.dt[tid + 1] * (1.0f - s.edec[tid + 1]);
        else if (t0 + tid + 1 < a.length) nxt = s.wsum[4] * (1.0f - s.wsum[5]);
        scale = gamma + nxt;
        diag = gamma / scale;
      }
      s.scale[tid] = scale;
      s.diag[tid] = diag;
    }
  }
  __syncthreads();
  if (tid < TOK) {
    const int w = tid >> 5;
    for (int i = 0; i < w; ++i) v += s.wsum[i];
    s.cum[tid] = v;
  }
  __syncthreads();
  const float cl = s.cum[nt - 1];
  if (tid < TOK) {
    const float c = s.cum[tid];
    s.ecum[tid] = tid < nt ? expf(c) : 0.0f;
    s.edec[tid] = tid < nt ? expf(cl - c) : 0.0f;
  }
  last_decay = expf(cl);
  __syncthreads();
}

// Phase of every token of the tile, s_ph[j * ph_stride + s].
//  - precomputed phase tensor: copy.
//  - angle logits: blocked accumulation of mamba3/model.py:215-256 — increments
//    fmod(pi tanh(angle) dt, 2pi) summed from the start of each 64-token block, the block offset
//    carried in `carry_off` and reduced mod 2pi at every block end; the running within-block sum
//    is carried across tiles in `carry_loc` (tiles may be shorter than a block).
// `seg_buf` needs 3 * 256 floats; TOK is a power of two <= 128 and blockDim.x >= 256 (only the
// first 256 threads take part in the segment sums), so each segment of SL tokens lies inside one
// 64-token block. Ends with __syncthreads().
__device__ inline void tile_phase(const m3_scan_args& a, int b, int h, int t0, int nt, int TOK, const float* s_dt,
                                  float* s_ph, int ph_stride, float* carry_off, float* carry_loc, float* seg_buf) {
  const int S = a.num_angles;
  const int tid = threadIdx.x;
  if (a.phase.data) {
    for (int i = tid; i < TOK * S; i += blockDim.x) {
      const int j = i / S, sidx = i % S;
      float v = 0.0f;
      if (j < nt) {
        const int t = scan_token(a, t0 + j);
        v = ld_t(a.phase, b * a.phase.stride[0] + (int64_t)t * a.phase.stride[1] + h * a.phase.stride[2] +
                              sidx * a.phase.stride[3]);
      }
      s_ph[j * ph_stride + sidx] = v;
    }
    __syncthreads();
    return;
  }
  // Round 1: every increment, loads issued in parallel (consecutive threads -> consecutive angles).
  for (int i = tid; i < TOK * S; i += blockDim.x) {
    const int j = i / S, sidx = i % S;
    float inc = 0.0f;
    if (j < nt) {
      const int t = scan_token(a, t0 + j);
      const float th = ld_t(a.angles, b * a.angles.stride[0] + (int64_t)t * a.angles.stride[1] +
                                          sidx * a.angles.stride[2]);
      inc = fmodf((kPi * tanhf(th)) * s_dt[j], kTwoPi);
    }
    s_ph[j * ph_stride + sidx] = inc;
  }
  __syncthreads();
  // Round 2: segment-local inclusive sums (S_pad threads per segment row, nseg segments).
  int S_pad = 1;
  while (S_pad < S) S_pad <<= 1;
  const int nseg_max = 256 / S_pad;
  int nseg = 1;
  while (nseg * 2 <= nseg_max && TOK % (nseg * 2) == 0) nseg <<= 1;
  const int SL = TOK / nseg;
  const int sidx = tid % S_pad;
  const int seg = tid / S_pad;
  const bool active = tid < 256 && sidx < S && seg < nseg;
  if (active) {
    float local = 0.0f;
    for (int j = seg * SL; j < (seg + 1) * SL; ++j) {
      local += s_ph[j * ph_stride + sidx];
      s_ph[j * ph_stride + sidx] = local;
    }
    seg_buf[seg * S_pad + sidx] = local;
  }
  __syncthreads();
  if (tid < S) {
    float off = carry_off[tid], loc = carry_loc[tid];
    for (int sg = 0; sg < nseg; ++sg) {
      const int gi = t0 + sg * SL;
      if (gi > 0 && (gi % kPhaseBlock) == 0) {  // a new 64-token block starts here
        off = fmodf(off + loc, kTwoPi);
        loc = 0.0f;
      }
      const float tot = seg_buf[sg * S_pad + tid];
      seg_buf[256 + sg * S_pad + tid] = loc;  // within-block sum before this segment
      seg_buf[512 + sg * S_pad + tid] = off;  // block offset for this segment
      loc += tot;
    }
    carry_off[tid] = off;
    carry_loc[tid] = loc;
  }
  __syncthreads();
  if (active) {
    const float base = seg_buf[256 + seg * S_pad + sidx];
    const float off = seg_buf[512 + seg * S_pad + sidx];
    for (int j = seg * SL; j < (seg + 1) * SL; ++j) {
      s_ph[j * ph_stride + sidx] = fmodf((base + s_ph[j * ph_stride + sidx]) + off, kTwoPi);
    }
  }
  __syncthreads();
}

}  // namespace m3
