// C ABI entry points: argument validation, kernel selection and error reporting.
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"

namespace m3 {
int read_device_error(int clear);

cudaError_t launch_step(const m3_step_args& a, cudaStream_t stream);
const char* last_step_kernel();
int64_t step_workspace_bytes(const m3_step_args& a);
cudaError_t launch_scan_simt(const m3_scan_args& a, cudaStream_t stream);
size_t scan_simt_smem_bytes(int rank, int N, int P, int S);
bool scan_umma_supported(const m3_scan_args& a);
int64_t scan_umma_workspace_bytes(const m3_scan_args& a);
int scan_umma_segments(const m3_scan_args& a);
cudaError_t launch_scan_summary(const m3_scan_args& a, float* record, float* blocks, cudaStream_t stream);
int scan_summary_record_floats(int rank);
cudaError_t launch_scan_umma(const m3_scan_args& a, cudaStream_t stream);
}  // namespace m3

namespace {

thread_local std::string g_last_error;
thread_local const char* g_last_scan_kernel = "none";

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

bool present(const m3_tensor& t) { return t.data != nullptr; }

bool is_float_dtype(int d) { return d == M3_F32 || d == M3_F16 || d == M3_BF16; }

#define M3_REQUIRE(cond, code, msg)        \
  do {                                     \
    if (!(cond)) return fail((code), (msg)); \
  } while (0)

int check_tensor(const m3_tensor& t, const char* name, int ndim, bool required) {
  if (!present(t)) {
    if (required) return fail(M3_ERR_ARGUMENT, std::string("missing required tensor ") + name);
    return M3_OK;
  }
  if (!is_float_dtype(t.dtype)) return fail(M3_ERR_DTYPE, std::string("unsupported dtype for ") + name);
  if (t.ndim != ndim)
    return fail(M3_ERR_SHAPE, std::string(name) + " must have " + std::to_string(ndim) + " dimensions");
  return M3_OK;
}

// Make `device` current for this host thread (the stream and tensors live there).
int select_device(int device) {
  if (device < 0) return M3_OK;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return fail(M3_ERR_CUDA, "cudaGetDevice failed");
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return fail(M3_ERR_CUDA, "cudaSetDevice failed");
  return M3_OK;
}

}  // namespace

namespace m3 {
// Record `msg` as this thread's m3_last_error() and return `code` (for other translation units).
int report_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace m3

extern "C" {

const char* m3_last_error(void) { return g_last_error.c_str(); }

int m3_abi_version(void) { return M3_ABI_VERSION; }

const char* m3_last_scan_kernel(void) { return g_last_scan_kernel; }

const char* m3_last_step_kernel(void) { return m3::last_step_kernel(); }

int m3_device_error(int clear) { return m3::read_device_error(clear); }

int64_t m3_step_workspace_bytes(const m3_step_args* args) {
  if (args == nullptr) return -fail(M3_ERR_ARGUMENT, "null argument struct");
  return m3::step_workspace_bytes(*args);
}

int m3_step_fwd(const m3_step_args* args, void* stream) {
  M3_REQUIRE(args != nullptr, M3_ERR_ARGUMENT, "null argument struct");
  const m3_step_args& a = *args;
  M3_REQUIRE(a.batch > 0 && a.heads > 0 && a.head_dim > 0 && a.d_state > 0, M3_ERR_SHAPE,
             "batch, heads, head_dim and d_state must be positive");
  M3_REQUIRE(a.rank == 1 || a.rank == 2 || a.rank == 4 || a.rank == 8, M3_ERR_SHAPE, "rank must be 1, 2, 4 or 8");
  M3_REQUIRE(a.d_state % 2 == 0 && a.d_state <= 256, M3_ERR_SHAPE, "d_state must be even and at most 256");
  M3_REQUIRE(a.num_angles >= 0 && a.num_angles <= 64 && 2 * a.num_angles <= a.d_state, M3_ERR_SHAPE,
             "angle width must be in [0, min(64, d_state / 2)]");
  M3_REQUIRE(a.rank == 1 || 4 * a.num_angles == a.d_state, M3_ERR_SHAPE,
             "MIMO decoding requires 4 * num_angles == d_state");
  struct Item { const m3_tensor* t; const char* name; int nd; bool req; };
  const Item items[] = {
      {&a.q, "q", 4, true}, {&a.k, "k", 4, true}, {&a.q_bias, "q_bias", 3, false}, {&a.k_bias, "k_bias", 3, false},
      {&a.value, "value", 3, true}, {&a.gate, "gate", 3, true}, {&a.adt, "adt", 2, true}, {&a.dt, "dt", 2, true},
      {&a.trap, "trap_logits", 2, true}, {&a.angle_rate, "angle_rate", 2, true}, {&a.D, "D", 1, true},
      {&a.mimo_x, "mimo_x", 3, a.rank > 1}, {&a.mimo_z, "mimo_z", 3, a.rank > 1},
      {&a.mimo_out, "mimo_out", 3, a.rank > 1}, {&a.phase, "phase", 3, true}, {&a.state, "state", 4, true},
      {&a.prev_k, "previous_k", 4, true}, {&a.prev_value, "previous_value", 3, true}, {&a.y, "output", 3, true},
      {&a.out_phase, "output_phase", 3, true}, {&a.out_state, "output_state", 4, true},
      {&a.out_k, "output_k", 4, true}, {&a.workspace, "workspace", 1, false},
      {&a.q_norm_w, "q_norm_w", 1, false}, {&a.k_norm_w, "k_norm_w", 1, false}, {&a.dt_bias, "dt_bias", 1, false},
  };
  for (const Item& it : items) {
    const int rc = check_tensor(*it.t, it.name, it.nd, it.req);
    if (rc != M3_OK) return rc;
  }
  M3_REQUIRE(present(a.q_bias) == present(a.k_bias), M3_ERR_ARGUMENT, "q_bias and k_bias must be given together");
  M3_REQUIRE(present(a.q_norm_w) == present(a.k_norm_w), M3_ERR_ARGUMENT,
             "q_norm_w and k_norm_w must be given together");
  M3_REQUIRE(!present(a.q_norm_w) || a.norm_eps > 0.0f, M3_ERR_ARGUMENT, "norm_eps must be positive");
  const bool raw_dt = present(a.dt_bias);
  const int act = a.value.dtype;
  M3_REQUIRE(a.q.dtype == act && a.k.dtype == act && a.gate.dtype == act && a.y.dtype == act &&
                 a.out_k.dtype == act && a.prev_k.dtype == act && a.prev_value.dtype == act,
             M3_ERR_DTYPE, "q, k, value, gate, output and the K/value caches must share one dtype");
  M3_REQUIRE(a.phase.dtype == M3_F32 && a.state.dtype == M3_F32 && a.out_phase.dtype == M3_F32 &&
                 a.out_state.dtype == M3_F32,
             M3_ERR_DTYPE, "phase and state must be float32");
  M3_REQUIRE(raw_dt || (a.adt.dtype == M3_F32 && a.dt.dtype == M3_F32), M3_ERR_DTYPE,
             "adt and dt must be float32 unless dt_bias is given");
  M3_REQUIRE(a.rank > 1 || !present(a.mimo_x), M3_ERR_ARGUMENT, "MIMO projections require rank > 1");
  M3_REQUIRE(a.out_phase.data != a.phase.data && a.out_k.data != a.prev_k.data, M3_ERR_LAYOUT,
             "output phase / k must not alias the input cache");
  const int64_t need = m3::step_workspace_bytes(a);
  M3_REQUIRE(need == 0 || (present(a.workspace) && a.workspace.dtype == M3_F32), M3_ERR_ARGUMENT,
             "a float32 workspace of m3_step_workspace_bytes() bytes is required");
  m3_step_args run = a;
  if (need == 0) run.workspace = m3_tensor{};
  const int dev_rc = select_device(a.device);
  if (dev_rc != M3_OK) return dev_rc;
  const cudaError_t e = m3::launch_step(run, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("step launch failed: ") + cudaGetErrorString(e));
  return M3_OK;
}

int64_t m3_scan_workspace_bytes(const m3_scan_args* args) {
  if (args == nullptr) return -fail(M3_ERR_ARGUMENT, "null argument struct");
  const m3_scan_args& a = *args;
  if (a.batch <= 0 || a.length <= 0 || a.heads <= 0 || a.groups <= 0 || a.rank <= 0 || a.num_angles < 0)
    return -fail(M3_ERR_SHAPE, "batch, length, heads, groups and rank must be positive");
  return m3::scan_umma_supported(a) ? m3::scan_umma_workspace_bytes(a) : 0;
}

int m3_scan_segments(const m3_scan_args* args) {
  if (args == nullptr) return -fail(M3_ERR_ARGUMENT, "null argument struct");
  if (args->batch <= 0 || args->length <= 0 || args->heads <= 0)
    return -fail(M3_ERR_SHAPE, "batch, length and heads must be positive");
  return m3::scan_umma_segments(*args);
}

int m3_scan_summary_floats(int rank) {
  if (rank != 1 && rank != 2 && rank != 4 && rank != 8) return -fail(M3_ERR_SHAPE, "rank must be 1, 2, 4 or 8");
  return m3::scan_summary_record_floats(rank);
}

int m3_scan_summary(const m3_scan_args* args, float* record, float* blocks, void* stream) {
  M3_REQUIRE(args != nullptr && record != nullptr, M3_ERR_ARGUMENT, "null argument");
  m3_scan_args a = *args;
  a.segments = 1;
  M3_REQUIRE(a.batch > 0 && a.length > 0 && a.heads > 0 && a.groups > 0, M3_ERR_SHAPE,
             "batch, length, heads and groups must be positive");
  M3_REQUIRE(!a.reverse, M3_ERR_ARGUMENT, "sequence summaries are forward scans");
  M3_REQUIRE(m3::scan_umma_supported(a), M3_ERR_LAYOUT,
             "sequence summaries need the tensor-core scan layout (bf16/fp16, d_state 128, head_dim 64, "
             "16-byte aligned contiguous rows)");
  M3_REQUIRE(a.angles.data == nullptr || a.length % 64 == 0 || blocks == nullptr, M3_ERR_SHAPE,
             "with in-kernel phases the summarised length must be a multiple of 64");
  M3_REQUIRE(a.angles.data == nullptr || blocks != nullptr, M3_ERR_ARGUMENT,
             "in-kernel phases need the block-total output");
  const int64_t need = m3::scan_umma_workspace_bytes(a);
  M3_REQUIRE(need == 0 || (present(a.workspace) && a.workspace.dtype == M3_F32), M3_ERR_ARGUMENT,
             "a float32 workspace of m3_scan_workspace_bytes() bytes (segments = 1) is required");
  const int dev_rc = select_device(a.device);
  if (dev_rc != M3_OK) return dev_rc;
  const cudaError_t e = m3::launch_scan_summary(a, record, blocks, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("summary launch failed: ") + cudaGetErrorString(e));
  return M3_OK;
}

int m3_scan_fwd(const m3_scan_args* args, void* stream) {
  M3_REQUIRE(args != nullptr, M3_ERR_ARGUMENT, "null argument struct");
  const m3_scan_args& a = *args;
  M3_REQUIRE(a.batch > 0 && a.length > 0 && a.heads > 0 && a.groups > 0 && a.head_dim > 0 && a.d_state > 0,
             M3_ERR_SHAPE, "batch, length, heads, groups, head_dim and d_state must be positive");
  M3_REQUIRE(a.heads % a.groups == 0, M3_ERR_SHAPE, "value heads must be divisible by Q/K groups");
  M3_REQUIRE(a.rank == 1 || a.rank == 2 || a.rank == 4 || a.rank == 8, M3_ERR_SHAPE, "rank must be 1, 2, 4 or 8");
  M3_REQUIRE(a.chunk_hint > 0, M3_ERR_SHAPE, "chunk_size must be positive");
  M3_REQUIRE(a.d_state <= 256 && a.head_dim <= 128, M3_ERR_SHAPE, "d_state <= 256 and head_dim <= 128 supported");
  const bool has_phase = present(a.phase) || present(a.angles);
  M3_REQUIRE(!(present(a.phase) && present(a.angles)), M3_ERR_ARGUMENT, "give either phase or angles, not both");
  M3_REQUIRE(!has_phase || (a.num_angles > 0 && a.num_angles <= 128 &&
                            2 * a.num_angles <= a.d_state),
             M3_ERR_SHAPE, "phase has too many angles for the Q/K state width");
  struct Item { const m3_tensor* t; const char* name; int nd; bool req; };
  const Item items[] = {
      {&a.q, "q", 5, true}, {&a.k, "k", 5, true}, {&a.q_norm_w, "q_norm_w", 1, false},
      {&a.k_norm_w, "k_norm_w", 1, false}, {&a.q_bias, "q_bias", 3, false}, {&a.k_bias, "k_bias", 3, false},
      {&a.value, "value", 4, true}, {&a.gate, "gate", 4, true}, {&a.adt, "adt", 3, true}, {&a.dt, "dt", 3, true},
      {&a.trap, "trap_logits", 3, true}, {&a.dt_bias, "dt_bias", 1, false}, {&a.phase, "phase", 4, false},
      {&a.angles, "angles", 3, false}, {&a.initial_phase, "initial_phase", 3, false}, {&a.D, "D", 1, true},
      {&a.mimo_x, "mimo_x", 3, a.rank > 1}, {&a.mimo_z, "mimo_z", 3, a.rank > 1},
      {&a.mimo_out, "mimo_out", 3, a.rank > 1}, {&a.initial_state, "initial_state", 4, false},
      {&a.initial_k, "initial_k", 4, false}, {&a.initial_value, "initial_value", 3, false},
      {&a.y, "output", 4, true}, {&a.final_state, "final_state", 4, true},
      {&a.final_phase, "final_phase", 3, false}, {&a.final_k, "final_k", 4, false},
      {&a.workspace, "workspace", 1, false}, {&a.y_reverse, "y_reverse", 4, a.reverse == 2},
  };
  for (const Item& it : items) {
    const int rc = check_tensor(*it.t, it.name, it.nd, it.req);
    if (rc != M3_OK) return rc;
  }
  M3_REQUIRE(a.reverse >= 0 && a.reverse <= 2, M3_ERR_ARGUMENT, "reverse must be 0, 1 or 2");
  if (a.reverse == 2) {
    bool same = a.y_reverse.dtype == a.y.dtype;
    for (int i = 0; i < 4; ++i) same = same && a.y_reverse.stride[i] == a.y.stride[i];
    M3_REQUIRE(same, M3_ERR_LAYOUT, "y_reverse must have the dtype and strides of y");
    M3_REQUIRE(!present(a.initial_state) && !present(a.initial_k) && !present(a.initial_phase) &&
                   !present(a.final_phase) && !present(a.final_k),
               M3_ERR_ARGUMENT, "the two-direction scan takes and returns no caches");
  }
  M3_REQUIRE(present(a.q_bias) == present(a.k_bias), M3_ERR_ARGUMENT, "q_bias and k_bias must be given together");
  M3_REQUIRE(present(a.q_norm_w) == present(a.k_norm_w), M3_ERR_ARGUMENT,
             "q_norm_w and k_norm_w must be given together");
  M3_REQUIRE(present(a.initial_k) == present(a.initial_value), M3_ERR_ARGUMENT,
             "initial_k and initial_value must be given together");
  M3_REQUIRE(a.rank > 1 || !present(a.mimo_x), M3_ERR_ARGUMENT, "SISO inputs must not provide MIMO projections");
  const int act = a.value.dtype;
  M3_REQUIRE(a.q.dtype == act && a.k.dtype == act && a.gate.dtype == act && a.y.dtype == act &&
                 (!present(a.final_k) || a.final_k.dtype == act),
             M3_ERR_DTYPE, "q, k, value, gate and output must share one dtype");
  M3_REQUIRE(a.final_state.dtype == M3_F32 && (!present(a.final_phase) || a.final_phase.dtype == M3_F32),
             M3_ERR_DTYPE, "state and phase outputs must be float32");
  M3_REQUIRE(!present(a.final_phase) || has_phase, M3_ERR_ARGUMENT, "final_phase requires phase or angles");
  M3_REQUIRE(!has_phase || !a.mimo_rotation || 4 * a.num_angles <= a.d_state, M3_ERR_SHAPE,
             "phase has too many angles for the Q/K state width");
  const int dev_rc = select_device(a.device);
  if (dev_rc != M3_OK) return dev_rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (m3::scan_umma_supported(a)) {
    const int64_t need = m3::scan_umma_workspace_bytes(a);
    M3_REQUIRE(need == 0 || (present(a.workspace) && a.workspace.dtype == M3_F32), M3_ERR_ARGUMENT,
               "a float32 workspace of m3_scan_workspace_bytes() bytes is required");
    g_last_scan_kernel = "umma";
    e = m3::launch_scan_umma(a, s);
  } else {
    M3_REQUIRE(m3::scan_simt_smem_bytes(a.rank, a.d_state, a.head_dim, a.num_angles) <= 227 * 1024,
               M3_ERR_SHAPE, "d_state x head_dim too large for the scan kernel");
    g_last_scan_kernel = "simt";
    if (a.reverse == 2) {  // two launches: backward first, so the forward one writes final_state last
      m3_scan_args bwd = a;
      bwd.reverse = 1;
      bwd.y = a.y_reverse;
      m3_scan_args fwd = a;
      fwd.reverse = 0;
      e = m3::launch_scan_simt(bwd, s);
      if (e == cudaSuccess) e = m3::launch_scan_simt(fwd, s);
    } else {
      e = m3::launch_scan_simt(a, s);
    }
  }
  if (e != cudaSuccess) return fail(M3_ERR_CUDA, std::string("scan launch failed: ") + cudaGetErrorString(e));
  return M3_OK;
}

}  // extern "C"
