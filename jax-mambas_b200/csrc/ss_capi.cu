// extern "C" entry points of libmamba_ss_b200.so (declared in
// include/mamba_selective_scan.h). They validate arguments the way the
// reference's FFI handlers do (native/selective_scan_cuda.cu:400-440,
// native/selective_scan_bwd.cu:45-79), launch on the caller's stream and
// report errors through a status code plus a per-thread message.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <string>

#include "ss_launch.h"

namespace {

thread_local std::string g_last_error;

// poll limit of the scan kernels' staging waits (test hook; see
// mamba_ss_debug_set_wait_polls)
std::atomic<uint32_t> g_wait_polls{mss::kWaitPolls};

// deterministic dB / dC (mamba_ss_set_deterministic)
std::atomic<int> g_deterministic{0};

mss_status fail(mss_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

mss_status cuda_fail(const char* what, cudaError_t e) {
  return fail(MSS_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

bool valid_dstate(int n) {
  return n == 1 || n == 2 || n == 4 || n == 8 || n == 16;
}

mss_status check_dims(const char* op, int io_dtype, int discretization,
                      int batch, int length, int dim, int dstate) {
  if (batch <= 0 || length <= 0 || dim <= 0)
    return fail(MSS_INVALID_ARGUMENT,
                std::string(op) + ": selective scan dimensions must be positive");
  if (!valid_dstate(dstate))
    return fail(MSS_INVALID_ARGUMENT,
                std::string(op) + ": N must be one of 1, 2, 4, 8, or 16");
  if (discretization != MSS_EULER && discretization != MSS_ZOH)
    return fail(MSS_INVALID_ARGUMENT,
                std::string(op) + ": discretization must be 0 (Euler) or 1 (ZOH)");
  if (io_dtype != MSS_F32 && io_dtype != MSS_BF16)
    return fail(MSS_INVALID_ARGUMENT,
                std::string(op) + ": io_dtype must be 0 (f32) or 1 (bf16)");
  if (static_cast<int64_t>(batch) * dim >= (1ll << 31) ||
      static_cast<int64_t>(dim) * dstate >= (1ll << 31))
    return fail(MSS_INVALID_ARGUMENT, std::string(op) + ": sizes too large");
  return MSS_OK;
}

int n_chunks_of(int length) { return (length + mss::kCkpt - 1) / mss::kCkpt; }

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct BwdWorkspace {
  int n_seg, seg_tiles;
  size_t dA_part, dD_part, dbias_part, seg_G, seg_dsum, seg_carry, dB_acc, dC_acc, B32, C32,
      dBC_part, total;
  int n_cols;
};

BwdWorkspace bwd_layout(int batch, int length, int dim, int dstate,
                        int io_dtype) {
  BwdWorkspace w{};
  const mss::SegPlan sp = mss::seg_plan(batch, length, dim, dstate);
  w.n_seg = sp.n_seg;
  w.seg_tiles = sp.seg_tiles;
  // per (segment, batch) partial sums of dA, dD, ddelta_bias
  const size_t sbd = static_cast<size_t>(sp.n_seg) * batch * dim;
  size_t off = 0;
  w.dA_part = off;
  off += align256(sizeof(float) * sbd * dstate);
  w.dD_part = off;
  off += align256(sizeof(float) * sbd);
  w.dbias_part = off;
  off += align256(sizeof(float) * sbd);
  w.seg_G = w.seg_dsum = w.seg_carry = 0;
  if (sp.n_seg > 1) {
    w.seg_G = off;
    off += align256(sizeof(float) * sbd * dstate);
    w.seg_dsum = off;
    off += align256(sizeof(float) * sbd);
    w.seg_carry = off;
    off += align256(sizeof(float) * sbd * dstate);
  }
  w.dB_acc = w.dC_acc = w.B32 = w.C32 = 0;
  if (io_dtype == MSS_BF16) {
    // fp32 accumulators of dB / dC, and B / C widened to fp32 for the kernels
    const size_t bnl =
        align256(sizeof(float) * static_cast<size_t>(batch) * dstate * length);
    w.dB_acc = off;
    off += bnl;
    w.dC_acc = off;
    off += bnl;
    w.B32 = off;
    off += bnl;
    w.C32 = off;
    off += bnl;
  }
  // deterministic mode: per warp-column partials of dB and dC
  w.dBC_part = 0;
  w.n_cols = (dim + mss::scan_channels_per_cta(dstate) - 1) / mss::scan_channels_per_cta(dstate);
  if (g_deterministic.load(std::memory_order_relaxed)) {
    w.dBC_part = off;
    off += align256(sizeof(float) * static_cast<size_t>(batch) * w.n_cols * 2 * dstate * length);
  }
  w.total = off;
  return w;
}

}  // namespace

namespace mss {
mss_status set_error(mss_status code, const std::string& msg) { return fail(code, msg); }

SegPlan seg_plan(int batch, int length, int dim, int dstate) {
  const int n_tiles = (length + kScanTile - 1) / kScanTile;
  const int ch = scan_channels_per_cta(dstate);
  const long long ctas = static_cast<long long>(batch) * ((dim + ch - 1) / ch);
  // Segments only when the grid is short of work: under about 9 one-warp
  // CTAs per SM (a configs[1] layer, 10.4 per SM, runs faster unsegmented:
  // the end-state and adjoint passes cost more than the added warps return).
  // Then many short segments: measured on configs[4]'s single sequence
  // (640 CTAs), 2 / 3 / 4 / 6 / 12 / 24 segments gave 20.5 / 24.2 / 23.2 /
  // 26.9 / 27.5 / 27.9 Gelem/s, i.e. finer, better balanced work units keep
  // paying long after one wave is full, and the extra passes' cost does not
  // grow with the count. So aim for about 100 CTAs per SM, with segments of
  // at least 8 tiles.
  constexpr long long kSegmentBelow = 148 * 9;
  constexpr long long kTarget = 148 * 100;
  int n = 1;
  if (const char* env = getenv("MAMBA_SS_SEGMENTS")) {
    n = std::max(1, atoi(env));
  } else if (ctas < kSegmentBelow) {
    const long long want = (kTarget + ctas - 1) / std::max(1LL, ctas);
    n = static_cast<int>(std::min<long long>(want, n_tiles / 8));
  }
  n = std::max(1, std::min(n, n_tiles));
  SegPlan sp;
  sp.seg_tiles = (n_tiles + n - 1) / n;
  sp.n_seg = (n_tiles + sp.seg_tiles - 1) / sp.seg_tiles;
  return sp;
}

size_t fwd_seg_scratch_elems(int batch, int length, int dim, int dstate) {
  const SegPlan sp = seg_plan(batch, length, dim, dstate);
  if (sp.n_seg <= 1) return 0;
  // end states and entering states (batch, dim, n_seg, dstate), delta sums
  const size_t bds = static_cast<size_t>(batch) * dim * sp.n_seg;
  return bds * (2 * static_cast<size_t>(dstate) + 1);
}
}  // namespace mss

extern "C" {

const char* mamba_ss_last_error(void) { return g_last_error.c_str(); }

const char* mamba_ss_version(void) { return "mamba-ss-b200 0.1 sm_100a"; }

uint32_t mamba_ss_take_device_error(void) {
  return mss::take_fwd_device_error() | mss::take_bwd_device_error();
}

int32_t mamba_ss_bounds_checked(void) {
#ifdef MSS_BOUNDS_CHECK
  return 1;
#else
  return 0;
#endif
}

uint64_t mamba_ss_take_bounds_violations(int64_t* first) {
  unsigned long long f[4], b[4];
  mss::take_fwd_bounds(f);
  mss::take_bwd_bounds(b);
  const unsigned long long* rec = f[0] != 0 ? f : b;
  if (first) {
    first[0] = static_cast<int64_t>(rec[1]);
    first[1] = static_cast<int64_t>(rec[2]);
    first[2] = static_cast<int64_t>(rec[3]);
  }
  return f[0] + b[0];
}

mss_status mamba_ss_bounds_selftest(void) {
  const cudaError_t e = mss::launch_bounds_selftest(1000);
  if (e != cudaSuccess)
    return mss::set_error(MSS_INTERNAL, std::string("bounds self-test: ") + cudaGetErrorString(e));
  return MSS_OK;
}

void mamba_ss_set_deterministic(int32_t on) {
  g_deterministic.store(on ? 1 : 0, std::memory_order_relaxed);
}

int32_t mamba_ss_deterministic(void) { return g_deterministic.load(std::memory_order_relaxed); }

void mamba_ss_debug_set_wait_polls(int64_t polls) {
  g_wait_polls.store(polls < 0 ? mss::kWaitPolls
                               : static_cast<uint32_t>(std::min<int64_t>(polls, mss::kWaitPolls)),
                     std::memory_order_relaxed);
}

int32_t mamba_ss_segments(int32_t batch, int32_t length, int32_t dim, int32_t dstate) {
  if (batch <= 0 || length <= 0 || dim <= 0 || dstate <= 0) return 0;
  return mss::seg_plan(batch, length, dim, dstate).n_seg;
}

int64_t mamba_ss_chunk_states_elems(int32_t batch, int32_t length, int32_t dim,
                                    int32_t dstate) {
  if (batch <= 0 || length <= 0 || dim <= 0 || dstate <= 0) return 0;
  return static_cast<int64_t>(batch) * dim * n_chunks_of(length) * dstate +
         static_cast<int64_t>(mss::fwd_seg_scratch_elems(batch, length, dim, dstate));
}

size_t mamba_ss_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                    int32_t dstate, int32_t io_dtype) {
  if (batch <= 0 || length <= 0 || dim <= 0 || dstate <= 0) return 0;
  return bwd_layout(batch, length, dim, dstate, io_dtype).total;
}

mss_status mamba_ss_fused_fwd(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    void* out, void* out_pre, float* last_state, float* chunk_states) {
  mss_status st = check_dims("mamba_ss_fused_fwd", io_dtype, discretization,
                             batch, length, dim, dstate);
  if (st != MSS_OK) return st;
  if (!u || !delta || !A || !B || !C || !out)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_fwd: u, delta, A, B, C and out must be non-null");
  if (reinterpret_cast<uintptr_t>(chunk_states) & 15)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_fused_fwd: chunk_states must be 16-byte aligned");
  mss::FwdParams p{};
  p.wait_polls = g_wait_polls.load(std::memory_order_relaxed);
  p.batch = batch;
  p.dim = dim;
  p.seqlen = length;
  p.n_chunks = n_chunks_of(length);
  p.delta_softplus = delta_softplus ? 1 : 0;
  p.u = u;
  p.delta = delta;
  p.z = z;
  p.B = B;
  p.C = C;
  p.A = A;
  p.D = D;
  p.delta_bias = delta_bias;
  p.h0 = initial_state;
  p.seq_lens = seq_lens;
  p.out = out;
  p.out_pre = out_pre;
  p.last_state = last_state;
  p.chunk_states = chunk_states;
  cudaError_t e = mss::launch_fwd(p, dstate, io_dtype, discretization,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching selective scan forward", e);
  return MSS_OK;
}

mss_status mamba_ss_fused_bwd(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const void* out_pre, const void* dout,
    const float* dlast_state, void* du, void* ddelta, float* dA, void* dB, void* dC, float* dD,
    void* dz, float* ddelta_bias, float* dinitial_state, void* workspace,
    size_t workspace_bytes) {
  mss_status st = check_dims("mamba_ss_fused_bwd", io_dtype, discretization,
                             batch, length, dim, dstate);
  if (st != MSS_OK) return st;
  if (!u || !delta || !A || !B || !C || !chunk_states || !dout || !du ||
      !ddelta || !dA || !dB || !dC)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_bwd: u, delta, A, B, C, chunk_states, dout, du, "
                "ddelta, dA, dB and dC must be non-null");
  if (reinterpret_cast<uintptr_t>(chunk_states) & 15)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_fused_bwd: chunk_states must be 16-byte aligned");
  if (z && (!dz || !out_pre))
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_bwd: z given without dz or out_pre");
  const BwdWorkspace w = bwd_layout(batch, length, dim, dstate, io_dtype);
  if (!workspace || workspace_bytes < w.total)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_bwd: workspace needs " + std::to_string(w.total) +
                    " bytes, got " + std::to_string(workspace_bytes));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_bwd: workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  mss::BwdParams p{};
  p.wait_polls = g_wait_polls.load(std::memory_order_relaxed);
  p.batch = batch;
  p.dim = dim;
  p.seqlen = length;
  p.n_chunks = n_chunks_of(length);
  p.delta_softplus = delta_softplus ? 1 : 0;
  p.u = u;
  p.delta = delta;
  p.z = z;
  p.B = B;
  p.C = C;
  p.A = A;
  p.D = D;
  p.delta_bias = delta_bias;
  p.h0 = initial_state;
  p.seq_lens = seq_lens;
  p.chunk_states = chunk_states;
  p.out_pre = out_pre;
  p.dout = dout;
  p.dlast = dlast_state;
  p.du = du;
  p.ddelta = ddelta;
  p.dz = z ? dz : nullptr;
  p.dA_part = reinterpret_cast<float*>(ws + w.dA_part);
  p.dD_part = reinterpret_cast<float*>(ws + w.dD_part);
  p.dbias_part = reinterpret_cast<float*>(ws + w.dbias_part);
  p.n_seg = w.n_seg;
  p.seg_tiles = w.seg_tiles;
  if (w.n_seg > 1) {
    p.seg_G = reinterpret_cast<float*>(ws + w.seg_G);
    p.seg_dsum = reinterpret_cast<float*>(ws + w.seg_dsum);
    p.seg_carry = reinterpret_cast<float*>(ws + w.seg_carry);
  }
  if (io_dtype == MSS_BF16) {
    p.dB_acc = reinterpret_cast<float*>(ws + w.dB_acc);
    p.dC_acc = reinterpret_cast<float*>(ws + w.dC_acc);
    p.B32 = reinterpret_cast<float*>(ws + w.B32);
    p.C32 = reinterpret_cast<float*>(ws + w.C32);
  } else {
    p.dB_acc = static_cast<float*>(dB);
    p.dC_acc = static_cast<float*>(dC);
    p.B32 = static_cast<float*>(const_cast<void*>(B));
    p.C32 = static_cast<float*>(const_cast<void*>(C));
  }
  p.dh0 = dinitial_state;
  p.n_cols = w.n_cols;
  p.dBC_part = w.dBC_part ? reinterpret_cast<float*>(ws + w.dBC_part) : nullptr;
  cudaError_t e = mss::launch_bwd(p, dstate, io_dtype, discretization, dB, dC,
                                  dA, D ? dD : nullptr,
                                  delta_bias ? ddelta_bias : nullptr,
                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching selective scan backward", e);
  return MSS_OK;
}

mss_status mamba_ss_fused_step(void* stream, int32_t io_dtype, int32_t discretization,
                               int32_t batch, int32_t dim, int32_t dstate, float* state,
                               const void* u, const void* delta, const float* A,
                               const void* B, const void* C, const float* D, const void* z,
                               const float* delta_bias, int32_t delta_softplus, void* out) {
  mss_status st = check_dims("mamba_ss_fused_step", io_dtype, discretization, batch, 1, dim,
                             dstate);
  if (st != MSS_OK) return st;
  if (!state || !u || !delta || !A || !B || !C || !out)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_fused_step: state, u, delta, A, B, C and out must be non-null");
  if (reinterpret_cast<uintptr_t>(state) & 15)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_fused_step: state must be 16-byte aligned");
  mss::StepParams p{};
  p.batch = batch;
  p.dim = dim;
  p.delta_softplus = delta_softplus ? 1 : 0;
  p.state = state;
  p.u = u;
  p.delta = delta;
  p.z = z;
  p.B = B;
  p.C = C;
  p.A = A;
  p.D = D;
  p.delta_bias = delta_bias;
  p.out = out;
  cudaError_t e = mss::launch_step(p, dstate, io_dtype, discretization,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching selective scan step", e);
  return MSS_OK;
}

mss_status mamba_ss_fwd(void* stream, int32_t discretization, int32_t batch,
                        int32_t length, int32_t dim, int32_t dstate,
                        const float* A, const float* deltas, const float* B,
                        const float* C, const float* u, const float* initial_x,
                        float* y, float* final_x, float* chunk_states) {
  return mamba_ss_fused_fwd(stream, MSS_F32, discretization, batch, length, dim,
                            dstate, u, deltas, A, B, C, nullptr, nullptr,
                            nullptr, 0, initial_x, nullptr, y, nullptr, final_x,
                            chunk_states);
}

mss_status mamba_ss_fwd_bench(void* stream, int32_t discretization,
                              int32_t repeats, int32_t batch, int32_t length,
                              int32_t dim, int32_t dstate, const float* A,
                              const float* deltas, const float* B,
                              const float* C, const float* u,
                              const float* initial_x, float* y, float* final_x,
                              float* chunk_states) {
  if (repeats <= 0)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_fwd_bench: repeats must be positive");
  for (int r = 0; r < repeats; ++r) {
    mss_status st = mamba_ss_fwd(stream, discretization, batch, length, dim,
                                 dstate, A, deltas, B, C, u, initial_x, y,
                                 final_x, chunk_states);
    if (st != MSS_OK) return st;
  }
  return MSS_OK;
}

mss_status mamba_ss_bwd(void* stream, int32_t discretization, int32_t batch,
                        int32_t length, int32_t dim, int32_t dstate,
                        const float* A, const float* deltas, const float* B,
                        const float* C, const float* u, const float* initial_x,
                        const float* chunk_states, const float* dy,
                        const float* dfinal_x, float* dA, float* ddeltas,
                        float* dB, float* dC, float* du, float* dinitial_x,
                        void* workspace, size_t workspace_bytes) {
  return mamba_ss_fused_bwd(stream, MSS_F32, discretization, batch, length, dim,
                            dstate, u, deltas, A, B, C, nullptr, nullptr,
                            nullptr, 0, initial_x, nullptr, chunk_states, nullptr,
                            dy, dfinal_x, du, ddeltas, dA, dB, dC, nullptr, nullptr,
                            nullptr, dinitial_x, workspace, workspace_bytes);
}

size_t mamba_ss_conv1d_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                           int32_t kwidth) {
  if (batch <= 0 || length <= 0 || dim <= 0 || kwidth <= 0) return 0;
  const size_t bd = static_cast<size_t>(batch) * mss::conv_segments(length) * dim;
  return align256(sizeof(float) * bd * kwidth) + align256(sizeof(float) * bd);
}

static mss_status check_conv(const char* op, int32_t io_dtype, int32_t batch, int32_t length,
                             int32_t dim, int32_t kwidth) {
  if (io_dtype != MSS_F32 && io_dtype != MSS_BF16)
    return fail(MSS_INVALID_ARGUMENT, std::string(op) + ": io_dtype must be 0 (f32) or 1 (bf16)");
  if (batch <= 0 || length <= 0 || dim <= 0)
    return fail(MSS_INVALID_ARGUMENT, std::string(op) + ": batch, length and dim must be positive");
  if (kwidth < 1 || kwidth > 4)
    return fail(MSS_INVALID_ARGUMENT, std::string(op) + ": kwidth must be 1 .. 4");
  if (static_cast<int64_t>(batch) * dim >= (1ll << 31))
    return fail(MSS_INVALID_ARGUMENT, std::string(op) + ": sizes too large");
  return MSS_OK;
}

mss_status mamba_ss_conv1d_fwd(void* stream, int32_t io_dtype, int32_t batch, int32_t length,
                               int32_t dim, int32_t kwidth, const void* x,
                               const float* weight, const float* bias,
                               const int32_t* seq_lens, const void* conv_state, void* u,
                               void* final_state) {
  mss_status st = check_conv("mamba_ss_conv1d_fwd", io_dtype, batch, length, dim, kwidth);
  if (st != MSS_OK) return st;
  if (!x || !weight || !u)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_conv1d_fwd: x, weight and u must be non-null");
  mss::ConvParams p{};
  p.batch = batch;
  p.dim = dim;
  p.seqlen = length;
  p.x = x;
  p.weight = weight;
  p.bias = bias;
  p.seq_lens = seq_lens;
  p.state_in = kwidth > 1 ? conv_state : nullptr;
  p.u = u;
  p.state_out = kwidth > 1 ? final_state : nullptr;
  cudaError_t e = mss::launch_conv(p, kwidth, io_dtype, false, nullptr, nullptr,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching causal conv1d forward", e);
  return MSS_OK;
}

mss_status mamba_ss_conv1d_bwd(void* stream, int32_t io_dtype, int32_t batch, int32_t length,
                               int32_t dim, int32_t kwidth, const void* x,
                               const float* weight, const float* bias,
                               const int32_t* seq_lens, const void* conv_state,
                               const void* du, void* dx, float* dweight, float* dbias,
                               void* dconv_state, void* workspace, size_t workspace_bytes) {
  mss_status st = check_conv("mamba_ss_conv1d_bwd", io_dtype, batch, length, dim, kwidth);
  if (st != MSS_OK) return st;
  if (!x || !weight || !du || !dx || !dweight)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_conv1d_bwd: x, weight, du, dx and dweight must be non-null");
  const size_t need = mamba_ss_conv1d_bwd_workspace_bytes(batch, length, dim, kwidth);
  if (!workspace || workspace_bytes < need)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_conv1d_bwd: workspace needs " +
                                          std::to_string(need) + " bytes, got " +
                                          std::to_string(workspace_bytes));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_conv1d_bwd: workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  mss::ConvParams p{};
  p.batch = batch;
  p.dim = dim;
  p.seqlen = length;
  p.x = x;
  p.weight = weight;
  p.bias = bias;
  p.seq_lens = seq_lens;
  p.state_in = kwidth > 1 ? conv_state : nullptr;
  p.du = du;
  p.dx = dx;
  p.dstate_in = kwidth > 1 ? dconv_state : nullptr;
  p.dw_part = reinterpret_cast<float*>(ws);
  p.db_part = reinterpret_cast<float*>(
      ws + align256(sizeof(float) * static_cast<size_t>(batch) * mss::conv_segments(length) *
                    dim * kwidth));
  cudaError_t e = mss::launch_conv(p, kwidth, io_dtype, true, dweight, bias ? dbias : nullptr,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching causal conv1d backward", e);
  return MSS_OK;
}

mss_status mamba_ss_conv1d_step(void* stream, int32_t io_dtype, int32_t batch, int32_t dim,
                                int32_t kwidth, const void* x, const float* weight,
                                const float* bias, void* conv_state, void* u) {
  mss_status st = check_conv("mamba_ss_conv1d_step", io_dtype, batch, 1, dim, kwidth);
  if (st != MSS_OK) return st;
  if (!x || !weight || !u || (kwidth > 1 && !conv_state))
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_conv1d_step: x, weight, u and (kwidth > 1) conv_state must be non-null");
  mss::ConvParams p{};
  p.batch = batch;
  p.dim = dim;
  p.seqlen = 1;
  p.x = x;
  p.weight = weight;
  p.bias = bias;
  p.u = u;
  p.state_out = conv_state;
  cudaError_t e = mss::launch_conv_step(p, kwidth, io_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching causal conv1d step", e);
  return MSS_OK;
}

int64_t mamba_ss_complex_chunk_states_elems(int32_t batch, int32_t length, int32_t dim,
                                            int32_t dstate) {
  if (batch <= 0 || length <= 0 || dim <= 0 || dstate <= 0) return 0;
  return 2 * static_cast<int64_t>(batch) * dim * n_chunks_of(length) * dstate;
}

size_t mamba_ss_complex_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                            int32_t dstate) {
  if (batch <= 0 || length <= 0 || dim <= 0 || dstate <= 0) return 0;
  const size_t bd = static_cast<size_t>(batch) * dim;
  const size_t bnl = static_cast<size_t>(batch) * dstate * length;
  return align256(sizeof(float) * bd * dstate * 2) + 2 * align256(sizeof(float) * bd) +
         4 * align256(sizeof(float) * bnl);
}

static mss::CplxParams complex_params(int32_t batch, int32_t length, int32_t dim,
                                      const float* u, const float* delta, const void* A,
                                      const void* B, const void* C, const float* D,
                                      const float* z, const float* delta_bias,
                                      int32_t delta_softplus, const void* initial_state,
                                      const int32_t* seq_lens) {
  mss::CplxParams p{};
  p.batch = batch;
  p.dim = dim;
  p.seqlen = length;
  p.n_chunks = n_chunks_of(length);
  p.delta_softplus = delta_softplus ? 1 : 0;
  p.u = u;
  p.delta = delta;
  p.z = z;
  p.A = A;
  p.B = B;
  p.C = C;
  p.D = D;
  p.delta_bias = delta_bias;
  p.h0 = initial_state;
  p.seq_lens = seq_lens;
  return p;
}

mss_status mamba_ss_complex_fwd(void* stream, int32_t discretization, int32_t batch,
                                int32_t length, int32_t dim, int32_t dstate, const float* u,
                                const float* delta, const void* A, const void* B, const void* C,
                                const float* D, const float* z, const float* delta_bias,
                                int32_t delta_softplus, const void* initial_state,
                                const int32_t* seq_lens, float* out, float* out_pre,
                                void* last_state, float* chunk_states) {
  mss_status st = check_dims("mamba_ss_complex_fwd", MSS_F32, discretization, batch, length,
                             dim, dstate);
  if (st != MSS_OK) return st;
  if (!u || !delta || !A || !B || !C || !out || !chunk_states)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_complex_fwd: u, delta, A, B, C, out and chunk_states must be non-null");
  mss::CplxParams p = complex_params(batch, length, dim, u, delta, A, B, C, D, z, delta_bias,
                                     delta_softplus, initial_state, seq_lens);
  p.out = out;
  p.out_pre = out_pre;
  p.last_state = last_state;
  p.chunk_states = chunk_states;
  cudaError_t e = mss::launch_cplx_fwd(p, dstate, discretization,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching complex selective scan forward", e);
  return MSS_OK;
}

mss_status mamba_ss_complex_bwd(
    void* stream, int32_t discretization, int32_t batch, int32_t length, int32_t dim,
    int32_t dstate, const float* u, const float* delta, const void* A, const void* B,
    const void* C, const float* D, const float* z, const float* delta_bias,
    int32_t delta_softplus, const void* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const float* out_pre, const float* dout, const void* dlast_state,
    float* du, float* ddelta, void* dA, void* dB, void* dC, float* dD, float* dz,
    float* ddelta_bias, void* dinitial_state, void* workspace, size_t workspace_bytes) {
  mss_status st = check_dims("mamba_ss_complex_bwd", MSS_F32, discretization, batch, length,
                             dim, dstate);
  if (st != MSS_OK) return st;
  if (!u || !delta || !A || !B || !C || !chunk_states || !dout || !du || !ddelta || !dA ||
      !dB || !dC)
    return fail(MSS_INVALID_ARGUMENT,
                "mamba_ss_complex_bwd: u, delta, A, B, C, chunk_states, dout, du, ddelta, dA, "
                "dB and dC must be non-null");
  if (z && (!dz || !out_pre))
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_complex_bwd: z given without dz or out_pre");
  const size_t need = mamba_ss_complex_bwd_workspace_bytes(batch, length, dim, dstate);
  if (!workspace || workspace_bytes < need)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_complex_bwd: workspace needs " +
                                          std::to_string(need) + " bytes, got " +
                                          std::to_string(workspace_bytes));
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(MSS_INVALID_ARGUMENT, "mamba_ss_complex_bwd: workspace must be 256-byte aligned");
  mss::CplxParams p = complex_params(batch, length, dim, u, delta, A, B, C, D, z, delta_bias,
                                     delta_softplus, initial_state, seq_lens);
  p.chunk_states = const_cast<float*>(chunk_states);
  p.out_pre = const_cast<float*>(out_pre);
  p.dout = dout;
  p.dlast = dlast_state;
  p.du = du;
  p.ddelta = ddelta;
  p.dz = z ? dz : nullptr;
  p.dh0 = dinitial_state;
  const size_t bd = static_cast<size_t>(batch) * dim;
  const size_t bnl = static_cast<size_t>(batch) * dstate * length;
  char* ws = static_cast<char*>(workspace);
  size_t off = 0;
  p.dA_part = reinterpret_cast<float*>(ws + off);
  off += align256(sizeof(float) * bd * dstate * 2);
  p.dD_part = reinterpret_cast<float*>(ws + off);
  off += align256(sizeof(float) * bd);
  p.dbias_part = reinterpret_cast<float*>(ws + off);
  off += align256(sizeof(float) * bd);
  float** planes[4] = {&p.dB_acc_r, &p.dB_acc_i, &p.dC_acc_r, &p.dC_acc_i};
  for (float** pl : planes) {
    *pl = reinterpret_cast<float*>(ws + off);
    off += align256(sizeof(float) * bnl);
  }
  cudaError_t e = mss::launch_cplx_bwd(p, dstate, discretization, dA, dB, dC, D ? dD : nullptr,
                                       delta_bias ? ddelta_bias : nullptr,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail("launching complex selective scan backward", e);
  return MSS_OK;
}

}  // extern "C"
