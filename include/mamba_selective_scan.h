/*
 * C ABI of the B200 (sm_100a) Mamba-1 selective scan.
 *
 * These entry points replace the XLA typed-FFI handlers of the JAX-Mambas
 * reference (MambaSelectiveScan, MambaSelectiveScanBackward and
 * MambaSelectiveScanBenchmark in native/selective_scan_cuda.cu and
 * native/selective_scan_bwd.cu). Arguments are plain device pointers, sizes
 * and a cudaStream_t passed as void*; nothing here allocates device memory or
 * synchronises the host. Every function returns an mss_status; on failure
 * mamba_ss_last_error() gives a message for the calling host thread.
 *
 * Physical layouts (row-major, last index fastest):
 *   u, delta, z, y / out, du, ddelta, dz, dy ... (batch, dim, length)
 *   B, C, dB, dC ............................... (batch, dstate, length)
 *   A, dA ...................................... (dim, dstate)        fp32
 *   D, delta_bias, dD, ddelta_bias ............. (dim)                fp32
 *   initial_state, last_state, d_* ............. (batch, dim, dstate) fp32
 *   chunk_states ............................... batch*n_chunks*dim*dstate fp32,
 *                                                  16-byte aligned; layout private
 *   seq_lens ................................... (batch) int32
 * These are the physical layouts the reference pins through its ffi_call
 * input_layouts/output_layouts (mamba/selective_scan_cuda.py:138-146,180-198).
 */
#ifndef MAMBA_SELECTIVE_SCAN_H_
#define MAMBA_SELECTIVE_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MSS_OK = 0,
  MSS_INVALID_ARGUMENT = 1, /* like ffi::Error::InvalidArgument, cu:402-440 */
  MSS_INTERNAL = 2          /* like ffi::Error::Internal, cu:334-337 */
} mss_status;

typedef enum { MSS_F32 = 0, MSS_BF16 = 1 } mss_dtype;

typedef enum { MSS_EULER = 0, MSS_ZOH = 1 } mss_discretization;

/* Time steps covered by one saved carry (one entry of chunk_states). */
#define MSS_CHUNK 4

/* Message of the last failed call on this host thread ("" if none). */
const char* mamba_ss_last_error(void);

/* Library version string, e.g. "mamba-ss-b200 0.1 sm_100a". */
const char* mamba_ss_version(void);

/* Returns and clears the device-side error word of the current device:
 * bit 0 = a kernel gave up waiting (bounded) for its TMA copies and returned
 * early, so its outputs are incomplete. Synchronous; no counterpart in the
 * reference, whose kernels have no waits. */
uint32_t mamba_ss_take_device_error(void);

/* Debug bounds build (libmamba_ss_b200_bounds.so, compiled with
 * -DMSS_BOUNDS_CHECK; CMake option MAMBA_SS_DEBUG_BOUNDS). Its forward and
 * backward scan kernels check every computed global index, and every TMA
 * store coordinate, against the extent of its array before the access; an
 * index outside it is counted and the access skipped instead of faulting.
 * No counterpart in the reference, which has no such build; it stands in
 * for compute-sanitizer, which is not available on every machine.
 *   mamba_ss_bounds_checked()  1 in the bounds build, 0 in the normal one.
 *   mamba_ss_take_bounds_violations(first)  synchronous; returns and clears
 *     the number of violations since the last call; if first is not NULL it
 *     receives {site, index, extent} of the first one (site numbers are the
 *     BoundsSite values of csrc/ss_common.cuh). Always 0 in the normal build.
 *   mamba_ss_bounds_selftest()  launches one thread that checks an index
 *     past its extent without any memory access, so that the next
 *     mamba_ss_take_bounds_violations() returns 1 with site 99 in the bounds
 *     build (0 in the normal one). */
int32_t mamba_ss_bounds_checked(void);
uint64_t mamba_ss_take_bounds_violations(int64_t* first);
mss_status mamba_ss_bounds_selftest(void);

/* Deterministic dB and dC (process-wide, default off). The backward sums
 * dB and dC over channels; by default every warp adds its 8-channel sum into
 * fp32 accumulators with atomics, so the order of the additions, and the last
 * bits of dB / dC, vary from run to run (as the reference's per-element
 * atomicAdd, native/upstream_mamba/selective_scan_bwd_kernel.cuh:315-316).
 * With deterministic mode on, each warp writes its sum to a partial buffer
 * of the workspace (batch * ceil(dim / channels per warp) * 2 * dstate *
 * length fp32) and a second kernel adds the partials in a fixed order, so dB
 * and dC are bitwise reproducible; every other output already is. It costs
 * that extra traffic (measured: configs[2] backward 3.55 -> 4.32 ms,
 * configs[1] 0.51 -> 0.60 ms). It changes
 * mamba_ss_bwd_workspace_bytes: query the size after setting the mode. The
 * complex scan is not affected. */
void mamba_ss_set_deterministic(int32_t on);
int32_t mamba_ss_deterministic(void);

/* Test hook for the bounded waits: sets the number of polls after which
 * the scan kernels launched from now on (any host thread) give up waiting
 * for a tile's TMA staging, report bit 0 through
 * mamba_ss_take_device_error() and return with incomplete outputs (they
 * still let their copies in flight land first). 0 makes every such wait
 * give up at once; a negative value restores the default (2^22 polls, far
 * longer than any copy takes). No counterpart in the reference, whose
 * kernels do not wait on copies. */
void mamba_ss_debug_set_wait_polls(int64_t polls);

/* Number of time segments the launcher cuts each sequence into for this
 * problem (1 = none; more when there are too few (batch, channel-block) work
 * units to fill the GPU, or as forced by MAMBA_SS_SEGMENTS). Each segment
 * count above 1 adds an end-state pass and a combine to the forward and an
 * adjoint pass and a combine to the backward. No counterpart in the
 * reference, whose kernels always walk the whole sequence per block. */
int32_t mamba_ss_segments(int32_t batch, int32_t length, int32_t dim, int32_t dstate);

/* Number of fp32 elements of chunk_states: batch*dim*ceil(length/4)*dstate.
 * The reference sizes the same residual (batch, dim, ceil(L/2048), N, 2)
 * (mamba/selective_scan_cuda.py:129-134); it is private to the custom_vjp. */
int64_t mamba_ss_chunk_states_elems(int32_t batch, int32_t length, int32_t dim,
                                    int32_t dstate);

/* ---------------------------------------------------------------------------
 * Reference contract (fp32, no D / z / bias / softplus in the kernel).
 * ------------------------------------------------------------------------- */

/* Replaces MambaSelectiveScan (native/selective_scan_cuda.cu:554-573):
 * attrs discretization, batch, length, dim, dstate; args A, deltas, B, C, u,
 * initial_x; rets y, final_x, chunk_states. */
mss_status mamba_ss_fwd(void* stream, int32_t discretization, int32_t batch,
                        int32_t length, int32_t dim, int32_t dstate,
                        const float* A, const float* deltas, const float* B,
                        const float* C, const float* u, const float* initial_x,
                        float* y, float* final_x, float* chunk_states);

/* Replaces MambaSelectiveScanBenchmark (native/selective_scan_cuda.cu:578-598):
 * the forward launched `repeats` times behind one call. */
mss_status mamba_ss_fwd_bench(void* stream, int32_t discretization,
                              int32_t repeats, int32_t batch, int32_t length,
                              int32_t dim, int32_t dstate, const float* A,
                              const float* deltas, const float* B,
                              const float* C, const float* u,
                              const float* initial_x, float* y, float* final_x,
                              float* chunk_states);

/* Bytes of caller-provided scratch the backward needs (both contracts). */
size_t mamba_ss_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                    int32_t dstate, int32_t io_dtype);

/* Replaces MambaSelectiveScanBackward (native/selective_scan_bwd.cu:166-190):
 * attrs batch, length, dim, dstate; args A, deltas, B, C, u, initial_x,
 * chunk_states, dy, dfinal_x; rets dA, ddeltas, dB, dC, du, dinitial_x.
 * The reference backward is Euler-only and falls back to JAX autodiff for
 * ZOH (mamba/selective_scan_cuda.py:236-256); this one takes discretization
 * as well. workspace must hold mamba_ss_bwd_workspace_bytes(...,MSS_F32). */
mss_status mamba_ss_bwd(void* stream, int32_t discretization, int32_t batch,
                        int32_t length, int32_t dim, int32_t dstate,
                        const float* A, const float* deltas, const float* B,
                        const float* C, const float* u, const float* initial_x,
                        const float* chunk_states, const float* dy,
                        const float* dfinal_x, float* dA, float* ddeltas,
                        float* dB, float* dC, float* du, float* dinitial_x,
                        void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Fused contract: selective_scan(u, delta, A, B, C, D, z, delta_bias,
 * delta_softplus, return_last_state) of the north-star signature, plus
 * initial_state, discretization and per-sequence valid lengths.
 *   delta_eff = softplus(delta + delta_bias)  (softplus if delta_softplus)
 *   h_t = exp(delta_eff*A) h_{t-1} + delta_eff*B_t*u_t          (Euler)
 *   out = (sum_n C_t h_t + D*u) * silu(z)
 * Optional pointers (D, z, delta_bias, initial_state, seq_lens, last_state,
 * dfinal_state and their gradients) may be NULL. out_pre receives the
 * pre-gate output y + D*u (io_dtype, same layout as out); the backward needs
 * it whenever z is given, and it may be NULL when z is NULL. With seq_lens, steps
 * t >= seq_lens[b] are padding: their delta and u count as 0, their output
 * and input gradients are written as exact zeros.
 * io_dtype (MSS_F32 or MSS_BF16) types u, delta, z, B, C, out and their
 * gradients; the state, A, D, delta_bias and reductions stay fp32.
 * chunk_states (the saved carries the backward reads) may be NULL in the
 * forward when no backward follows; the scan then also runs without time
 * segments.
 * ------------------------------------------------------------------------- */
mss_status mamba_ss_fused_fwd(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    void* out, void* out_pre, float* last_state, float* chunk_states);

mss_status mamba_ss_fused_bwd(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const void* out_pre, const void* dout,
    const float* dlast_state,
    void* du, void* ddelta, float* dA, void* dB, void* dC, float* dD,
    void* dz, float* ddelta_bias, float* dinitial_state, void* workspace,
    size_t workspace_bytes);

/* One recurrent decode step: the state update of S6.step / Mamba.step
 * (mamba/mamba1.py:200-214; pure JAX in the reference, no FFI counterpart).
 * For one new token per sequence: u, delta, z, out are (batch, dim), B, C
 * (batch, dstate) in io_dtype; state (batch, dim, dstate) fp32 is updated in
 * place (16-byte aligned); A, D, delta_bias as in mamba_ss_fused_fwd. */
mss_status mamba_ss_fused_step(void* stream, int32_t io_dtype, int32_t discretization,
                               int32_t batch, int32_t dim, int32_t dstate, float* state,
                               const void* u, const void* delta, const float* A,
                               const void* B, const void* C, const float* D, const void* z,
                               const float* delta_bias, int32_t delta_softplus, void* out);

/* ---------------------------------------------------------------------------
 * Complex SSM (S6 with complex_ssm = True, mamba/mamba1.py:170-176, 196;
 * pure JAX in the reference, no FFI counterpart): A (dim, dstate), B, C
 * (batch, dstate, length), initial/last state and its gradient (batch, dim,
 * dstate) are complex64 (interleaved float pairs); u, delta, z, out, out_pre,
 * dout and the other gradients are fp32 (batch, dim, length);
 * out = (Re(C . h) + D u) * silu(z). Gradients of complex arguments are
 * dL/dRe + i dL/dIm (torch's convention; JAX's cotangent is the conjugate).
 * chunk_states holds complex carries (mamba_ss_complex_chunk_states_elems
 * floats); the backward needs mamba_ss_complex_bwd_workspace_bytes of
 * 256-byte aligned workspace.
 * ------------------------------------------------------------------------- */
int64_t mamba_ss_complex_chunk_states_elems(int32_t batch, int32_t length, int32_t dim,
                                            int32_t dstate);
size_t mamba_ss_complex_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                            int32_t dstate);

mss_status mamba_ss_complex_fwd(void* stream, int32_t discretization, int32_t batch,
                                int32_t length, int32_t dim, int32_t dstate, const float* u,
                                const float* delta, const void* A, const void* B, const void* C,
                                const float* D, const float* z, const float* delta_bias,
                                int32_t delta_softplus, const void* initial_state,
                                const int32_t* seq_lens, float* out, float* out_pre,
                                void* last_state, float* chunk_states);

mss_status mamba_ss_complex_bwd(
    void* stream, int32_t discretization, int32_t batch, int32_t length, int32_t dim,
    int32_t dstate, const float* u, const float* delta, const void* A, const void* B,
    const void* C, const float* D, const float* z, const float* delta_bias,
    int32_t delta_softplus, const void* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const float* out_pre, const float* dout, const void* dlast_state,
    float* du, float* ddelta, void* dA, void* dB, void* dC, float* dD, float* dz,
    float* ddelta_bias, void* dinitial_state, void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Causal depthwise conv1d + bias + SiLU + padding mask: the operation between
 * the input projection and the scan in Mamba.__call__ (mamba/mamba1.py:
 * 313-329: projed *= mask; silu(nnx.Conv(feature_group_count = d_inner,
 * padding = CAUSAL)(cache ++ projed)) * mask; the conv at mamba1.py:250-255).
 * Pure JAX / flax in the reference, no FFI counterpart.
 *
 * x, u, du, dx: (batch, dim, length) in io_dtype (the scan's layout);
 * weight, dweight: (kwidth, dim) fp32 (flax's (kwidth, 1, dim) kernel);
 * bias, dbias: (dim) fp32 or NULL; seq_lens: (batch) or NULL (steps at or past
 * a sequence's length are masked: inputs read as 0, outputs written as 0);
 * conv_state, final_state, dconv_state: (batch, dim, kwidth - 1) in io_dtype
 * or NULL: the kwidth - 1 (masked) inputs before t = 0 (the reference's conv
 * cache, time-major there), the last kwidth - 1 masked inputs after this
 * call, and the gradient of conv_state. 1 <= kwidth <= 4.
 * ------------------------------------------------------------------------- */
size_t mamba_ss_conv1d_bwd_workspace_bytes(int32_t batch, int32_t length, int32_t dim,
                                           int32_t kwidth);

mss_status mamba_ss_conv1d_fwd(void* stream, int32_t io_dtype, int32_t batch, int32_t length,
                               int32_t dim, int32_t kwidth, const void* x,
                               const float* weight, const float* bias,
                               const int32_t* seq_lens, const void* conv_state, void* u,
                               void* final_state);

mss_status mamba_ss_conv1d_bwd(void* stream, int32_t io_dtype, int32_t batch, int32_t length,
                               int32_t dim, int32_t kwidth, const void* x,
                               const float* weight, const float* bias,
                               const int32_t* seq_lens, const void* conv_state,
                               const void* du, void* dx, float* dweight, float* dbias,
                               void* dconv_state, void* workspace, size_t workspace_bytes);

/* One decode token of the conv (Mamba.step, mamba/mamba1.py:339-355):
 * x, u (batch, dim); conv_state (batch, dim, kwidth - 1) holds the last
 * kwidth - 1 inputs and is shifted in place (the reference's cache update,
 * mamba1.py:351-352); u = silu(bias + sum_k weight[k] * (conv_state ++ x)[k]). */
mss_status mamba_ss_conv1d_step(void* stream, int32_t io_dtype, int32_t batch, int32_t dim,
                                int32_t kwidth, const void* x, const float* weight,
                                const float* bias, void* conv_state, void* u);

/* ---------------------------------------------------------------------------
 * Allocation-free backward. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory (a host runtime that owns
 * all device memory and only passes tensor pointers across its FFI, or code
 * running where cudaMalloc is not allowed): same arguments and results as
 * mamba_ss_fused_bwd minus the workspace, which comes instead from a fixed
 * 16 MiB array inside the library (mamba_ss_noalloc_scratch_bytes()), held on
 * every GPU that loads the library until the process exits. Problems needing
 * more scratch than that (mamba_ss_bwd_workspace_bytes) are rejected with
 * MSS_INVALID_ARGUMENT. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture. All calls on a device share the
 * array, so calls whose GPU work overlaps (unordered streams) race and give
 * wrong results. Nothing is allocated or freed.
 * ------------------------------------------------------------------------- */
size_t mamba_ss_noalloc_scratch_bytes(void);

mss_status mamba_ss_fused_bwd_noalloc(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const void* out_pre, const void* dout,
    const float* dlast_state, void* du, void* ddelta, float* dA, void* dB,
    void* dC, float* dD, void* dz, float* ddelta_bias, float* dinitial_state);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_SELECTIVE_SCAN_H_ */
