// Host-side launchers shared by the C ABI (ss_capi.cu).
#pragma once

#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <string>

#include "ss_common.cuh"

namespace mss {

// Steps per tile of both scan kernels.
constexpr int kScanTile = 32;

// Channels per CTA of both scan kernels (8 for N = 16).
inline int scan_channels_per_cta(int dstate) {
  const int s = dstate < 4 ? dstate : 4;  // states per lane
  const int cpw = 32 / (dstate / s);      // channels per warp
  return cpw < 8 ? 8 : cpw;
}

// Time segments of a scan: when a problem has too few (batch, channel-block)
// CTAs to fill the GPU (a single long sequence), L is cut into n_seg segments
// of seg_tiles tiles that run in parallel; a light pass finds each segment's
// entering state (forward) or adjoint (backward) first. The environment
// variable MAMBA_SS_SEGMENTS forces a segment count (tests).
struct SegPlan {
  int n_seg;      // >= 1
  int seg_tiles;  // tiles per segment (the last may be shorter)
};
SegPlan seg_plan(int batch, int length, int dim, int dstate);

// fp32 elements of the segment scratch the forward keeps after the carries
// in chunk_states (0 when n_seg == 1).
size_t fwd_seg_scratch_elems(int batch, int length, int dim, int dstate);

cudaError_t launch_fwd(const FwdParams& p, int dstate, int io_dtype, int zoh,
                       cudaStream_t stream);

// Runs the backward scan kernel, the batch reduction of the parameter
// gradients and (bf16 I/O) the fp32 -> bf16 conversion of dB/dC.
// dB_out/dC_out are the caller's output buffers; p.dB_acc/p.dC_acc are the
// fp32 accumulators (the outputs themselves for fp32 I/O).
cudaError_t launch_bwd(const BwdParams& p, int dstate, int io_dtype, int zoh,
                       void* dB_out, void* dC_out, float* dA, float* dD,
                       float* ddelta_bias, cudaStream_t stream);

// Causal conv1d + SiLU forward, or backward (then also the batch reduction
// of dweight / dbias from p.dw_part / p.db_part).
cudaError_t launch_conv(const ConvParams& p, int kwidth, int io_dtype, bool backward,
                        float* dweight, float* dbias, cudaStream_t stream);

// Segments per row of the conv kernels (their dweight / dbias partials are
// per (batch, segment)).
int conv_segments(int length);

// One decode token of the conv: p.x, p.u (batch, dim), p.state_out the conv
// state (batch, dim, kwidth - 1), shifted in place.
cudaError_t launch_conv_step(const ConvParams& p, int kwidth, int io_dtype, cudaStream_t stream);

// Complex scan: forward; backward incl. the batch reductions and the
// interleaving of dB / dC into complex64 outputs.
cudaError_t launch_cplx_fwd(const CplxParams& p, int dstate, int zoh, cudaStream_t stream);
cudaError_t launch_cplx_bwd(const CplxParams& p, int dstate, int zoh, void* dA, void* dB,
                            void* dC, float* dD, float* ddelta_bias, cudaStream_t stream);

// Fixed-order batch sums of per-batch partials: dA (dim * dstate), dD and
// ddelta_bias (dim); dD / ddelta_bias may be null.
cudaError_t launch_param_reduce(const float* dA_part, const float* dD_part,
                                const float* dbias_part, float* dA, float* dD, float* dbias,
                                int batch, int dim, int dstate, cudaStream_t stream);

cudaError_t launch_step(const StepParams& p, int dstate, int io_dtype, int zoh,
                        cudaStream_t stream);

// Records `msg` as this host thread's mamba_ss_last_error() and returns code.
mss_status set_error(mss_status code, const std::string& msg);

// Returns and clears the forward / backward kernels' device error words.
unsigned int take_fwd_device_error();
unsigned int take_bwd_device_error();

// Debug bounds build: copy and clear the forward / backward compilation
// units' out-of-bounds records ([0] count, [1] site, [2] index, [3] extent;
// all zero without MSS_BOUNDS_CHECK), and launch the checker's self-test.
void take_fwd_bounds(unsigned long long out[4]);
void take_bwd_bounds(unsigned long long out[4]);
cudaError_t launch_bounds_selftest(long long n);

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace mss
