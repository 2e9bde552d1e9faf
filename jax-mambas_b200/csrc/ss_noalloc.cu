// Allocation-free variant of the fused backward (mamba_ss_fused_bwd_noalloc).
//
// The regular backward needs a caller-provided scratch buffer (per-batch
// partial sums of dA, dD and ddelta_bias, plus fp32 accumulators of dB/dC
// for bf16 I/O). Some callers cannot hand one over: code that runs where a
// device allocation is not allowed or not possible (for example inside a
// framework callback that forbids cudaMalloc, or a host runtime that owns
// all device memory and only passes tensor pointers across an FFI). This
// entry point serves them from a fixed scratch array that lives in the
// library's own device image instead.
//
// The array is a file-scope __device__ object of kNoAllocScratchBytes, so
// every GPU on which the library is loaded holds it until the process exits.
// Its address is looked up with cudaGetSymbolAddress the first time the entry
// point runs on a device (with that device current); that first call should
// therefore happen before any stream capture. All calls on a device share the
// one array: calls whose work overlaps on the GPU (different streams, no
// ordering between them) race on it and give wrong results.
#include <mutex>
#include <string>

#include "ss_launch.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" {

size_t mamba_ss_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

mss_status mamba_ss_fused_bwd_noalloc(
    void* stream, int32_t io_dtype, int32_t discretization, int32_t batch,
    int32_t length, int32_t dim, int32_t dstate, const void* u,
    const void* delta, const float* A, const void* B, const void* C,
    const float* D, const void* z, const float* delta_bias,
    int32_t delta_softplus, const float* initial_state, const int32_t* seq_lens,
    const float* chunk_states, const void* out_pre, const void* dout,
    const float* dlast_state, void* du, void* ddelta, float* dA, void* dB,
    void* dC, float* dD, void* dz, float* ddelta_bias, float* dinitial_state) {
  const size_t need = mamba_ss_bwd_workspace_bytes(batch, length, dim, dstate, io_dtype);
  if (need > kNoAllocScratchBytes)
    return mss::set_error(
        MSS_INVALID_ARGUMENT,
        "mamba_ss_fused_bwd_noalloc: this problem needs " + std::to_string(need) +
            " bytes of scratch, more than the fixed " +
            std::to_string(kNoAllocScratchBytes) +
            "; call mamba_ss_fused_bwd with a caller-provided workspace instead");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return mss::set_error(MSS_INTERNAL, "mamba_ss_fused_bwd_noalloc: no usable current device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || !ptr)
        return mss::set_error(MSS_INTERNAL,
                              std::string("mamba_ss_fused_bwd_noalloc: cudaGetSymbolAddress: ") +
                                  cudaGetErrorString(e));
      g_scratch_ptr[dev] = ptr;
    }
    scratch = g_scratch_ptr[dev];
  }
  return mamba_ss_fused_bwd(stream, io_dtype, discretization, batch, length, dim, dstate,
                            u, delta, A, B, C, D, z, delta_bias, delta_softplus,
                            initial_state, seq_lens, chunk_states, out_pre, dout,
                            dlast_state, du, ddelta, dA, dB, dC, dD, dz, ddelta_bias,
                            dinitial_state, scratch, kNoAllocScratchBytes);
}

}  // extern "C"
